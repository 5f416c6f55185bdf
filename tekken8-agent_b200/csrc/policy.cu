// Actor-critic policy and PPO update: the GpuActorCritic contract (include/t8_v2/ppo.hpp:112-193,
// src/ppo.cu) on tcgen05 GEMMs, with its C ABI (include/t8b.h, t8b_policy_*).
//
// Network: observation -> shared tanh layers (hidden_size) -> [query (feature_size), value];
// candidate scores are query . F[table, candidate] / sqrt(feature_size) (the parametric head).
// Master parameters, Adam moments and gradients are fp32 in the reference's canonical order
// (w1, b1, ..., w_out, b_out). Every matrix product runs bf16 x bf16 -> fp32 on the tensor
// cores; the Adam kernel refreshes the bf16 operand copies (row-major and transposed).
//
// Forward: k_forward_tc (normalise, bf16, both tanh layers and the output layer in one kernel,
// for two hidden layers of 512; otherwise k_prep -> GEMM+tanh per hidden layer -> GEMM+bias) ->
// k_sample (scores, masked softmax, sample). Update, per minibatch: k_prep gathers through the
// shuffled permutation -> the same forward GEMMs -> k_loss (scores, clipped objective, entropy,
// value loss, d/d(query, value)) -> backward GEMMs with the tanh derivative and bias column sums
// in the epilogue -> weight-gradient GEMMs reading the row-major activations as MN-major
// operands (samples as K, split-K) -> fixed-order reductions -> gradient norm -> Adam + casts.
#include "forward_tc.cuh"
#include "gemm_host.cuh"
#include "ppo_kernels.cuh"
#include "scorer_tc.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <string>
#include <memory>
#include <numeric>
#include <random>
#include <thread>
#include <vector>

namespace t8b {

using bf16 = __nv_bfloat16;
constexpr int kOutPad = 64;  // output layer width on the tensor cores (query + value + zero padding)

// The tensor-core scorer (ppo::k_loss_tc for the objective, ppo::k_sample_tc for the sampler)
// serves 32-feature tables of at most 368 candidates; other shapes take the SIMT kernels.
bool tensor_core_objective(int feature_size, int action_count) {
    return feature_size == ppo::kFeatures && action_count <= ppo::kTcCandidates && kOutPad == 64;
}

struct Comm {
    t8b_comm_t hooks{};
    bool active() const { return hooks.allreduce_sum_f32 != nullptr && hooks.world_size > 1; }
};

// The reference's weight initialisation (src/ppo.cu:1030-1061, 1083-1121): modified Gram-Schmidt
// with one re-orthogonalisation pass on normal draws in double, or Xavier normal draws.
std::vector<float> orthogonal(int rows, int cols, float gain, std::mt19937_64& random) {
    const size_t tall = static_cast<size_t>(std::max(rows, cols));
    const size_t narrow = static_cast<size_t>(std::min(rows, cols));
    std::normal_distribution<double> normal(0.0, 1.0);
    std::vector<double> basis(tall * narrow);
    for (double& v : basis) v = normal(random);
    for (size_t k = 0; k < narrow; ++k) {
        double* cur = basis.data() + k * tall;
        for (int pass = 0; pass < 2; ++pass) {
            for (size_t j = 0; j < k; ++j) {
                const double* prev = basis.data() + j * tall;
                double dot = 0.0;
                for (size_t i = 0; i < tall; ++i) dot += prev[i] * cur[i];
                for (size_t i = 0; i < tall; ++i) cur[i] -= dot * prev[i];
            }
        }
        double norm = 0.0;
        for (size_t i = 0; i < tall; ++i) norm += cur[i] * cur[i];
        norm = std::sqrt(norm);
        for (size_t i = 0; i < tall; ++i) cur[i] /= norm;
    }
    std::vector<float> out(static_cast<size_t>(rows) * cols);
    for (int r = 0; r < rows; ++r) {
        for (int c = 0; c < cols; ++c) {
            const double v = rows >= cols ? basis[static_cast<size_t>(c) * tall + r] : basis[static_cast<size_t>(r) * tall + c];
            out[static_cast<size_t>(r) * cols + c] = gain * static_cast<float>(v);
        }
    }
    return out;
}

std::vector<float> xavier(int rows, int cols, std::mt19937_64& random, float deviation_override) {
    const float deviation = deviation_override > 0.0f ? deviation_override : std::sqrt(2.0f / static_cast<float>(rows + cols));
    std::normal_distribution<float> normal(0.0f, deviation);
    std::vector<float> out(static_cast<size_t>(rows) * cols);
    for (float& v : out) v = normal(random);
    return out;
}

}  // namespace t8b

using namespace t8b;

namespace t8b {
// [n][cols] fp32 rows into a zero-padded [n][ld] bf16 operand.
__global__ void k_rows_to_bf16(const float* in, size_t n, int cols, bf16* out, int ld) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n * static_cast<size_t>(ld)) return;
    const size_t row = i / static_cast<size_t>(ld);
    const int col = static_cast<int>(i % static_cast<size_t>(ld));
    out[i] = __float2bfloat16_rn(col < cols ? in[row * static_cast<size_t>(cols) + col] : 0.0f);
}
}  // namespace t8b

struct t8b_policy {
    t8b_actor_config_t config{};
    size_t capacity = 0;
    int layers = 0;      // shared hidden layers
    int hidden = 0;
    int width = 0;       // observation floats
    int padded = 0;      // layer-1 operand row (multiple of 64)
    int outputs = 0;     // feature_size + 1
    int feature_size = 0;
    size_t param_count = 0;
    std::vector<size_t> w_off, b_off;  // per layer, then the output layer last
    Buffer<float> params, grads, m1, m2;
    std::vector<Buffer<bf16>> w_bf, wt_bf;  // operand copies per layer (index layers = output)
    // activations
    Buffer<bf16> x;
    std::vector<Buffer<bf16>> h, dz;
    std::vector<Buffer<float>> colsum;
    Buffer<float> out;   // [capacity][64]
    Buffer<bf16> dout;   // [capacity][64]
    Buffer<float> out_colsum;
    Buffer<float> split_part;
    // inference outputs
    Buffer<float> logits, log_probs, values, entropies;
    Buffer<int64_t> actions;
    // minibatch side data
    Buffer<uint32_t> mb_bits, perm, grouped, group_counts;
    Buffer<int32_t> bucket_start;
    Buffer<int32_t> mb_actions, mb_tables;
    Buffer<float> mb_old_lp, mb_old_v, mb_adv, mb_ret;
    Buffer<double> block_metrics, metrics, norm_partial, norm_sq, entropy_sums;
    Buffer<uint4> table_images;  // the tensor-core scorer's per-table shared-memory images
    Buffer<float> sample_entropy;
    Buffer<uint8_t> sample_decision;
    Buffer<int> error, invalid;
    Buffer<double> kl_pair, obs_gathered;
    // features
    Buffer<float> features;
    int tables = 0;
    bool features_ready = false;
    // observation normaliser
    Buffer<float> obs_mean, obs_var, obs_istd;
    Buffer<double> obs_chunks;
    uint64_t obs_count = 0;
    uint64_t optimizer_step = 0;
    ppo::AdamSpec adam{};
    Comm comm;
    // prepared permutations
    std::thread shuffler;
    std::vector<std::vector<uint32_t>> prepared;
    size_t prepared_samples = 0;
    int prepared_epochs = 0;
    uint64_t prepared_seed = 0;
    bool prepared_valid = false;

    ~t8b_policy() {
        if (shuffler.joinable()) shuffler.join();
    }
    bool normalizing() const { return config.observation_normalization && obs_count > 0; }
    int bn_hidden() const { return hidden % 256 == 0 ? 256 : 64; }

    void refresh_operands(cudaStream_t stream) {
        launch("k_adam", ppo::k_adam, blocks(param_count, 256), 256, 0, stream, params.data(), grads.data(), m1.data(), m2.data(),
                                                                  param_count, norm_sq.data(), 1.0f, 0.0f, 0.9f, 0.999f,
                                                                  1e-5f, 1.0f, 1.0f, adam, 0);
        check(cudaGetLastError(), "refresh operand copies");
    }

    template <int BN, class Epi>
    void dense(const char* label, const Operand& a, const Operand& b, Epi epi, cudaStream_t stream, int splits = 1) {
        gemm<BN, false, false>(label, a, b, splits, error.data(), epi, stream);
    }

    // forward of the network on x[0..n) -> out [n][64]
    // rows [row, row + n) of the activation buffers: two row ranges can run on two streams at once
    void network(size_t n, cudaStream_t stream, size_t row = 0) {
        const int m = static_cast<int>(n);
        bf16* x0 = x.data() + row * static_cast<size_t>(padded);
        for (int l = 0; l < layers; ++l) {
            bf16* below = l == 0 ? x0 : h[l - 1].data() + row * static_cast<size_t>(hidden);
            const Operand a = l == 0 ? Operand{below, m, padded, padded, false} : Operand{below, m, hidden, hidden, false};
            const Operand b{w_bf[l].data(), hidden, a.k, a.k, false};
            const ppo::EpiTanh epi{params.data() + b_off[l],
                                   make_store_map(h[l].data() + row * static_cast<size_t>(hidden), hidden, m, hidden), hidden,
                                   m, hidden};
            if (bn_hidden() == 256) dense<256>("gemm_forward_hidden", a, b, epi, stream); else dense<64>("gemm_forward_hidden", a, b, epi, stream);
        }
        const Operand a{h[layers - 1].data() + row * static_cast<size_t>(hidden), m, hidden, hidden, false};
        const Operand b{w_bf[layers].data(), kOutPad, hidden, hidden, false};
        dense<64>("gemm_forward_output", a, b,
                  ppo::EpiBias{params.data() + b_off[layers], out.data() + row * static_cast<size_t>(kOutPad), kOutPad, m, outputs},
                  stream);
    }

    // The inference forward as one kernel (ppo::k_forward_tc): two hidden layers of 512, at most
    // 512 padded inputs and 64 outputs; bit-identical to k_prep + network().
    bool fused_forward() const {
        return layers == 2 && hidden == ppo::kFwHidden && padded <= ppo::kFwHidden && outputs <= kOutPad;
    }
    void forward_fused(size_t row, size_t n, const float* obs, cudaStream_t st) {
        const CUtensorMap m1 = make_map(w_bf[0].data(), padded, hidden, padded, 64, 256);
        const CUtensorMap m2 = make_map(w_bf[1].data(), hidden, hidden, hidden, 64, 256);
        const CUtensorMap mo = make_map(w_bf[2].data(), hidden, kOutPad, hidden, 64, 64);
        ppo::Forward f{};
        f.obs = obs + row * static_cast<size_t>(width);
        f.width = width;
        f.in_blocks = padded / 64;
        f.mean = obs_mean.data();
        f.istd = obs_istd.data();
        f.clip = config.observation_clip;
        f.normalize = normalizing() ? 1 : 0;
        f.b1 = params.data() + b_off[0];
        f.b2 = params.data() + b_off[1];
        f.b_out = params.data() + b_off[2];
        f.outputs = outputs;
        f.out = out.data() + row * static_cast<size_t>(kOutPad);
        f.n = static_cast<int>(n);
        f.error = error.data();
        check(cudaFuncSetAttribute(ppo::k_forward_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, ppo::kFwSmemBytes),
              "forward smem");
        const int tiles = static_cast<int>((n + ppo::kFwRows - 1) / ppo::kFwRows);
        launch("k_forward_tc", ppo::k_forward_tc, std::min(tiles, sm_count()), ppo::kFwThreads, ppo::kFwSmemBytes, st, m1, m2,
               mo, f);
        check(cudaGetLastError(), "fused forward");
    }

    // k_prep then the layer GEMMs: the forward of the shapes the fused kernel does not serve.
    void forward_network(size_t row, size_t n, const float* obs, cudaStream_t st) {
        ppo::Prep prep{};
        prep.obs = obs + row * static_cast<size_t>(width);
        prep.width = width;
        prep.padded = padded;
        prep.mean = obs_mean.data();
        prep.istd = obs_istd.data();
        prep.clip = config.observation_clip;
        prep.normalize = normalizing() ? 1 : 0;
        prep.count = n;
        prep.x = x.data() + row * static_cast<size_t>(padded);
        launch("k_prep", ppo::k_prep, blocks(n, ppo::kWarps), 32 * ppo::kWarps, 0, st, prep);
        check(cudaGetLastError(), "prepare inputs");
        network(n, st, row);
    }

    // forward's work on rows [row, row + n) of a batch: the inputs are the batch's base pointers
    // (observations [batch][width], packed masks [batch][12] or uint8 masks [batch][action_count],
    // tables [batch]) and the outputs land in rows [row, row + n) of the inference buffers; the
    // sampler's uniforms are keyed by the row in the batch, so a batch forwarded in row ranges
    // samples exactly as a whole one.
    void forward_rows(size_t row, size_t n, const float* obs, const uint8_t* masks, const uint32_t* mask_bits,
                      const int32_t* tables, uint64_t seed, uint64_t step, int deterministic, bool want_logits,
                      cudaStream_t st, cudaEvent_t masks_ready = nullptr) {
        if (!features_ready) raise(T8B_ESTATE, "parametric policy action features have not been installed");
        if (row + n > capacity) raise(T8B_EINVAL, "forward rows exceed the policy capacity");
        if (fused_forward()) {
            forward_fused(row, n, obs, st);
        } else {
            forward_network(row, n, obs, st);
        }
        if (masks_ready != nullptr) check(cudaStreamWaitEvent(st, masks_ready, 0), "wait for the masks");
        ppo::Sample smp{};
        smp.out = out.data() + row * static_cast<size_t>(kOutPad);
        smp.ld = kOutPad;
        smp.feature_size = feature_size;
        smp.action_count = config.action_count;
        smp.features = features.data();
        smp.table_count = this->tables;
        smp.tables = tables ? tables + row : nullptr;
        smp.bits = mask_bits ? mask_bits + row * 12 : nullptr;
        smp.bytes = mask_bits ? nullptr : masks + row * static_cast<size_t>(config.action_count);
        smp.count = n;
        smp.seed = seed;
        smp.step = step;
        smp.lane_offset = row;
        smp.deterministic = deterministic;
        smp.logits = want_logits ? logits.data() + row * static_cast<size_t>(config.action_count) : nullptr;
        smp.actions = actions.data() + row;
        smp.log_probs = log_probs.data() + row;
        smp.values = values.data() + row;
        smp.entropies = entropies.data() + row;
        // one group per feature table (plus one for out-of-range table indices), each split into
        // parts so that the grid fills one wave of two blocks per SM (at most 256 samples a block
        // beyond that): at 32,768 samples over 42 groups, 7 parts (294 blocks) measured 12 %
        // faster than 13 parts of about 64 samples (546 blocks, 1.8 waves)
        const size_t groups = tables ? static_cast<size_t>(this->tables) + 1 : 1;
        if (tensor_core_objective(feature_size, config.action_count)) {
            // one wave of one CTA per SM: (groups x parts) CTAs
            const int parts = std::max(1, static_cast<int>(static_cast<size_t>(sm_count()) / groups));
            launch("k_sample", ppo::k_sample_tc, static_cast<unsigned>(groups * parts), ppo::kTcThreads, ppo::kTsSmemBytes, st,
                   smp, static_cast<const uint4*>(table_images.data()), parts, error.data());
            check(cudaGetLastError(), "sample actions");
            return;
        }
        const size_t wave = static_cast<size_t>(2 * sm_count()) / groups;
        smp.parts = static_cast<unsigned>(std::min<size_t>(std::max<size_t>({(n + groups * 256 - 1) / (groups * 256), wave, 1}), 4096));
        const unsigned sample_grid = static_cast<unsigned>(groups * smp.parts);
        const size_t sample_bytes = ppo::sample_smem(feature_size);
        if (feature_size == 48) {
            launch("k_sample", ppo::k_sample<48>, sample_grid, 32 * ppo::kSampleWarps, sample_bytes, st, smp);
        } else {
            launch("k_sample", ppo::k_sample<32>, sample_grid, 32 * ppo::kSampleWarps, sample_bytes, st, smp);
        }
        check(cudaGetLastError(), "sample actions");
    }

    int splits_for(int tiles) const {
        const int s = sm_count() / std::max(1, tiles);
        return std::max(1, s);
    }

    // backward from dout [n][64] into grads (unclipped, averaged by the loss scaling)
    void backward(size_t n, cudaStream_t stream) {
        const int m = static_cast<int>(n);
        const int tiles_rows = (m + tc::BM - 1) / tc::BM;
        // output layer weight gradient: dW_out^T [hidden][64] = H_L^T . dO
        {
            const Operand a{h[layers - 1].data(), hidden, m, hidden, true};
            const Operand b{dout.data(), kOutPad, m, kOutPad, true};
            const int splits = splits_for(hidden / tc::BM);
            gemm<64, true, true>("gemm_weight_grad", a, b, splits, error.data(), ppo::EpiSplit{split_part.data(), hidden, kOutPad}, stream);
            const int k_blocks = (m + tc::BK - 1) / tc::BK;
            const int used = std::min(splits, k_blocks);
            launch("k_reduce_split", ppo::k_reduce_split, blocks(static_cast<size_t>(outputs) * hidden, 256), 256, 0, stream, 
                split_part.data(), used, hidden, kOutPad, grads.data() + w_off[layers], outputs, hidden, 1);
        }
        // output layer input gradient through tanh of the top hidden layer
        {
            const Operand a{dout.data(), m, kOutPad, kOutPad, false};
            const Operand b{wt_bf[layers].data(), hidden, kOutPad, kOutPad, false};
            const ppo::EpiTanhGrad epi{h[layers - 1].data(), make_store_map(dz[layers - 1].data(), hidden, m, hidden),
                                       colsum[layers - 1].data(), hidden, m};
            if (bn_hidden() == 256) dense<256>("gemm_input_grad", a, b, epi, stream); else dense<64>("gemm_input_grad", a, b, epi, stream);
        }
        for (int l = layers - 1; l >= 0; --l) {
            column_sums(colsum[l].data(), tiles_rows * 4, hidden, hidden, grads.data() + b_off[l], stream);
            // weight gradient dW_l [hidden][in] = dZ_l^T . A_{l-1}
            const int in_rows = l == 0 ? padded : hidden;
            const bf16* in = l == 0 ? x.data() : h[l - 1].data();
            const Operand a{dz[l].data(), hidden, m, hidden, true};
            const Operand b{in, in_rows, m, in_rows, true};
            const int k_blocks = (m + tc::BK - 1) / tc::BK;
            if (l == 0 && padded % 256 != 0) {
                const int tiles = (hidden / tc::BM) * ((in_rows + 191) / 192);
                const int splits = splits_for(tiles);
                if (padded == 192) {
                    gemm<192, true, true>("gemm_weight_grad", a, b, splits, error.data(), ppo::EpiSplit{split_part.data(), hidden, in_rows}, stream);
                } else {
                    gemm<64, true, true>("gemm_weight_grad", a, b, splits, error.data(), ppo::EpiSplit{split_part.data(), hidden, in_rows}, stream);
                }
                launch("k_reduce_split", ppo::k_reduce_split, blocks(static_cast<size_t>(hidden) * width, 256), 256, 0, stream, 
                    split_part.data(), std::min(splits, k_blocks), hidden, in_rows, grads.data() + w_off[0], hidden, width, 0);
            } else {
                const int tiles = (hidden / tc::BM) * (in_rows / 256);
                const int splits = splits_for(tiles);
                gemm<256, true, true>("gemm_weight_grad", a, b, splits, error.data(), ppo::EpiSplit{split_part.data(), hidden, in_rows}, stream);
                const int cols = l == 0 ? width : hidden;
                launch("k_reduce_split", ppo::k_reduce_split, blocks(static_cast<size_t>(hidden) * cols, 256), 256, 0, stream, 
                    split_part.data(), std::min(splits, k_blocks), hidden, in_rows, grads.data() + w_off[l], hidden, cols, 0);
            }
            if (l > 0) {
                // dZ_{l-1} = (dZ_l . W_l) * (1 - H_{l-1}^2)
                const Operand da{dz[l].data(), m, hidden, hidden, false};
                const Operand db{wt_bf[l].data(), hidden, hidden, hidden, false};
                const ppo::EpiTanhGrad epi{h[l - 1].data(), make_store_map(dz[l - 1].data(), hidden, m, hidden),
                                           colsum[l - 1].data(), hidden, m};
                if (bn_hidden() == 256) dense<256>("gemm_input_grad", da, db, epi, stream); else dense<64>("gemm_input_grad", da, db, epi, stream);
            }
        }
        check(cudaGetLastError(), "backward");
    }

    Buffer<float> column_scratch;
    // grad[c] = sum over rows of in[r][c], two fixed-order levels
    void column_sums(const float* in, int rows, int ld, int cols, float* grad, cudaStream_t stream) {
        const size_t need = static_cast<size_t>(ppo::kColumnChunks) * cols;
        if (column_scratch.size() < need) column_scratch.allocate(std::max<size_t>(need, ppo::kColumnChunks * 1024));
        dim3 grid((cols + 31) / 32, ppo::kColumnChunks);
        launch("k_column_partials", ppo::k_column_partials, grid, dim3(32, 8), 0, stream, in, rows, ld, cols, column_scratch.data());
        launch("k_reduce_columns", ppo::k_reduce_columns, blocks(cols, 128), 128, 0, stream, column_scratch.data(), ppo::kColumnChunks, cols, cols, grad);
        check(cudaGetLastError(), "column sums");
    }

    // The flag is set by any tensor-core kernel whose bounded wait ran out (the GEMMs, the
    // scorer kernels of the forward and of the update) and stays set until a check reports it,
    // so a forward's stall surfaces at the next update or synchronisation.
    void sync_error(cudaStream_t stream) {
        int flag = 0;
        error.download(&flag, 1, stream);
        if (flag) {
            error.zero(stream);
            raise(T8B_ECUDA, "a tensor-core kernel stalled and was aborted");
        }
    }
};

namespace {

template <typename Body>
int with_policy(t8b_policy* p, Body&& body) {
    return guarded([&] {
        if (p == nullptr) raise(T8B_EINVAL, "null policy handle");
        body(*p);
    });
}

// The host permutations of update_ppo (src/ppo.cu:1570-1579): one std::shuffle per epoch with
// a std::mt19937_64 seeded by the shuffle seed.
std::vector<std::vector<uint32_t>> make_permutations(size_t count, int epochs, uint64_t seed) {
    std::mt19937_64 random(seed);
    std::vector<uint32_t> order(count);
    std::iota(order.begin(), order.end(), 0u);
    std::vector<std::vector<uint32_t>> out;
    for (int e = 0; e < epochs; ++e) {
        std::shuffle(order.begin(), order.end(), random);
        out.push_back(order);
    }
    return out;
}

// decision_flags_kernel + deterministic_decision_entropy_kernel (src/ppo.cu:570-610), multi-block:
// per-block fp64 (entropy sum, decision count) in index order, then a fixed-order total.
__global__ void k_decision_partials(const float* entropy, const uint8_t* decision, const uint8_t* bytes,
                                    const uint32_t* bits, int actions_per_sample, size_t n, double* partial) {
    __shared__ double se[256], sd[256];
    double e = 0.0, d = 0.0;
    for (size_t s = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; s < n;
         s += static_cast<size_t>(gridDim.x) * blockDim.x) {
        bool choice;
        if (decision) {
            choice = decision[s] != 0;
        } else {
            int legal = 0;
            for (int w = 0; w < 12 && legal < 2; ++w) {
                if (bits) {
                    legal += __popc(bits[s * 12 + w]);
                } else {
                    for (int b = 0; b < 32 && w * 32 + b < actions_per_sample; ++b) {
                        legal += bytes[s * actions_per_sample + w * 32 + b] != 0;
                    }
                }
            }
            choice = legal > 1;
        }
        if (choice) {
            e += entropy[s];
            d += 1.0;
        }
    }
    se[threadIdx.x] = e;
    sd[threadIdx.x] = d;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            se[threadIdx.x] += se[threadIdx.x + w];
            sd[threadIdx.x] += sd[threadIdx.x + w];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        partial[2 * blockIdx.x] = se[0];
        partial[2 * blockIdx.x + 1] = sd[0];
    }
}

__global__ void k_decision_finish(const double* partial, int blocks, double* out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    double e = 0.0, d = 0.0;
    for (int b = 0; b < blocks; ++b) {
        e += partial[2 * b];
        d += partial[2 * b + 1];
    }
    out[0] = e;
    out[1] = d;
}

// Grid of k_loss for a minibatch of n rows: one block per run of at most kLossRows rows of one
// feature table; the runs of the kBuckets tables add at most one partial run each.
size_t loss_blocks(size_t n) { return (n + ppo::kLossRows - 1) / ppo::kLossRows + ppo::kBuckets; }


// Reorders every minibatch slice of the epoch permutation (s.perm) by feature table into
// s.grouped and records each slice's table offsets in s.bucket_start.
void group_minibatches(t8b_policy& s, const t8b_rollout_view_t& r, size_t samples, size_t minibatch, cudaStream_t st) {
    const size_t slices = (samples + minibatch - 1) / minibatch;
    const int per_slice = static_cast<int>((minibatch + ppo::kGroupRows - 1) / ppo::kGroupRows);
    const size_t grid = slices * static_cast<size_t>(per_slice);
    if (s.group_counts.size() < grid * ppo::kBuckets) s.group_counts.allocate(grid * ppo::kBuckets);
    if (s.bucket_start.size() < slices * (ppo::kBuckets + 1)) s.bucket_start.allocate(slices * (ppo::kBuckets + 1));
    ppo::Group g{};
    g.perm = s.perm.data();
    g.tables = r.feature_tables;
    g.table_count = s.tables;
    g.samples = samples;
    g.minibatch = minibatch;
    g.blocks_per_slice = per_slice;
    g.counts = s.group_counts.data();
    g.sorted = s.grouped.data();
    g.bucket_start = s.bucket_start.data();
    launch("k_group_count", ppo::k_group_count, static_cast<unsigned>(grid), 256, 0, st, g);
    launch("k_group_offsets", ppo::k_group_offsets, static_cast<unsigned>(slices), 64, 0, st, g);
    launch("k_group_scatter", ppo::k_group_scatter, static_cast<unsigned>(grid), 256, 0, st, g);
    check(cudaGetLastError(), "group minibatches by feature table");
}

}  // namespace

extern "C" {

void t8b_actor_config_default(t8b_actor_config_t* c) {
    std::memset(c, 0, sizeof *c);
    c->observation_size = 151;
    c->action_count = T8B_MAX_CANDIDATES;
    c->hidden_size = 512;
    c->action_feature_size = T8B_FEATURE_SIZE;
    c->universal_action_count = T8B_UNIVERSAL_COUNT;
    c->shared_layers = 2;
    c->head_layers = 0;
    c->observation_normalization = 1;
    c->orthogonal_initialization = 1;
    c->observation_clip = 10.0f;
    c->observation_epsilon = 1e-8f;
    c->matmul_precision = 2;
}

void t8b_ppo_config_default(t8b_ppo_config_t* c) {
    std::memset(c, 0, sizeof *c);
    c->epochs = 4;
    c->minibatch_size = 4096;
    c->learning_rate = 3e-4f;
    c->clip_range = 0.2f;
    c->value_clip_range = 0.2f;
    c->target_kl = 0.02f;
    c->value_coefficient = 0.5f;
    c->entropy_coefficient = 0.01f;
    c->max_gradient_norm = 0.5f;
    c->adam_beta1 = 0.9f;
    c->adam_beta2 = 0.999f;
    c->adam_epsilon = 1e-5f;
}

int t8b_policy_create(size_t capacity, const t8b_actor_config_t* config, uint64_t seed, t8b_policy** out) {
    return guarded([&] {
        if (out == nullptr || config == nullptr) raise(T8B_EINVAL, "null argument");
        *out = nullptr;
        const t8b_actor_config_t& c = *config;
        // validate_actor_config (src/ppo.cu:26-45), restricted to the parametric full-move head
        if (capacity == 0 || capacity > (1ull << 31)) raise(T8B_EINVAL, "policy capacity must be positive and fit 32-bit rows");
        if (c.observation_size <= 0 || c.action_count <= 1 || c.hidden_size <= 0) {
            raise(T8B_EINVAL, "actor-critic dimensions must be positive and representable");
        }
        if (c.shared_layers < 1 || c.shared_layers > 8 || c.head_layers < 0 || c.head_layers > 6) {
            raise(T8B_EINVAL, "actor-critic depth must be 1-8 shared layers and 0-6 head layers");
        }
        if (c.head_layers != 0) raise(T8B_EINVAL, "separate policy/value heads are not supported by this library");
        if ((c.action_feature_size != 32 && c.action_feature_size != 48) || c.action_count > T8B_MAX_CANDIDATES) {
            raise(T8B_EINVAL, "this library implements the parametric head with 32 or 48 features and at most 368 candidates");
        }
        if (c.hidden_size % 64 != 0 || c.hidden_size % tc::BM != 0) raise(T8B_EINVAL, "hidden_size must be a multiple of 128");
        if (!std::isfinite(c.observation_clip) || c.observation_clip <= 0.0f || !std::isfinite(c.observation_epsilon) ||
            c.observation_epsilon <= 0.0f) {
            raise(T8B_EINVAL, "observation normalizer clip/epsilon must be finite and positive");
        }
        auto p = std::make_unique<t8b_policy>();
        p->config = c;
        p->capacity = capacity;
        p->layers = c.shared_layers;
        p->hidden = c.hidden_size;
        p->width = c.observation_size;
        p->padded = (c.observation_size + 63) / 64 * 64;
        p->feature_size = c.action_feature_size;
        p->outputs = c.action_feature_size + 1;
        // canonical order: w1, b1, ..., w_out, b_out
        size_t off = 0;
        for (int l = 0; l < p->layers; ++l) {
            const int in = l == 0 ? p->width : p->hidden;
            p->w_off.push_back(off);
            off += static_cast<size_t>(p->hidden) * in;
            p->b_off.push_back(off);
            off += p->hidden;
        }
        p->w_off.push_back(off);
        off += static_cast<size_t>(p->outputs) * p->hidden;
        p->b_off.push_back(off);
        off += p->outputs;
        p->param_count = off;
        p->params.allocate(off);
        p->grads.allocate(off);
        p->m1.allocate(off);
        p->m2.allocate(off);
        // bf16 operand copies
        for (int l = 0; l <= p->layers; ++l) {
            Buffer<bf16> w, wt;
            if (l < p->layers) {
                const int in = l == 0 ? p->padded : p->hidden;
                w.allocate(static_cast<size_t>(p->hidden) * in);
                if (l > 0) wt.allocate(static_cast<size_t>(p->hidden) * p->hidden);
            } else {
                w.allocate(static_cast<size_t>(kOutPad) * p->hidden);
                wt.allocate(static_cast<size_t>(p->hidden) * kOutPad);
            }
            p->w_bf.push_back(std::move(w));
            p->wt_bf.push_back(std::move(wt));
        }
        int t = 0;
        for (int l = 0; l <= p->layers; ++l) {
            const bool top = l == p->layers;
            const int rows = top ? p->outputs : p->hidden;
            const int cols = l == 0 ? p->width : p->hidden;
            ppo::TensorSpec w{p->w_off[l], rows, cols, p->w_bf[l].data(), l == 0 ? p->padded : p->hidden,
                              p->wt_bf[l].size() ? p->wt_bf[l].data() : nullptr, top ? kOutPad : p->hidden};
            ppo::TensorSpec b{p->b_off[l], 1, rows, nullptr, 0, nullptr, 0};
            p->adam.t[t++] = w;
            p->adam.t[t++] = b;
        }
        p->adam.count = t;
        // activations
        const size_t cap = capacity;
        p->x.allocate(cap * p->padded);
        const size_t row_tiles = (cap + tc::BM - 1) / tc::BM;
        for (int l = 0; l < p->layers; ++l) {
            p->h.emplace_back(cap * p->hidden);
            p->dz.emplace_back(cap * p->hidden);
            p->colsum.emplace_back(row_tiles * 4 * p->hidden);
        }
        p->out.allocate(cap * kOutPad);
        p->dout.allocate(cap * kOutPad);
        const size_t partial_rows = std::max({(cap + ppo::kWarps - 1) / ppo::kWarps, loss_blocks(cap), ppo::tc_tiles(cap)});
        p->out_colsum.allocate(partial_rows * kOutPad);
        check(cudaFuncSetAttribute(ppo::k_loss<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, ppo::kMaxTableBytes),
              "objective shared memory");
        check(cudaFuncSetAttribute(ppo::k_loss<48>, cudaFuncAttributeMaxDynamicSharedMemorySize, ppo::kMaxTableBytes),
              "objective shared memory");
        check(cudaFuncSetAttribute(ppo::k_loss_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, ppo::kTcSmemBytes),
              "objective shared memory");
        check(cudaFuncSetAttribute(ppo::k_sample_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, ppo::kTsSmemBytes),
              "sampler shared memory");
        check(cudaFuncSetAttribute(ppo::k_sample<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(ppo::sample_smem(32))), "sampler shared memory");
        check(cudaFuncSetAttribute(ppo::k_sample<48>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(ppo::sample_smem(48))), "sampler shared memory");
        const size_t sms = static_cast<size_t>(sm_count());
        const size_t part = std::max({sms * p->hidden * kOutPad, sms * static_cast<size_t>(p->hidden) * p->hidden,
                                      sms * static_cast<size_t>(p->hidden) * p->padded});
        p->split_part.allocate(part);
        p->logits.allocate(cap * static_cast<size_t>(c.action_count));
        p->log_probs.allocate(cap);
        p->values.allocate(cap);
        p->entropies.allocate(cap);
        p->actions.allocate(cap);
        p->mb_bits.allocate(cap * 12);
        p->mb_actions.allocate(cap);
        p->mb_tables.allocate(cap);
        p->mb_old_lp.allocate(cap);
        p->mb_old_v.allocate(cap);
        p->mb_adv.allocate(cap);
        p->mb_ret.allocate(cap);
        p->block_metrics.allocate(partial_rows * ppo::kMetrics);
        p->metrics.allocate(ppo::kMetrics);
        p->norm_partial.allocate(1024);
        p->norm_sq.allocate(1);
        p->entropy_sums.allocate(2 * 1024 + 2);
        p->error.allocate(1);
        p->invalid.allocate(1);
        p->kl_pair.allocate(2);
        p->obs_mean.allocate(p->width);
        p->obs_var.allocate(p->width);
        p->obs_istd.allocate(p->width);
        const std::vector<float> zeros(p->width, 0.0f), ones(p->width, 1.0f);
        p->obs_mean.upload(zeros.data(), p->width, nullptr);
        p->obs_var.upload(ones.data(), p->width, nullptr);
        launch("k_refresh_istd", ppo::k_refresh_istd, blocks(p->width, 128), 128, 0, nullptr, p->obs_var.data(), p->obs_istd.data(), p->width,
                                                           c.observation_epsilon);
        // initial weights: hidden layers, then the output layer, from one mt19937_64(seed)
        std::mt19937_64 random(seed);
        std::vector<float> host(p->param_count, 0.0f);
        for (int l = 0; l < p->layers; ++l) {
            const int in = l == 0 ? p->width : p->hidden;
            const auto w = c.orthogonal_initialization ? orthogonal(p->hidden, in, std::sqrt(2.0f), random)
                                                       : xavier(p->hidden, in, random, 0.0f);
            std::copy(w.begin(), w.end(), host.begin() + static_cast<std::ptrdiff_t>(p->w_off[l]));
        }
        if (c.orthogonal_initialization) {
            auto w = orthogonal(p->outputs, p->hidden, 1.0f, random);
            for (int r = 0; r + 1 < p->outputs; ++r) {
                for (int col = 0; col < p->hidden; ++col) w[static_cast<size_t>(r) * p->hidden + col] *= 0.01f;
            }
            std::copy(w.begin(), w.end(), host.begin() + static_cast<std::ptrdiff_t>(p->w_off[p->layers]));
        } else {
            const auto w = xavier(p->outputs, p->hidden, random, 0.01f);
            std::copy(w.begin(), w.end(), host.begin() + static_cast<std::ptrdiff_t>(p->w_off[p->layers]));
        }
        p->params.upload(host.data(), host.size(), nullptr);
        p->refresh_operands(nullptr);
        check(cudaStreamSynchronize(nullptr), "create policy");
        *out = p.release();
    });
}

int t8b_policy_destroy(t8b_policy* p) {
    return guarded([&] {
        if (p != nullptr) cudaDeviceSynchronize();
        delete p;
    });
}

size_t t8b_policy_capacity(const t8b_policy* p) { return p ? p->capacity : 0; }
size_t t8b_policy_parameter_count(const t8b_policy* p) { return p ? p->param_count : 0; }
int t8b_policy_action_feature_tables(const t8b_policy* p) { return p ? p->tables : 0; }

int t8b_policy_set_action_feature_tables(t8b_policy* p, const float* features, int tables, void* stream) {
    return with_policy(p, [&](t8b_policy& s) {
        if (tables <= 0) raise(T8B_EINVAL, "at least one action feature table is required");
        const size_t count = static_cast<size_t>(tables) * s.config.action_count * s.feature_size;
        for (size_t i = 0; i < count; ++i) {
            if (!std::isfinite(features[i])) raise(T8B_EINVAL, "parametric action feature tensor has non-finite values");
        }
        if (s.features.size() != count) s.features.allocate(count);
        s.features.upload(features, count, static_cast<cudaStream_t>(stream));
        if (tensor_core_objective(s.feature_size, s.config.action_count)) {
            const size_t chunks = static_cast<size_t>(tables) * ppo::kTcImageChunks;
            if (s.table_images.size() != chunks) s.table_images.allocate(chunks);
            const dim3 grid((ppo::kTcCandidates * 8 + 32 * 96 + 255) / 256, static_cast<unsigned>(tables));
            launch("k_table_images", ppo::k_table_images, grid, 256, 0, static_cast<cudaStream_t>(stream), s.features.data(),
                   s.config.action_count, tables, s.table_images.data());
            check(cudaGetLastError(), "feature table images");
        }
        check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "upload features");
        s.tables = tables;
        s.features_ready = true;
    });
}

}  // extern "C"

namespace t8b::internal {

void policy_forward_rows(t8b_policy* p, size_t row, size_t n, const float* observations, const uint32_t* mask_bits,
                         const int32_t* tables, uint64_t seed, uint64_t step, int deterministic, cudaStream_t stream,
                         t8b_policy_output_t* out, cudaEvent_t masks_ready) {
    if (observations == nullptr || mask_bits == nullptr || n == 0) raise(T8B_EINVAL, "policy input pointers cannot be null");
    p->forward_rows(row, n, observations, nullptr, mask_bits, tables, seed, step, deterministic, false, stream, masks_ready);
    out->logits = nullptr;
    out->actions = p->actions.data();
    out->log_probabilities = p->log_probs.data();
    out->values = p->values.data();
    out->entropies = p->entropies.data();
    out->environment_count = row + n;
}

}  // namespace t8b::internal

extern "C" {

int t8b_policy_forward(t8b_policy* p, const float* obs, const uint8_t* masks, const uint32_t* mask_bits, size_t n,
                       uint64_t seed, uint64_t step, int deterministic, void* stream, const int32_t* tables,
                       int want_logits, t8b_policy_output_t* out) {
    return with_policy(p, [&](t8b_policy& s) {
        if (obs == nullptr || (masks == nullptr && mask_bits == nullptr)) raise(T8B_EINVAL, "policy input pointers cannot be null");
        if (n == 0 || n > s.capacity) raise(T8B_EINVAL, "environment_count exceeds policy capacity");
        s.forward_rows(0, n, obs, masks, mask_bits, tables, seed, step, deterministic, want_logits != 0,
                       static_cast<cudaStream_t>(stream));
        if (out) {
            out->logits = want_logits ? s.logits.data() : nullptr;
            out->actions = s.actions.data();
            out->log_probabilities = s.log_probs.data();
            out->values = s.values.data();
            out->entropies = s.entropies.data();
            out->environment_count = n;
        }
    });
}

int t8b_policy_prepare_shuffle(t8b_policy* p, size_t sample_count, int epochs, uint64_t shuffle_seed) {
    return with_policy(p, [&](t8b_policy& s) {
        if (s.shuffler.joinable()) s.shuffler.join();
        s.prepared_valid = false;
        s.prepared_samples = sample_count;
        s.prepared_epochs = epochs;
        s.prepared_seed = shuffle_seed;
        s.shuffler = std::thread([&s, sample_count, epochs, shuffle_seed] {
            s.prepared = make_permutations(sample_count, epochs, shuffle_seed);
        });
        s.prepared_valid = true;
    });
}

int t8b_policy_set_comm(t8b_policy* p, const t8b_comm_t* comm) {
    return with_policy(p, [&](t8b_policy& s) { s.comm.hooks = comm ? *comm : t8b_comm_t{}; });
}

int t8b_policy_update_ppo(t8b_policy* p, const t8b_rollout_view_t* view, const t8b_ppo_config_t* cfg, uint64_t shuffle_seed,
                          void* stream, t8b_ppo_metrics_t* metrics_out) {
    return with_policy(p, [&](t8b_policy& s) {
        if (view == nullptr || cfg == nullptr) raise(T8B_EINVAL, "null argument");
        const t8b_rollout_view_t& r = *view;
        if (r.sample_count == 0 || !r.observations || (!r.action_masks && !r.action_mask_bits) || !r.actions ||
            !r.old_log_probabilities || !r.old_values || !r.advantages || !r.returns) {
            raise(T8B_EINVAL, "rollout view is incomplete");
        }
        if (cfg->epochs <= 0 || cfg->minibatch_size == 0 || cfg->minibatch_size > s.capacity) {
            raise(T8B_EINVAL, "PPO epochs/minibatch size are invalid for policy capacity");
        }
        const float coefficients[] = {cfg->learning_rate, cfg->clip_range, cfg->value_clip_range, cfg->target_kl,
                                      cfg->value_coefficient, cfg->entropy_coefficient, cfg->max_gradient_norm,
                                      cfg->adam_beta1, cfg->adam_beta2, cfg->adam_epsilon};
        bool finite = true;
        for (float v : coefficients) finite = finite && std::isfinite(v);
        if (!finite || cfg->learning_rate <= 0.0f || cfg->clip_range < 0.0f || cfg->value_clip_range < 0.0f ||
            cfg->target_kl < 0.0f || cfg->value_coefficient < 0.0f || cfg->entropy_coefficient < 0.0f ||
            cfg->max_gradient_norm <= 0.0f || cfg->adam_beta1 < 0.0f || cfg->adam_beta1 >= 1.0f ||
            cfg->adam_beta2 < 0.0f || cfg->adam_beta2 >= 1.0f || cfg->adam_epsilon <= 0.0f) {
            raise(T8B_EINVAL, "PPO optimizer coefficients are invalid or non-finite");
        }
        if (!s.features_ready) raise(T8B_ESTATE, "parametric policy action features have not been installed");
        if (r.sample_count > 0xffffffffull) raise(T8B_EINVAL, "rollout too large for 32-bit sample indices");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const size_t samples = r.sample_count;
        // validate_rollout_kernel (src/ppo.cu:423-451, 1545-1559), with the batch moments of the
        // observations for the normaliser taken in the same pass (merged after the update)
        // chunks of 1,024-8,192 samples: enough blocks for a single minibatch, few chunks to merge
        // for a whole rollout (the merge walks the chunks in order)
        const size_t chunk = std::min<size_t>(8192, std::max<size_t>(1024, (samples / 512 + 7) / 8 * 8));
        const size_t chunks = (samples + chunk - 1) / chunk;
        const bool normalizing = s.config.observation_normalization;
        if (normalizing && s.obs_chunks.size() < chunks * s.width * 3) s.obs_chunks.allocate(chunks * s.width * 3);
        s.invalid.zero(st);
        ppo::Scan scan{};
        scan.obs = r.observations;
        scan.width = s.width;
        scan.samples = samples;
        scan.chunk = chunk;
        scan.moments = normalizing ? s.obs_chunks.data() : nullptr;
        scan.bytes = r.action_masks;
        scan.bits = r.action_mask_bits;
        scan.actions_per_sample = s.config.action_count;
        scan.actions = r.actions;
        scan.lp = r.old_log_probabilities;
        scan.v = r.old_values;
        scan.adv = r.advantages;
        scan.ret = r.returns;
        scan.invalid = s.invalid.data();
        launch("k_scan", ppo::k_scan, dim3(static_cast<unsigned>((s.width + 31) / 32 + 1), static_cast<unsigned>(chunks)), 256,
               0, st, scan);
        check(cudaGetLastError(), "validate rollout");
        int invalid = 0;
        s.invalid.download(&invalid, 1, st);
        if (invalid) raise(T8B_ENONFINITE, "PPO rollout contains a non-finite value or invalid action");
        s.metrics.zero(st);
        if (s.sample_entropy.size() < samples) {
            s.sample_entropy.allocate(samples);
            s.sample_decision.allocate(samples);
        }
        if (s.perm.size() < samples) {
            s.perm.allocate(samples);
            s.grouped.allocate(samples);
        }
        // permutations: prepared in the background when the caller announced them
        std::vector<std::vector<uint32_t>> perms;
        if (s.shuffler.joinable()) s.shuffler.join();
        if (s.prepared_valid && s.prepared_samples == samples && s.prepared_seed == shuffle_seed &&
            s.prepared_epochs >= cfg->epochs) {
            perms = std::move(s.prepared);
        } else {
            perms = make_permutations(samples, cfg->epochs, shuffle_seed);
        }
        s.prepared_valid = false;
        const size_t mb = cfg->minibatch_size;
        size_t minibatches = 0;
        int epochs_completed = 0;
        bool early = false;
        double previous_kl = 0.0;
        const int norm_blocks = 256;
        for (int epoch = 0; epoch < cfg->epochs; ++epoch) {
            s.perm.upload(perms[static_cast<size_t>(epoch)].data(), samples, st);
            group_minibatches(s, r, samples, mb, st);
            for (size_t offset = 0; offset < samples; offset += mb) {
                const size_t n = std::min(mb, samples - offset);
                ++minibatches;
                ppo::Prep prep{};
                prep.obs = r.observations;
                prep.width = s.width;
                prep.padded = s.padded;
                prep.mean = s.obs_mean.data();
                prep.istd = s.obs_istd.data();
                prep.clip = s.config.observation_clip;
                prep.normalize = s.normalizing() ? 1 : 0;
                prep.perm = s.grouped.data();
                prep.offset = offset;
                prep.count = n;
                prep.x = s.x.data();
                prep.src_bits = r.action_mask_bits;
                prep.src_bytes = r.action_mask_bits ? nullptr : r.action_masks;
                prep.action_count = s.config.action_count;
                prep.bits = s.mb_bits.data();
                prep.src_actions = r.actions;
                prep.actions = s.mb_actions.data();
                prep.src_old_lp = r.old_log_probabilities;
                prep.old_lp = s.mb_old_lp.data();
                prep.src_old_v = r.old_values;
                prep.old_v = s.mb_old_v.data();
                prep.src_adv = r.advantages;
                prep.adv = s.mb_adv.data();
                prep.src_ret = r.returns;
                prep.ret = s.mb_ret.data();
                prep.src_tables = r.feature_tables;
                prep.tables = s.mb_tables.data();
                launch("k_gather", ppo::k_gather, blocks((n + ppo::kGatherRows - 1) / ppo::kGatherRows, ppo::kWarps),
                       32 * ppo::kWarps, 0, st, prep);
                check(cudaGetLastError(), "gather minibatch");
                s.network(n, st);
                ppo::Loss loss{};
                loss.out = s.out.data();
                loss.ld = kOutPad;
                loss.feature_size = s.feature_size;
                loss.action_count = s.config.action_count;
                loss.features = s.features.data();
                loss.table_count = s.tables;
                loss.tables = s.mb_tables.data();
                loss.bits = s.mb_bits.data();
                loss.actions = s.mb_actions.data();
                loss.old_lp = s.mb_old_lp.data();
                loss.old_v = s.mb_old_v.data();
                loss.adv = s.mb_adv.data();
                loss.ret = s.mb_ret.data();
                loss.count = n;
                loss.inv_batch = 1.0f / static_cast<float>(n);
                loss.clip = cfg->clip_range;
                loss.value_clip = cfg->value_clip_range;
                loss.value_coef = cfg->value_coefficient;
                loss.entropy_coef = cfg->entropy_coefficient;
                loss.dout = s.dout.data();
                loss.ld_grad = kOutPad;
                loss.block_metrics = s.block_metrics.data();
                loss.out_colsum = s.out_colsum.data();
                loss.sample_entropy = epoch == 0 ? s.sample_entropy.data() : nullptr;
                loss.sample_decision = epoch == 0 ? s.sample_decision.data() : nullptr;
                loss.perm = s.grouped.data();
                loss.offset = offset;
                loss.bucket_start = s.bucket_start.data() + (offset / mb) * (ppo::kBuckets + 1);
                unsigned loss_grid = static_cast<unsigned>(loss_blocks(n));
                const size_t table_bytes = static_cast<size_t>(s.config.action_count) * s.feature_size * sizeof(float);
                if (tensor_core_objective(s.feature_size, s.config.action_count)) {
                    // one row of partials per 128-row tile; persistent CTAs, one per SM
                    loss_grid = static_cast<unsigned>(ppo::tc_tiles(n));
                    const unsigned ctas = std::min(loss_grid, static_cast<unsigned>(sm_count()));
                    launch("k_loss", ppo::k_loss_tc, ctas, ppo::kTcThreads, ppo::kTcSmemBytes, st, loss,
                           static_cast<const uint4*>(s.table_images.data()), static_cast<int>(loss_grid), s.error.data());
                } else if (s.feature_size == 48) {
                    launch("k_loss", ppo::k_loss<48>, loss_grid, 32 * ppo::kWarps, table_bytes, st, loss);
                } else {
                    launch("k_loss", ppo::k_loss<32>, loss_grid, 32 * ppo::kWarps, table_bytes, st, loss);
                }
                check(cudaGetLastError(), "PPO objective");
                launch("k_sum_rows_f64", ppo::k_sum_rows_f64, ppo::kMetrics, 256, 0, st, s.block_metrics.data(), static_cast<int>(loss_grid),
                                                                   ppo::kMetrics, s.metrics.data(), 1);
                s.column_sums(s.out_colsum.data(), static_cast<int>(loss_grid), kOutPad, s.outputs,
                              s.grads.data() + s.b_off[s.layers], st);
                s.backward(n, st);
                if (s.comm.active()) {
                    // data parallel: the mean of the ranks' minibatch gradients, before the norm clip
                    s.comm.hooks.allreduce_sum_f32(s.grads.data(), s.param_count, stream, s.comm.hooks.user);
                    launch("k_scale", ppo::k_scale, blocks(s.param_count, 256), 256, 0, st, s.grads.data(), s.param_count,
                                                                              1.0f / static_cast<float>(s.comm.hooks.world_size));
                }
                launch("k_square_partials", ppo::k_square_partials, norm_blocks, 256, 0, st, s.grads.data(), s.param_count, s.norm_partial.data());
                launch("k_norm_finish", ppo::k_norm_finish, 1, 32, 0, st, s.norm_partial.data(), norm_blocks, s.norm_sq.data(), s.metrics.data());
                ++s.optimizer_step;
                const float bc1 = 1.0f - std::pow(cfg->adam_beta1, static_cast<float>(s.optimizer_step));
                const float bc2 = 1.0f - std::pow(cfg->adam_beta2, static_cast<float>(s.optimizer_step));
                launch("k_adam", ppo::k_adam, blocks(s.param_count, 256), 256, 0, st, 
                    s.params.data(), s.grads.data(), s.m1.data(), s.m2.data(), s.param_count, s.norm_sq.data(),
                    cfg->max_gradient_norm, cfg->learning_rate, cfg->adam_beta1, cfg->adam_beta2, cfg->adam_epsilon, bc1,
                    bc2, s.adam, 1);
                check(cudaGetLastError(), "Adam");
            }
            epochs_completed = epoch + 1;
            if (cfg->target_kl > 0.0f) {
                double sums[ppo::kMetrics];
                s.metrics.download(sums, ppo::kMetrics, st);
                double kl = sums[3] - previous_kl;
                previous_kl = sums[3];
                double global_samples = static_cast<double>(samples);
                if (s.comm.active() && s.comm.hooks.allreduce_sum_f64) {
                    // every rank early-stops together on the KL over all ranks' samples
                    double pair[2] = {kl, global_samples};
                    check(cudaMemcpyAsync(s.kl_pair.data(), pair, sizeof pair, cudaMemcpyHostToDevice, st), "KL");
                    s.comm.hooks.allreduce_sum_f64(s.kl_pair.data(), 2, stream, s.comm.hooks.user);
                    s.kl_pair.download(pair, 2, st);
                    kl = pair[0];
                    global_samples = pair[1];
                }
                const double mean_kl = kl / global_samples;
                if (!std::isfinite(mean_kl)) raise(T8B_ENONFINITE, "PPO KL became non-finite; optimizer update aborted");
                if (mean_kl > cfg->target_kl) {
                    early = true;
                    break;
                }
            }
        }
        // merge the observation normaliser after the update (src/ppo.cu:1663-1667)
        if (normalizing) {
            if (s.comm.active() && s.comm.hooks.allreduce_sum_f64) {
                // data parallel: every rank's batch moments land in its own slot of a zeroed
                // [world][width][3] buffer, a sum all-reduce gathers them, and each rank merges
                // the slots in rank order into identical running statistics
                const int world = s.comm.hooks.world_size;
                const size_t slot = static_cast<size_t>(s.width) * 3;
                if (s.obs_gathered.size() < world * slot) s.obs_gathered.allocate(world * slot);
                s.obs_gathered.zero(st);
                launch("k_obs_merge", ppo::k_obs_merge, blocks(s.width, 128), 128, 0, st, s.obs_chunks.data(), static_cast<int>(chunks),
                       s.width, 0.0, nullptr, nullptr, nullptr, s.config.observation_epsilon,
                       s.obs_gathered.data() + static_cast<size_t>(s.comm.hooks.rank) * slot);
                s.comm.hooks.allreduce_sum_f64(s.obs_gathered.data(), world * slot, stream, s.comm.hooks.user);
                launch("k_obs_merge", ppo::k_obs_merge, blocks(s.width, 128), 128, 0, st, s.obs_gathered.data(), world, s.width,
                       static_cast<double>(s.obs_count), s.obs_mean.data(), s.obs_var.data(), s.obs_istd.data(),
                       s.config.observation_epsilon, nullptr);
                s.obs_count += samples * static_cast<uint64_t>(world);  // ranks hold equal-size rollouts
            } else {
                launch("k_obs_merge", ppo::k_obs_merge, blocks(s.width, 128), 128, 0, st, s.obs_chunks.data(), static_cast<int>(chunks),
                       s.width, static_cast<double>(s.obs_count), s.obs_mean.data(), s.obs_var.data(), s.obs_istd.data(),
                       s.config.observation_epsilon, nullptr);
                s.obs_count += samples;
            }
            check(cudaGetLastError(), "merge observation statistics");
        }
        // rollout decision entropy (src/ppo.cu:1671-1683)
        const int dblocks = 256;
        if (r.entropies) {
            launch("k_decision_partials", k_decision_partials, dblocks, 256, 0, st, r.entropies, nullptr, r.action_mask_bits ? nullptr : r.action_masks,
                                                        r.action_mask_bits, s.config.action_count, samples, s.entropy_sums.data());
        } else {
            launch("k_decision_partials", k_decision_partials, dblocks, 256, 0, st, s.sample_entropy.data(), s.sample_decision.data(), nullptr, nullptr,
                                                        s.config.action_count, samples, s.entropy_sums.data());
        }
        launch("k_decision_finish", k_decision_finish, 1, 32, 0, st, s.entropy_sums.data(), dblocks, s.entropy_sums.data() + 2 * 1024);
        check(cudaGetLastError(), "decision entropy");
        if (s.comm.active() && s.comm.hooks.allreduce_sum_f64) {
            // the entropy-floor controller sees the decision entropy of every rank's rollout
            s.comm.hooks.allreduce_sum_f64(s.entropy_sums.data() + 2 * 1024, 2, stream, s.comm.hooks.user);
        }
        double m[ppo::kMetrics];
        s.metrics.download(m, ppo::kMetrics, st);
        double ent[2];
        check(cudaMemcpyAsync(ent, s.entropy_sums.data() + 2 * 1024, sizeof ent, cudaMemcpyDeviceToHost, st), "entropy");
        check(cudaStreamSynchronize(st), "update");
        s.sync_error(st);
        for (double v : m) {
            if (!std::isfinite(v)) raise(T8B_ENONFINITE, "PPO metrics became non-finite; checkpoint was not written");
        }
        if (metrics_out) {
            const double visits = static_cast<double>(samples) * epochs_completed;
            t8b_ppo_metrics_t& o = *metrics_out;
            std::memset(&o, 0, sizeof o);
            o.policy_loss = static_cast<float>(m[0] / visits);
            o.value_loss = static_cast<float>(m[1] / visits);
            o.entropy = static_cast<float>(m[2] / visits);
            o.approximate_kl = static_cast<float>(m[3] / visits);
            o.clip_fraction = static_cast<float>(m[4] / visits);
            o.gradient_norm = static_cast<float>(m[5] / static_cast<double>(minibatches));
            o.decision_fraction = static_cast<float>(m[6] / visits);
            o.decision_entropy = m[6] > 0.0 ? static_cast<float>(m[7] / m[6]) : 0.0f;
            o.rollout_decision_entropy = ent[1] > 0.0 ? static_cast<float>(ent[0] / ent[1]) : 0.0f;
            o.minibatches = minibatches;
            o.epochs_completed = epochs_completed;
            o.early_stopped = early ? 1 : 0;
        }
    });
}

int t8b_policy_get_parameters(t8b_policy* p, float* host, size_t count) {
    return with_policy(p, [&](t8b_policy& s) {
        if (count != s.param_count) raise(T8B_EINVAL, "parameter count mismatch");
        s.params.download(host, count, nullptr);
    });
}

int t8b_policy_set_parameters(t8b_policy* p, const float* host, size_t count) {
    return with_policy(p, [&](t8b_policy& s) {
        if (count != s.param_count) raise(T8B_EINVAL, "parameter count mismatch");
        s.params.upload(host, count, nullptr);
        s.refresh_operands(nullptr);
        check(cudaStreamSynchronize(nullptr), "set parameters");
    });
}

int t8b_policy_get_gradients(t8b_policy* p, float* host, size_t count) {
    return with_policy(p, [&](t8b_policy& s) {
        if (count != s.param_count) raise(T8B_EINVAL, "parameter count mismatch");
        s.grads.download(host, count, nullptr);
    });
}

int t8b_policy_get_optimizer_state(t8b_policy* p, float* first, float* second, uint64_t* step) {
    return with_policy(p, [&](t8b_policy& s) {
        if (first) s.m1.download(first, s.param_count, nullptr);
        if (second) s.m2.download(second, s.param_count, nullptr);
        if (step) *step = s.optimizer_step;
    });
}

int t8b_policy_set_optimizer_state(t8b_policy* p, const float* first, const float* second, uint64_t step) {
    return with_policy(p, [&](t8b_policy& s) {
        if (first) s.m1.upload(first, s.param_count, nullptr);
        if (second) s.m2.upload(second, s.param_count, nullptr);
        s.optimizer_step = step;
        check(cudaStreamSynchronize(nullptr), "set optimizer state");
    });
}

int t8b_policy_get_observation_statistics(t8b_policy* p, float* mean, float* variance, uint64_t* count) {
    return with_policy(p, [&](t8b_policy& s) {
        if (mean) s.obs_mean.download(mean, s.width, nullptr);
        if (variance) s.obs_var.download(variance, s.width, nullptr);
        if (count) *count = s.obs_count;
    });
}

int t8b_policy_set_observation_statistics(t8b_policy* p, const float* mean, const float* variance, uint64_t count) {
    return with_policy(p, [&](t8b_policy& s) {
        s.obs_mean.upload(mean, s.width, nullptr);
        s.obs_var.upload(variance, s.width, nullptr);
        launch("k_refresh_istd", ppo::k_refresh_istd, blocks(s.width, 128), 128, 0, nullptr, s.obs_var.data(), s.obs_istd.data(), s.width,
                                                           s.config.observation_epsilon);
        check(cudaStreamSynchronize(nullptr), "set observation statistics");
        s.obs_count = count;
    });
}

}  // extern "C"

// ------------------------------------------------------------------ checkpoints
// The reference's .t8ppo file (src/ppo.cu:1704-1845), field for field so that checkpoints
// move between the two implementations: a 40-byte header, the 160-byte contract block, the
// 24-byte normaliser block (version 4+), the 16-byte integrity block and the payload
// (parameters, Adam first and second moments in the canonical order, then the observation
// mean and variance), checksummed with 64-bit FNV-1a over the payload bytes.
namespace t8b {
namespace ckpt {

struct CkptHeader {
    char magic[8];
    uint32_t version, observation_size, action_count, hidden_size;
    uint64_t optimizer_step, parameter_count;
};
struct CkptContract {
    char catalog_sha256[64], roster_version[24], observation_contract[32], action_contract[32];
    uint32_t action_feature_size, universal_action_count;
};
struct CkptNormalizer {
    uint32_t enabled, architecture;
    uint64_t count;
    float clip, epsilon;
};
struct CkptIntegrity {
    uint64_t payload_bytes, payload_checksum;
};
static_assert(sizeof(CkptHeader) == 40 && sizeof(CkptContract) == 160 && sizeof(CkptNormalizer) == 24 &&
                  sizeof(CkptIntegrity) == 16,
              "checkpoint blocks have the reference's sizes");

constexpr char kCkptMagic[8] = {'T', '8', 'V', '2', 'P', 'P', 'O', '\0'};
constexpr uint32_t kCkptVersion = 4, kCkptLayersVersion = 5;

inline uint32_t architecture_code(const t8b_actor_config_t& c) {
    if (c.shared_layers == 2 && c.head_layers == 0) return 0;
    return (1u << 16) | static_cast<uint32_t>(c.shared_layers) | (static_cast<uint32_t>(c.head_layers) << 8);
}

inline uint64_t fnv1a(const std::vector<float>& payload) {
    uint64_t h = 14695981039346656037ull;
    const auto* bytes = reinterpret_cast<const unsigned char*>(payload.data());
    for (size_t i = 0; i < payload.size() * sizeof(float); ++i) {
        h ^= bytes[i];
        h *= 1099511628211ull;
    }
    return h;
}

// The reference ActorCriticConfig's contract defaults (include/t8_v2/ppo.hpp:21-24).
inline t8b_checkpoint_contract_t contract_or_default(const t8b_checkpoint_contract_t* c) {
    if (c) return *c;
    t8b_checkpoint_contract_t d{};
    std::memset(d.catalog_sha256, '0', sizeof d.catalog_sha256);
    std::memcpy(d.roster_version, "compatibility", 13);
    std::memcpy(d.observation_contract, "v2-observation", 14);
    std::memcpy(d.action_contract, "fixed-24-compatibility", 22);
    return d;
}

template <size_t N>
std::string text(const char (&field)[N]) {
    size_t n = 0;
    while (n < N && field[n] != '\0') ++n;
    return std::string(field, n);
}

}  // namespace ckpt
}  // namespace t8b

extern "C" {

int t8b_policy_save_checkpoint(t8b_policy* p, const char* path, const t8b_checkpoint_contract_t* contract, void* stream) {
    using namespace t8b;
    using namespace t8b::ckpt;
    return with_policy(p, [&](t8b_policy& s) {
        if (!path) raise(T8B_EINVAL, "null checkpoint path");
        check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "synchronize before checkpoint save");
        const size_t n = s.param_count, w = static_cast<size_t>(s.width);
        std::vector<float> payload(3 * n + 2 * w);
        s.params.download(payload.data(), n, nullptr);
        s.m1.download(payload.data() + n, n, nullptr);
        s.m2.download(payload.data() + 2 * n, n, nullptr);
        s.obs_mean.download(payload.data() + 3 * n, w, nullptr);
        s.obs_var.download(payload.data() + 3 * n + w, w, nullptr);
        for (float v : payload) {
            if (!std::isfinite(v)) raise(T8B_ENONFINITE, std::string("refusing to save checkpoint with non-finite tensors: ") + path);
        }
        const t8b_actor_config_t& c = s.config;
        const uint32_t architecture = architecture_code(c);
        CkptHeader header{};
        std::memcpy(header.magic, kCkptMagic, 8);
        header.version = architecture == 0 ? kCkptVersion : kCkptLayersVersion;
        header.observation_size = static_cast<uint32_t>(c.observation_size);
        header.action_count = static_cast<uint32_t>(c.action_count);
        header.hidden_size = static_cast<uint32_t>(c.hidden_size);
        header.optimizer_step = s.optimizer_step;
        header.parameter_count = n;
        const t8b_checkpoint_contract_t text_fields = contract_or_default(contract);
        CkptContract block{};
        std::memcpy(block.catalog_sha256, text_fields.catalog_sha256, 64);
        std::memcpy(block.roster_version, text_fields.roster_version, 24);
        std::memcpy(block.observation_contract, text_fields.observation_contract, 32);
        std::memcpy(block.action_contract, text_fields.action_contract, 32);
        block.action_feature_size = static_cast<uint32_t>(c.action_feature_size);
        block.universal_action_count = static_cast<uint32_t>(c.universal_action_count);
        const CkptNormalizer normalizer{c.observation_normalization ? 1u : 0u, architecture, s.obs_count,
                                        c.observation_clip, c.observation_epsilon};
        const CkptIntegrity integrity{payload.size() * sizeof(float), fnv1a(payload)};
        const std::filesystem::path target(path);
        if (!target.parent_path().empty()) std::filesystem::create_directories(target.parent_path());
        if (std::filesystem::exists(target)) raise(T8B_ESTATE, std::string("refusing to overwrite checkpoint: ") + path);
        std::filesystem::path temporary = target;
        temporary += ".tmp";
        std::error_code ignored;
        std::filesystem::remove(temporary, ignored);
        {
            std::ofstream out(temporary, std::ios::binary | std::ios::trunc);
            if (!out) raise(T8B_ECUDA, "could not open checkpoint for writing: " + temporary.string());
            out.write(reinterpret_cast<const char*>(&header), sizeof header);
            out.write(reinterpret_cast<const char*>(&block), sizeof block);
            out.write(reinterpret_cast<const char*>(&normalizer), sizeof normalizer);
            out.write(reinterpret_cast<const char*>(&integrity), sizeof integrity);
            out.write(reinterpret_cast<const char*>(payload.data()), static_cast<std::streamsize>(payload.size() * sizeof(float)));
            out.flush();
            if (!out) raise(T8B_ECUDA, "checkpoint write failed: " + temporary.string());
        }
        std::filesystem::rename(temporary, target);
    });
}

int t8b_policy_load_checkpoint(t8b_policy* p, const char* path, int load_optimizer_state,
                               const t8b_checkpoint_contract_t* contract, void* stream) {
    using namespace t8b;
    using namespace t8b::ckpt;
    return with_policy(p, [&](t8b_policy& s) {
        if (!path) raise(T8B_EINVAL, "null checkpoint path");
        const std::string where(path);
        std::ifstream in(path, std::ios::binary);
        if (!in) raise(T8B_ECUDA, "could not open checkpoint for reading: " + where);
        t8b_actor_config_t& c = s.config;
        CkptHeader header{};
        in.read(reinterpret_cast<char*>(&header), sizeof header);
        const bool magic = in && std::memcmp(header.magic, kCkptMagic, 8) == 0;
        if (magic && header.version < 3) {
            raise(T8B_ECUDA, "legacy fixed-action checkpoint is incompatible with the full-roster policy contract: " + where);
        }
        if (!magic || (header.version != 3 && header.version != kCkptVersion && header.version != kCkptLayersVersion) ||
            header.observation_size != static_cast<uint32_t>(c.observation_size) ||
            header.action_count != static_cast<uint32_t>(c.action_count) ||
            header.hidden_size != static_cast<uint32_t>(c.hidden_size) || header.parameter_count != s.param_count) {
            raise(T8B_ECUDA, "checkpoint architecture/version mismatch: " + where);
        }
        const t8b_checkpoint_contract_t want = contract_or_default(contract);
        CkptContract block{};
        in.read(reinterpret_cast<char*>(&block), sizeof block);
        if (!in || text(block.catalog_sha256) != text(want.catalog_sha256) ||
            text(block.roster_version) != text(want.roster_version) ||
            text(block.observation_contract) != text(want.observation_contract) ||
            text(block.action_contract) != text(want.action_contract) ||
            block.action_feature_size != static_cast<uint32_t>(c.action_feature_size) ||
            block.universal_action_count != static_cast<uint32_t>(c.universal_action_count)) {
            raise(T8B_ECUDA, "checkpoint catalog/roster/action contract mismatch: " + where);
        }
        const bool has_normalizer = header.version >= 4;
        CkptNormalizer normalizer{};
        if (has_normalizer) {
            in.read(reinterpret_cast<char*>(&normalizer), sizeof normalizer);
            if (!in || normalizer.enabled > 1 || normalizer.architecture != architecture_code(c) ||
                !std::isfinite(normalizer.clip) || normalizer.clip <= 0.0f || !std::isfinite(normalizer.epsilon) ||
                normalizer.epsilon <= 0.0f) {
                raise(T8B_ECUDA, "checkpoint observation normalizer block is invalid: " + where);
            }
        }
        const size_t n = s.param_count, w = static_cast<size_t>(s.width);
        const size_t count = 3 * n + (has_normalizer ? 2 * w : 0);
        CkptIntegrity integrity{};
        in.read(reinterpret_cast<char*>(&integrity), sizeof integrity);
        if (!in || integrity.payload_bytes != count * sizeof(float)) raise(T8B_ECUDA, "checkpoint payload size mismatch: " + where);
        std::vector<float> payload(count);
        in.read(reinterpret_cast<char*>(payload.data()), static_cast<std::streamsize>(count * sizeof(float)));
        if (!in) raise(T8B_ECUDA, "checkpoint tensor is truncated: " + where);
        if (fnv1a(payload) != integrity.payload_checksum) raise(T8B_ECUDA, "checkpoint checksum mismatch: " + where);
        for (float v : payload) {
            if (!std::isfinite(v)) raise(T8B_ENONFINITE, "checkpoint contains non-finite tensors: " + where);
        }
        if (has_normalizer) {
            for (size_t i = 0; i < w; ++i) {
                if (payload[3 * n + w + i] < 0.0f) raise(T8B_ECUDA, "checkpoint observation variance is negative: " + where);
            }
        }
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        s.params.upload(payload.data(), n, st);
        if (load_optimizer_state) {
            s.m1.upload(payload.data() + n, n, st);
            s.m2.upload(payload.data() + 2 * n, n, st);
            s.optimizer_step = header.optimizer_step;
        } else {
            s.m1.zero(st);
            s.m2.zero(st);
            s.optimizer_step = 0;
        }
        if (has_normalizer) {
            c.observation_normalization = static_cast<uint8_t>(normalizer.enabled);
            c.observation_clip = normalizer.clip;
            c.observation_epsilon = normalizer.epsilon;
            s.obs_mean.upload(payload.data() + 3 * n, w, st);
            s.obs_var.upload(payload.data() + 3 * n + w, w, st);
            s.obs_count = normalizer.count;
        } else {
            c.observation_normalization = 0;
            const std::vector<float> zeros(w, 0.0f), ones(w, 1.0f);
            s.obs_mean.upload(zeros.data(), w, st);
            s.obs_var.upload(ones.data(), w, st);
            s.obs_count = 0;
        }
        launch("k_refresh_istd", ppo::k_refresh_istd, blocks(s.width, 128), 128, 0, st, s.obs_var.data(), s.obs_istd.data(),
               s.width, c.observation_epsilon);
        s.refresh_operands(st);
        check(cudaStreamSynchronize(st), "synchronize checkpoint load");
    });
}

// Test aid: the network outputs [n][query..., value] of the last forward (fp32).
int t8b_policy_download_outputs(t8b_policy* p, float* host, size_t n) {
    return with_policy(p, [&](t8b_policy& s) {
        if (n > s.capacity) raise(T8B_EINVAL, "count exceeds capacity");
        std::vector<float> rows(n * kOutPad);
        s.out.download(rows.data(), rows.size(), nullptr);
        for (size_t i = 0; i < n; ++i) std::copy(rows.begin() + i * kOutPad, rows.begin() + i * kOutPad + s.outputs, host + i * s.outputs);
    });
}

// Test aid: an intermediate of the last forward/backward as fp32 rows: which = 0 the layer-1
// input (padded width), 1 hidden activation `layer`, 2 its pre-activation gradient, 3 the output
// gradient row (64 wide).
int t8b_policy_download_activation(t8b_policy* p, int which, int layer, float* host, size_t n) {
    return with_policy(p, [&](t8b_policy& s) {
        if (n > s.capacity || layer < 0 || layer >= s.layers) raise(T8B_EINVAL, "activation request out of range");
        const bf16* src = which == 0 ? s.x.data() : which == 1 ? s.h[layer].data() : which == 2 ? s.dz[layer].data() : s.dout.data();
        const size_t width = which == 0 ? s.padded : which == 3 ? kOutPad : s.hidden;
        std::vector<bf16> rows(n * width);
        check(cudaMemcpy(rows.data(), src, rows.size() * sizeof(bf16), cudaMemcpyDeviceToHost), "download activation");
        for (size_t i = 0; i < rows.size(); ++i) host[i] = __bfloat162float(rows[i]);
    });
}

// The actor configuration in force (load_checkpoint adopts the file's normaliser setting).
int t8b_policy_get_config(const t8b_policy* p, t8b_actor_config_t* out) {
    return with_policy(const_cast<t8b_policy*>(p), [&](t8b_policy& s) {
        if (out == nullptr) raise(T8B_EINVAL, "null argument");
        *out = s.config;
    });
}

// The network alone on n device observations (normalised as forward does): raw outputs
// [n][outputs] into `outputs` when given, and with `output_gradients` ([n][outputs] fp32) the
// backward pass from them into the gradient buffer (t8b_policy_get_gradients).
int t8b_policy_debug_network(t8b_policy* p, const float* observations, size_t n, const float* output_gradients,
                             float* outputs, void* stream) {
    return with_policy(p, [&](t8b_policy& s) {
        if (observations == nullptr || n == 0 || n > s.capacity) raise(T8B_EINVAL, "debug batch must fit the capacity");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        ppo::Prep prep{};
        prep.obs = observations;
        prep.width = s.width;
        prep.padded = s.padded;
        prep.mean = s.obs_mean.data();
        prep.istd = s.obs_istd.data();
        prep.clip = s.config.observation_clip;
        prep.normalize = s.normalizing() ? 1 : 0;
        prep.count = n;
        prep.x = s.x.data();
        launch("k_prep", ppo::k_prep, blocks(n, ppo::kWarps), 32 * ppo::kWarps, 0, st, prep);
        check(cudaGetLastError(), "prepare inputs");
        s.network(n, st);
        if (outputs != nullptr) {
            check(cudaMemcpy2DAsync(outputs, sizeof(float) * s.outputs, s.out.data(), sizeof(float) * kOutPad,
                                    sizeof(float) * s.outputs, n, cudaMemcpyDeviceToDevice, st), "network outputs");
        }
        if (output_gradients != nullptr) {
            launch("k_rows_to_bf16", k_rows_to_bf16, blocks(n * kOutPad, 256), 256, 0, st, output_gradients, n, s.outputs,
                   s.dout.data(), kOutPad);
            s.column_sums(output_gradients, static_cast<int>(n), s.outputs, s.outputs, s.grads.data() + s.b_off[s.layers], st);
            s.backward(n, st);
        }
        s.sync_error(st);
    });
}

int t8b_policy_synchronize(t8b_policy* p, void* stream) {
    return with_policy(p, [&](t8b_policy& s) {
        check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "synchronize policy");
        s.sync_error(static_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
