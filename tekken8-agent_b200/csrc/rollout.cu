// Rollout buffer: the GpuRolloutBuffer contract (include/t8_v2/ppo.hpp:223-291, src/ppo.cu:2001-2481)
// with its C ABI (t8b_rollout_*), plus the raw-logits PPO objective (t8b_ppo_output_gradient).
//
// Storage is [step][environment] so a step's records are contiguous and GAE's reverse sweep
// reads coalesced rows. Masks are kept packed (12 words per sample) next to the uint8 view of
// the reference. GAE writes advantages and returns and, in the same pass, per-block fp64
// moments of the advantages, so normalisation needs one more pass instead of two.
#include "common.cuh"
#include "gemm_host.cuh"
#include "internal.cuh"
#include "ppo_kernels.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

namespace t8b {

// GAE block: 32 fights x chunks of 64 steps staged in shared memory (28 KB), 256 threads.
constexpr int kGaeFights = 32;
constexpr int kGaeChunk = 64;
constexpr unsigned kGaeThreads = 256;

// gae_kernel (src/ppo.cu:2003-2029) fused with advantage_stats_kernel (src/ppo.cu:2031-2063).
// The [step][fight] records of one block's 32 fights are staged a chunk of 64 steps at a time,
// latest chunk first: all 256 threads load the chunk's rows (each warp a 32-fight row of every
// array, every load issued before any is used), warp 0 runs the recurrence of the reference for
// its 32 fights, one lane each, over the chunk in reverse (the same fp32 operations in the same
// order, so advantages and returns are the reference's bit for bit), and all threads store the
// advantages and returns rows. The fp64 moments of each fight's advantages are summed in reverse
// step order and reduced over the warp into one partial per block.
__global__ void __launch_bounds__(kGaeThreads) k_gae(const float* rewards, const float* values, const uint8_t* terminated,
                                                     const uint8_t* truncated, const float* next_values, size_t envs,
                                                     size_t horizon, float gamma, float lambda, float* adv, float* ret,
                                                     double* partial) {
    __shared__ float s_reward[kGaeChunk][kGaeFights], s_value[kGaeChunk][kGaeFights], s_next[kGaeChunk][kGaeFights];
    __shared__ uint8_t s_term[kGaeChunk][kGaeFights], s_trunc[kGaeChunk][kGaeFights];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t fight0 = static_cast<size_t>(blockIdx.x) * kGaeFights;
    const size_t fight = fight0 + static_cast<size_t>(lane);
    const bool live = fight < envs;
    float next = 0.0f;
    double sum = 0.0, square = 0.0;
    for (size_t chunk_end = horizon; chunk_end > 0;) {
        const size_t first = chunk_end > static_cast<size_t>(kGaeChunk) ? chunk_end - kGaeChunk : 0;
        const int rows = static_cast<int>(chunk_end - first);
        constexpr int kRowsPerWarp = kGaeChunk / (kGaeThreads / 32);
        float r[kRowsPerWarp], v[kRowsPerWarp], nv[kRowsPerWarp];
        uint8_t te[kRowsPerWarp], tr[kRowsPerWarp];
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            const int row = warp + k * (kGaeThreads / 32);
            const size_t at = (first + static_cast<size_t>(row)) * envs + fight;
            const bool in = live && row < rows;
            r[k] = in ? rewards[at] : 0.0f;
            v[k] = in ? values[at] : 0.0f;
            nv[k] = in ? next_values[at] : 0.0f;
            te[k] = in ? terminated[at] : 0;
            tr[k] = in ? truncated[at] : 0;
        }
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            const int row = warp + k * (kGaeThreads / 32);
            s_reward[row][lane] = r[k];
            s_value[row][lane] = v[k];
            s_next[row][lane] = nv[k];
            s_term[row][lane] = te[k];
            s_trunc[row][lane] = tr[k];
        }
        __syncthreads();
        if (warp == 0) {
            for (int row = rows - 1; row >= 0; --row) {
                const bool time_limit = s_trunc[row][lane] != 0;
                const bool ended = s_term[row][lane] != 0;
                const float bootstrap = ended && !time_limit ? 0.0f : 1.0f;
                const float trace = ended || time_limit ? 0.0f : 1.0f;
                const float value = s_value[row][lane];
                const float delta = s_reward[row][lane] + gamma * s_next[row][lane] * bootstrap - value;
                next = delta + gamma * lambda * trace * next;
                s_reward[row][lane] = next;
                s_next[row][lane] = next + value;
                if (live) {
                    sum += static_cast<double>(next);
                    square += static_cast<double>(next) * static_cast<double>(next);
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kRowsPerWarp; ++k) {
            const int row = warp + k * (kGaeThreads / 32);
            if (live && row < rows) {
                const size_t at = (first + static_cast<size_t>(row)) * envs + fight;
                adv[at] = s_reward[row][lane];
                ret[at] = s_next[row][lane];
            }
        }
        __syncthreads();
        chunk_end = first;
    }
    if (warp == 0) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            sum += __shfl_xor_sync(0xffffffffu, sum, off);
            square += __shfl_xor_sync(0xffffffffu, square, off);
        }
        if (lane == 0) {
            partial[2 * blockIdx.x] = sum;
            partial[2 * blockIdx.x + 1] = square;
        }
    }
}

// Fixed-order total of [blocks][2] partial sums -> out[0..1]: each lane of one warp sums a
// strided share in index order, then a fixed butterfly adds the lanes.
__global__ void k_pair_total(const double* partial, int blocks, double* out) {
    if (blockIdx.x != 0 || threadIdx.x >= 32) return;
    double a = 0.0, b = 0.0;
    for (int i = static_cast<int>(threadIdx.x); i < blocks; i += 32) {
        a += partial[2 * i];
        b += partial[2 * i + 1];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, off);
        b += __shfl_xor_sync(0xffffffffu, b, off);
    }
    if (threadIdx.x == 0) {
        out[0] = a;
        out[1] = b;
    }
}

// Per-block fp64 (sum, sum of squares) of a float array, grid-stride in index order.
__global__ void k_moments(const float* values, size_t n, double* partial) {
    __shared__ double s1[256], s2[256];
    double a = 0.0, b = 0.0;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const double v = values[i];
        a += v;
        b += v * v;
    }
    s1[threadIdx.x] = a;
    s2[threadIdx.x] = b;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            s1[threadIdx.x] += s1[threadIdx.x + w];
            s2[threadIdx.x] += s2[threadIdx.x + w];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        partial[2 * blockIdx.x] = s1[0];
        partial[2 * blockIdx.x + 1] = s2[0];
    }
}

// normalize_advantages_kernel (src/ppo.cu:2079-2091); stats = (sum, sum of squares, count).
__global__ void k_normalize(float* adv, size_t n, const double* stats) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const double count = stats[2];
    const double mean = stats[0] / count;
    const double second = stats[1] / count;
    const double inv = 1.0 / sqrt(fmax(second - mean * mean, 1e-12));
    adv[i] = static_cast<float>((static_cast<double>(adv[i]) - mean) * inv);
}

__global__ void k_set_count(double* stats, double count) {
    if (threadIdx.x == 0 && blockIdx.x == 0) stats[2] = count;
}

// record_outcome_kernel (src/ppo.cu:2093-2112)
__global__ void k_record_outcome(float* rewards, uint8_t* terminated, uint8_t* truncated, float* next_values,
                                 const float* r, const uint8_t* term, const uint8_t* trunc, const float* nv, float scale,
                                 size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    rewards[i] = r[i] * scale;
    terminated[i] = term[i];
    truncated[i] = trunc[i];
    next_values[i] = nv[i];
}

// A decision's recording (record_policy_device, include/t8_v2/ppo.hpp:241-250) as one launch:
// up to seven contiguous blocks copied (or zero-filled where the source is null), each moved in
// 16-byte words when both ends and the size allow it, else in 4-byte words; threads stride over
// the blocks' words in order.
constexpr int kRecordBlocks = 7;
struct RecordCopies {
    const void* src[kRecordBlocks];
    void* dst[kRecordBlocks];
    size_t first[kRecordBlocks + 1];  // prefix of the blocks' word counts
    int wide[kRecordBlocks];          // 16-byte words (else 4-byte)
    int count;
};
__global__ void k_record(RecordCopies r) {
    const size_t total = r.first[r.count];
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        int b = 0;
        while (i >= r.first[b + 1]) ++b;
        const size_t k = i - r.first[b];
        if (r.wide[b]) {
            const uint4 v = r.src[b] ? reinterpret_cast<const uint4*>(r.src[b])[k] : make_uint4(0, 0, 0, 0);
            reinterpret_cast<uint4*>(r.dst[b])[k] = v;
        } else {
            reinterpret_cast<uint32_t*>(r.dst[b])[k] = r.src[b] ? reinterpret_cast<const uint32_t*>(r.src[b])[k] : 0u;
        }
    }
}

// uint8 masks [n][actions] -> 12 packed words per sample (candidates past `actions` are 0)
__global__ void k_pack_masks(const uint8_t* bytes, int actions, uint32_t* bits, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n * 12) return;
    const size_t sample = i / 12;
    const int word = static_cast<int>(i % 12);
    uint32_t w = 0;
    for (int b = 0; b < 32 && word * 32 + b < actions; ++b) {
        w |= (bytes[sample * actions + word * 32 + b] != 0 ? 1u : 0u) << b;
    }
    bits[i] = w;
}

__global__ void k_expand(const uint32_t* bits, uint8_t* bytes, int actions, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n * actions) return;
    const size_t sample = i / actions;
    const int c = static_cast<int>(i % actions);
    bytes[i] = (bits[sample * 12 + (c >> 5)] >> (c & 31)) & 1u;
}

// discounted_return_kernel (src/ppo.cu:2114-2131)
__global__ void k_discounted(const float* rewards, const uint8_t* terminated, const uint8_t* truncated, size_t envs,
                             size_t horizon, float gamma, float* running, float* samples) {
    const size_t env = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (env >= envs) return;
    float r = running[env];
    for (size_t t = 0; t < horizon; ++t) {
        const size_t at = t * envs + env;
        r = r * gamma + rewards[at];
        samples[at] = r;
        if (terminated[at] || truncated[at]) r = 0.0f;
    }
    running[env] = r;
}

// scale_rewards_kernel (src/ppo.cu:2133-2137)
__global__ void k_scale_rewards(float* rewards, size_t n, float scale, float clip) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) rewards[i] = fminf(clip, fmaxf(-clip, rewards[i] * scale));
}

// ppo_output_gradient_kernel (src/ppo.cu:453-565) on raw outputs [n][k + 1]: one warp per sample
// at a time, SLOTS logits per lane (k <= 32 * SLOTS). The grid is a fixed number of resident
// blocks whose warps stride over the samples; each warp loads its next sample's logits and mask
// bytes before it works on the current one, so a row is in flight while the previous is scored.
// The kernel is bound by instruction issue more than by memory, so each logit takes one fast
// exponential (the __expf intrinsic; p = e * (1 / sum), log p = logit - log sum), the legal count
// comes from ballots, and the per-sample factors of the gradient are formed once. Lane m < 8 of each warp
// adds metric m of every sample the warp scores in fp64, and each block writes one row of
// [grid][8] partials; the sample-to-warp assignment is fixed, so the sums are reproducible.
constexpr int kMaxLogitSlots = 16;  // per lane: k <= 512
constexpr int kObjectiveBlocksPerSm = 6;

template <int SLOTS>
__global__ void __launch_bounds__(32 * ppo::kWarps) k_logit_objective(
    const float* out, const uint8_t* masks, const int64_t* actions, const float* old_lp, const float* old_v,
    const float* adv, const float* ret, size_t n, int k, float inv_batch, float clip, float value_clip,
    float value_coef, float entropy_coef, float* grads, double* block_metrics) {
    __shared__ double metric[ppo::kWarps][ppo::kMetrics];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t stride = static_cast<size_t>(gridDim.x) * ppo::kWarps;
    double acc = 0.0;
    size_t i = static_cast<size_t>(blockIdx.x) * ppo::kWarps + warp;
    float next_logit[SLOTS];
    uint8_t next_mask[SLOTS];
    const auto load = [&](size_t row) {
        const float* o = out + row * static_cast<size_t>(k + 1);
        const uint8_t* m = masks + row * static_cast<size_t>(k);
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            const int a = j * 32 + lane;
            next_logit[j] = a < k ? o[a] : 0.0f;
            next_mask[j] = a < k ? m[a] : 0;
        }
    };
    if (i < n) load(i);
    for (; i < n; i += stride) {
        float logit[SLOTS];
        bool legal[SLOTS];
        unsigned legal_count = 0;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            logit[j] = next_logit[j];
            legal[j] = next_mask[j] != 0;
            legal_count += __popc(__ballot_sync(0xffffffffu, legal[j]));
        }
        if (i + stride < n) load(i + stride);
        const int64_t action = actions[i];
        const float old_log = old_lp[i], a_i = adv[i], r_i = ret[i], v_old = old_v[i];
        const float v = out[i * static_cast<size_t>(k + 1) + k];
        const bool any = legal_count != 0;
        if (!any) {
            legal_count = 1;
#pragma unroll
            for (int j = 0; j < SLOTS; ++j) legal[j] = j * 32 + lane == 0;
        }
        float local_max = -3.402823466e38f;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            if (legal[j]) local_max = fmaxf(local_max, logit[j]);
        }
        const float maximum = ppo::warp_max(local_max);
        float e[SLOTS];
        float local = 0.0f;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            e[j] = legal[j] ? __expf(logit[j] - maximum) : 0.0f;
            local += e[j];
        }
        const float sum = fmaxf(ppo::warp_sum(local), 1e-20f);
        const float inv_sum = 1.0f / sum;
        const float log_sum = logf(sum) + maximum;
        const int selected = any ? static_cast<int>(action) : 0;
        const float chosen = __shfl_sync(0xffffffffu, logit[(selected >> 5) % SLOTS], selected & 31);
        const float log_ratio = (chosen - log_sum) - old_log;
        const float ratio = expf(log_ratio);
        const float unclipped = ratio * a_i;
        const float clipped = fminf(1.0f + clip, fmaxf(1.0f - clip, ratio)) * a_i;
        const float lp_grad = unclipped <= clipped ? -a_i * ratio : 0.0f;
        float entropy = 0.0f;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            e[j] *= inv_sum;  // the probability
            entropy -= e[j] * (logit[j] - log_sum);  // zero for the illegal (p = 0)
        }
        entropy = ppo::warp_sum(entropy);
        // d/d logit = (lp_grad (onehot - p) + entropy_coef p (log p + entropy)) / batch
        const float policy_scale = lp_grad * inv_batch, entropy_scale = entropy_coef * inv_batch;
        const float shift = entropy - log_sum;
        float* g = grads + i * static_cast<size_t>(k + 1);
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            const int a = j * 32 + lane;
            if (a >= k) continue;
            const float onehot = a == selected ? 1.0f : 0.0f;
            g[a] = legal[j] ? policy_scale * (onehot - e[j]) + entropy_scale * e[j] * (logit[j] + shift) : 0.0f;
        }
        const float error = v - r_i;
        float vgrad = error;
        float vloss = 0.5f * error * error;
        if (value_clip > 0.0f) {
            const float delta = v - v_old;
            const float cv = v_old + fminf(value_clip, fmaxf(-value_clip, delta));
            const float cerr = cv - r_i;
            const float closs = 0.5f * cerr * cerr;
            if (closs > vloss) {
                vloss = closs;
                vgrad = fabsf(delta) <= value_clip ? cerr : 0.0f;
            }
        }
        if (lane == 0) g[k] = value_coef * vgrad * inv_batch;
        const bool decision = legal_count > 1;
        const float mine = lane == 0 ? -fminf(unclipped, clipped)
                         : lane == 1 ? vloss
                         : lane == 2 ? entropy
                         : lane == 3 ? (ratio - 1.0f) - log_ratio
                         : lane == 4 ? (fabsf(ratio - 1.0f) > clip ? 1.0f : 0.0f)
                         : lane == 6 ? (decision ? 1.0f : 0.0f)
                         : lane == 7 ? (decision ? entropy : 0.0f)
                                     : 0.0f;
        acc += static_cast<double>(mine);
    }
    if (lane < ppo::kMetrics) metric[warp][lane] = acc;
    __syncthreads();
    if (block_metrics != nullptr && threadIdx.x < ppo::kMetrics) {
        double s = 0.0;
        for (int w = 0; w < ppo::kWarps; ++w) s += metric[w][threadIdx.x];
        block_metrics[static_cast<size_t>(blockIdx.x) * ppo::kMetrics + threadIdx.x] = s;
    }
}

// The same objective with two samples per warp, one per half-warp (16 lanes, SLOTS logits per
// lane: k <= 16 * SLOTS), for k <= 128. (At k = 256 its 16 logits per lane took 128 registers,
// two blocks per SM, and it measured 3.33 ms against the one-sample warp's 3.18 ms over
// 4,194,304 samples, so k > 128 stays on k_logit_objective.) Reductions take four butterfly steps inside each half,
// and the per-sample work (the scalars, the ratio, the value loss, the metrics) is issued once
// for both samples, which matters because the kernel is bound by instruction issue. Each
// half-warp strides over sample pairs like the warps of k_logit_objective, with the next pair
// prefetched; the arithmetic per logit is that kernel's.
template <int SLOTS>
__global__ void __launch_bounds__(32 * ppo::kWarps) k_logit_objective_pair(
    const float* out, const uint8_t* masks, const int64_t* actions, const float* old_lp, const float* old_v,
    const float* adv, const float* ret, size_t n, int k, float inv_batch, float clip, float value_clip,
    float value_coef, float entropy_coef, float* grads, double* block_metrics) {
    __shared__ double metric[ppo::kWarps][ppo::kMetrics];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = lane >> 4, l = lane & 15;
    const unsigned full = 0xffffffffu;
    const size_t stride = static_cast<size_t>(gridDim.x) * ppo::kWarps * 2;
    double acc = 0.0;
    size_t i = (static_cast<size_t>(blockIdx.x) * ppo::kWarps + warp) * 2 + half;
    float next_logit[SLOTS] = {};
    uint8_t next_mask[SLOTS] = {};
    const auto load = [&](size_t row) {
        const float* o = out + row * static_cast<size_t>(k + 1);
        const uint8_t* m = masks + row * static_cast<size_t>(k);
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            const int a = j * 16 + l;
            next_logit[j] = a < k ? o[a] : 0.0f;
            next_mask[j] = a < k ? m[a] : 0;
        }
    };
    const auto half_sum = [](float v) {
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        return v;
    };
    const auto half_max = [](float v) {
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        return v;
    };
    if (i < n) load(i);
    // every lane runs every iteration (the shuffles span the warp); a half whose sample is past
    // the end computes on zeros and stores nothing
    for (size_t base = i - half; base < n; base += stride, i += stride) {
        const bool live = i < n;
        float logit[SLOTS];
        bool legal[SLOTS];
        unsigned legal_count = 0;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            logit[j] = next_logit[j];
            legal[j] = live && next_mask[j] != 0;
            legal_count += __popc((__ballot_sync(full, legal[j]) >> (16 * half)) & 0xffffu);
        }
        if (i + stride < n) load(i + stride);
        const size_t at = live ? i : 0;
        const int64_t action = actions[at];
        const float old_log = old_lp[at], a_i = adv[at], r_i = ret[at], v_old = old_v[at];
        const float v = out[at * static_cast<size_t>(k + 1) + k];
        const bool any = legal_count != 0;
        if (!any) {
            legal_count = 1;
#pragma unroll
            for (int j = 0; j < SLOTS; ++j) legal[j] = j * 16 + l == 0;
        }
        float local_max = -3.402823466e38f;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            if (legal[j]) local_max = fmaxf(local_max, logit[j]);
        }
        const float maximum = half_max(local_max);
        float e[SLOTS];
        float local = 0.0f;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            e[j] = legal[j] ? __expf(logit[j] - maximum) : 0.0f;
            local += e[j];
        }
        const float sum = fmaxf(half_sum(local), 1e-20f);
        const float inv_sum = 1.0f / sum;
        const float log_sum = logf(sum) + maximum;
        const int selected = any ? static_cast<int>(action) : 0;
        float mine_logit = 0.0f;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) mine_logit = j * 16 + l == selected ? logit[j] : mine_logit;
        const float chosen = __shfl_sync(full, mine_logit, (half << 4) | (selected & 15));
        const float log_ratio = (chosen - log_sum) - old_log;
        const float ratio = expf(log_ratio);
        const float unclipped = ratio * a_i;
        const float clipped = fminf(1.0f + clip, fmaxf(1.0f - clip, ratio)) * a_i;
        const float lp_grad = unclipped <= clipped ? -a_i * ratio : 0.0f;
        float entropy = 0.0f;
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            e[j] *= inv_sum;  // the probability
            entropy -= e[j] * (logit[j] - log_sum);
        }
        entropy = half_sum(entropy);
        const float policy_scale = lp_grad * inv_batch, entropy_scale = entropy_coef * inv_batch;
        const float shift = entropy - log_sum;
        if (live) {
            float* g = grads + i * static_cast<size_t>(k + 1);
#pragma unroll
            for (int j = 0; j < SLOTS; ++j) {
                const int a = j * 16 + l;
                if (a >= k) continue;
                const float onehot = a == selected ? 1.0f : 0.0f;
                g[a] = legal[j] ? policy_scale * (onehot - e[j]) + entropy_scale * e[j] * (logit[j] + shift) : 0.0f;
            }
        }
        const float error = v - r_i;
        float vgrad = error;
        float vloss = 0.5f * error * error;
        if (value_clip > 0.0f) {
            const float delta = v - v_old;
            const float cv = v_old + fminf(value_clip, fmaxf(-value_clip, delta));
            const float cerr = cv - r_i;
            const float closs = 0.5f * cerr * cerr;
            if (closs > vloss) {
                vloss = closs;
                vgrad = fabsf(delta) <= value_clip ? cerr : 0.0f;
            }
        }
        if (live && l == 0) grads[i * static_cast<size_t>(k + 1) + k] = value_coef * vgrad * inv_batch;
        const bool decision = legal_count > 1;
        const float mine = !live ? 0.0f
                         : l == 0 ? -fminf(unclipped, clipped)
                         : l == 1 ? vloss
                         : l == 2 ? entropy
                         : l == 3 ? (ratio - 1.0f) - log_ratio
                         : l == 4 ? (fabsf(ratio - 1.0f) > clip ? 1.0f : 0.0f)
                         : l == 6 ? (decision ? 1.0f : 0.0f)
                         : l == 7 ? (decision ? entropy : 0.0f)
                                  : 0.0f;
        acc += static_cast<double>(mine);
    }
    acc += __shfl_down_sync(full, acc, 16);  // the halves' sums, in fixed order
    if (lane < ppo::kMetrics) metric[warp][lane] = acc;
    __syncthreads();
    if (block_metrics != nullptr && threadIdx.x < ppo::kMetrics) {
        double sm = 0.0;
        for (int w = 0; w < ppo::kWarps; ++w) sm += metric[w][threadIdx.x];
        block_metrics[static_cast<size_t>(blockIdx.x) * ppo::kMetrics + threadIdx.x] = sm;
    }
}

// The objective's grid: the blocks that are resident at once (at most kObjectiveBlocksPerSm per
// SM, fewer when the instantiation's registers allow fewer), or fewer when n needs fewer.
unsigned objective_grid(size_t n) {
    const size_t blocks_needed = (n + 2 * ppo::kWarps - 1) / (2 * ppo::kWarps);
    return static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(blocks_needed,
                                                                        static_cast<size_t>(sm_count()) * kObjectiveBlocksPerSm)));
}

template <typename Kernel>
unsigned resident_grid(Kernel kernel, unsigned grid) {
    int per_sm = 0;
    check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 32 * ppo::kWarps, 0), "objective occupancy");
    return std::max(1u, std::min(grid, static_cast<unsigned>(std::max(per_sm, 1) * sm_count())));
}

// Launches the instantiation with the fewest logit slots per lane that holds k, on `grid` blocks
// at most; `partial` (when given) receives one row of metric partials per block launched, and the
// number of rows is returned.
unsigned launch_objective(cudaStream_t st, unsigned grid, const float* outputs, const uint8_t* masks,
                          const int64_t* actions, const float* old_lp, const float* old_v, const float* adv,
                          const float* ret, size_t n, int k, const t8b_ppo_config_t& c, float* gradients,
                          double* partial) {
    const float inv = 1.0f / static_cast<float>(n);
#define T8B_OBJECTIVE(KERNEL, SLOTS)                                                                                  \
    do {                                                                                                               \
        grid = resident_grid(KERNEL<SLOTS>, grid);                                                                     \
        launch("k_logit_objective", KERNEL<SLOTS>, grid, 32 * ppo::kWarps, 0, st, outputs, masks, actions, old_lp,      \
               old_v, adv, ret, n, k, inv, c.clip_range, c.value_clip_range, c.value_coefficient,                      \
               c.entropy_coefficient, gradients, partial);                                                             \
    } while (0)
    if (k <= 64) T8B_OBJECTIVE(k_logit_objective_pair, 4);
    else if (k <= 128) T8B_OBJECTIVE(k_logit_objective_pair, 8);
    else if (k <= 256) T8B_OBJECTIVE(k_logit_objective, 8);
    else if (k <= 384) T8B_OBJECTIVE(k_logit_objective, 12);
    else T8B_OBJECTIVE(k_logit_objective, 16);
#undef T8B_OBJECTIVE
    return grid;
}

// Scratch of t8b_ppo_output_gradient_static: the per-block metric partials (8 doubles per block;
// the objective's grid is at most kObjectiveBlocksPerSm blocks per SM, far below this array's
// 65,536 rows). One copy per device that loads the library, held until the process exits.
constexpr size_t kStaticObjectiveSamples = 524288;
constexpr size_t kStaticObjectiveBlocks = kStaticObjectiveSamples / ppo::kWarps;
static __device__ __align__(256) double g_objective_scratch[kStaticObjectiveBlocks * ppo::kMetrics];  // 4 MiB

// The library's stream-ordered memory pool on the current device (created once per device and
// kept until exit), for per-call scratch whose lifetime is one call's stream order. Its release
// threshold is unbounded, so freed blocks stay in the pool for the next call instead of going
// back to the driver at every synchronisation.
cudaMemPool_t scratch_pool() {
    int device = 0;
    check(cudaGetDevice(&device), "cudaGetDevice");
    static std::mutex lock;
    static cudaMemPool_t pools[128] = {};
    if (device < 0 || device >= 128) raise(T8B_ECUDA, "device index out of range");
    std::lock_guard<std::mutex> guard(lock);
    if (pools[device] == nullptr) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        check(cudaMemPoolCreate(&pools[device], &props), "cudaMemPoolCreate");
        uint64_t keep = UINT64_MAX;
        check(cudaMemPoolSetAttribute(pools[device], cudaMemPoolAttrReleaseThreshold, &keep), "pool threshold");
    }
    return pools[device];
}

// Device address of the scratch on the current device. The array's name is only a host-side
// stand-in in host code, so the address is asked for once per device (with that device
// current) and kept.
double* objective_scratch() {
    int device = 0;
    check(cudaGetDevice(&device), "cudaGetDevice");
    static std::mutex lock;
    static double* addresses[128] = {};
    if (device < 0 || device >= 128) raise(T8B_ECUDA, "device index out of range");
    std::lock_guard<std::mutex> guard(lock);
    if (addresses[device] == nullptr) {
        void* pointer = nullptr;
        check(cudaGetSymbolAddress(&pointer, g_objective_scratch), "cudaGetSymbolAddress of the objective scratch");
        addresses[device] = static_cast<double*>(pointer);
    }
    return addresses[device];
}

}  // namespace t8b

using namespace t8b;

struct t8b_rollout {
    size_t envs = 0, horizon = 0, samples = 0;
    int width = 0;
    int action_count = 0;  // candidates per sample (the uint8 mask row)
    Buffer<float> observations, log_probs, values, rewards, next_values, advantages, returns, entropies;
    Buffer<uint8_t> masks, terminated, truncated;
    Buffer<uint32_t> mask_bits;
    Buffer<int64_t> actions;
    Buffer<int32_t> tables;
    std::vector<uint8_t> entropy_recorded, bytes_current;
    Buffer<double> partial, stats;
    Buffer<float> discounted, return_samples;
    uint64_t return_count = 0;
    double return_mean = 0.0, return_variance = 1.0;
    t8b_comm_t comm{};
    bool comm_active() const { return comm.allreduce_sum_f64 != nullptr && comm.world_size > 1; }

    // One event per step, recorded on the stream of that step's record_policy_device after its
    // packed masks are written, so the uint8 expansion can wait for them whatever stream
    // recorded them.
    std::vector<cudaEvent_t> recorded;

    ~t8b_rollout() {
        for (cudaEvent_t e : recorded) {
            if (e != nullptr) cudaEventDestroy(e);
        }
    }

    void mark_recorded(size_t step, cudaStream_t stream) {
        if (recorded.empty()) recorded.assign(horizon, nullptr);
        if (recorded[step] == nullptr) check(cudaEventCreateWithFlags(&recorded[step], cudaEventDisableTiming), "event");
        check(cudaEventRecord(recorded[step], stream), "record event");
    }

    // uint8 masks materialised from the packed ones for the reference view, when stale. The
    // view has no stream argument (as the reference's device_view), so the expansion waits for
    // every stale step's recording, runs on the legacy stream and is complete on return; the
    // per-step flags are set only then.
    void expand_masks() {
        bool stale = false;
        for (uint8_t b : bytes_current) stale = stale || b == 0;
        if (!stale) return;
        if (masks.size() == 0) masks.allocate(samples * static_cast<size_t>(action_count));
        for (size_t step = 0; step < bytes_current.size(); ++step) {
            if (bytes_current[step] == 0 && !recorded.empty() && recorded[step] != nullptr) {
                check(cudaStreamWaitEvent(cudaStreamLegacy, recorded[step], 0), "wait for the recorded masks");
            }
        }
        launch("k_expand", k_expand, blocks(samples * static_cast<size_t>(action_count), 256), 256, 0, cudaStreamLegacy,
               mask_bits.data(), masks.data(), action_count, samples);
        check(cudaGetLastError(), "expand masks");
        check(cudaStreamSynchronize(cudaStreamLegacy), "expand masks");
        std::fill(bytes_current.begin(), bytes_current.end(), 1);
    }

    // (sum, sum of squares) of values[0..n) in fixed order -> stats[0..1], then the global totals
    void moments(const float* values, size_t n, cudaStream_t stream, void* raw_stream) {
        const int grid = static_cast<int>(std::min<size_t>(1024, (n + 255) / 256));
        launch("k_moments", k_moments, grid, 256, 0, stream, values, n, partial.data());
        launch("k_pair_total", k_pair_total, 1, 32, 0, stream, partial.data(), grid, stats.data());
        launch("k_set_count", k_set_count, 1, 32, 0, stream, stats.data(), static_cast<double>(n));
        check(cudaGetLastError(), "moments");
        if (comm_active()) comm.allreduce_sum_f64(stats.data(), 3, raw_stream, comm.user);
    }
};

namespace {

template <typename Body>
int with_rollout(t8b_rollout* r, Body&& body) {
    return guarded([&] {
        if (r == nullptr) raise(T8B_EINVAL, "null rollout handle");
        body(*r);
    });
}

}  // namespace

extern "C" {

int t8b_rollout_create(size_t environments, size_t horizon, const t8b_actor_config_t* config, t8b_rollout** out) {
    return guarded([&] {
        if (out == nullptr || config == nullptr) raise(T8B_EINVAL, "null argument");
        *out = nullptr;
        if (environments == 0 || horizon == 0) raise(T8B_EINVAL, "rollout dimensions must be greater than zero");
        auto r = std::make_unique<t8b_rollout>();
        r->envs = environments;
        r->horizon = horizon;
        r->samples = environments * horizon;
        r->width = config->observation_size;
        if (config->action_count < 2 || config->action_count > T8B_MAX_CANDIDATES) {
            raise(T8B_EINVAL, "action_count must be 2-368");
        }
        r->action_count = config->action_count;
        const size_t n = r->samples;
        r->observations.allocate(n * static_cast<size_t>(r->width));
        r->mask_bits.allocate(n * 12);
        r->actions.allocate(n);
        r->log_probs.allocate(n);
        r->values.allocate(n);
        r->rewards.allocate(n);
        r->terminated.allocate(n);
        r->truncated.allocate(n);
        r->next_values.allocate(n);
        r->advantages.allocate(n);
        r->returns.allocate(n);
        r->tables.allocate(n);
        r->entropies.allocate(n);
        r->entropy_recorded.assign(horizon, 0);
        r->bytes_current.assign(horizon, 0);
        r->partial.allocate(2 * 1024);
        r->stats.allocate(4);
        r->discounted.allocate(environments);
        r->return_samples.allocate(n);
        *out = r.release();
    });
}

int t8b_rollout_destroy(t8b_rollout* r) {
    return guarded([&] {
        if (r) cudaDeviceSynchronize();
        delete r;
    });
}

static int rollout_view(const t8b_rollout* rc, t8b_rollout_view_t* out, bool bytes) {
    t8b_rollout* r = const_cast<t8b_rollout*>(rc);
    return with_rollout(r, [&](t8b_rollout& s) {
        if (bytes) s.expand_masks();
        std::memset(out, 0, sizeof *out);
        out->observations = s.observations.data();
        out->action_masks = bytes ? s.masks.data() : nullptr;
        out->action_mask_bits = s.mask_bits.data();
        out->actions = s.actions.data();
        out->old_log_probabilities = s.log_probs.data();
        out->old_values = s.values.data();
        out->rewards = s.rewards.data();
        out->terminated = s.terminated.data();
        out->truncated = s.truncated.data();
        out->next_values = s.next_values.data();
        out->advantages = s.advantages.data();
        out->returns = s.returns.data();
        out->environment_count = s.envs;
        out->horizon = s.horizon;
        out->sample_count = s.samples;
        out->feature_tables = s.tables.data();
        bool all = true;
        for (uint8_t v : s.entropy_recorded) all = all && v;
        out->entropies = all ? s.entropies.data() : nullptr;
    });
}

int t8b_rollout_device_view(const t8b_rollout* r, t8b_rollout_view_t* out) { return rollout_view(r, out, true); }
int t8b_rollout_packed_view(const t8b_rollout* r, t8b_rollout_view_t* out) { return rollout_view(r, out, false); }

int t8b_rollout_record_policy_device(t8b_rollout* r, size_t step, const float* observations, const uint8_t* masks,
                                     const uint32_t* mask_bits, const int64_t* actions, const float* log_probabilities,
                                     const float* values, void* stream, const int32_t* feature_tables,
                                     const float* entropies) {
    return with_rollout(r, [&](t8b_rollout& s) {
        if (step >= s.horizon) raise(T8B_ERANGE, "rollout step exceeds horizon");
        if (!observations || (!masks && !mask_bits) || !actions || !log_probabilities || !values) {
            raise(T8B_EINVAL, "rollout device pointers cannot be null");
        }
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const size_t at = step * s.envs;
        const size_t n = s.envs;
        if (!mask_bits) {
            launch("k_pack_masks", k_pack_masks, blocks(n * 12, 256), 256, 0, st, masks, s.action_count, s.mask_bits.data() + at * 12, n);
            check(cudaGetLastError(), "pack masks");
        }
        RecordCopies r{};
        size_t words = 0;
        const auto add = [&](const void* src, void* dst, size_t bytes) {
            const bool wide = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | bytes) & 15u) == 0;
            r.src[r.count] = src;
            r.dst[r.count] = dst;
            r.wide[r.count] = wide ? 1 : 0;
            r.first[r.count] = words;
            words += bytes / (wide ? 16 : 4);
            r.first[++r.count] = words;
        };
        add(observations, s.observations.data() + at * s.width, sizeof(float) * n * s.width);
        if (mask_bits) add(mask_bits, s.mask_bits.data() + at * 12, sizeof(uint32_t) * n * 12);
        add(actions, s.actions.data() + at, sizeof(int64_t) * n);
        add(log_probabilities, s.log_probs.data() + at, sizeof(float) * n);
        add(values, s.values.data() + at, sizeof(float) * n);
        add(feature_tables, s.tables.data() + at, sizeof(int32_t) * n);  // null: zeros
        if (entropies) add(entropies, s.entropies.data() + at, sizeof(float) * n);
        const unsigned grid = static_cast<unsigned>(std::min<size_t>(blocks(words, 256), static_cast<size_t>(sm_count()) * 8));
        launch("k_record", k_record, grid, 256, 0, st, r);
        check(cudaGetLastError(), "record policy");
        s.bytes_current[step] = 0;
        s.mark_recorded(step, st);
        s.entropy_recorded[step] = entropies != nullptr;
    });
}

int t8b_rollout_record_outcome_device(t8b_rollout* r, size_t step, const float* rewards, const uint8_t* terminated,
                                      const uint8_t* truncated, const float* next_values, float reward_scale,
                                      void* stream) {
    return with_rollout(r, [&](t8b_rollout& s) {
        if (step >= s.horizon) raise(T8B_ERANGE, "rollout step exceeds horizon");
        if (!rewards || !terminated || !truncated || !next_values) raise(T8B_EINVAL, "outcome device pointers cannot be null");
        if (!std::isfinite(reward_scale) || reward_scale <= 0.0f) raise(T8B_EINVAL, "reward scale must be finite and positive");
        const size_t at = step * s.envs;
        launch("k_record_outcome", k_record_outcome, blocks(s.envs, 256), 256, 0, static_cast<cudaStream_t>(stream), 
            s.rewards.data() + at, s.terminated.data() + at, s.truncated.data() + at, s.next_values.data() + at, rewards,
            terminated, truncated, next_values, reward_scale, s.envs);
        check(cudaGetLastError(), "record outcome");
    });
}

}  // extern "C"

namespace t8b::internal {

void rollout_record_policy_rows(t8b_rollout* r, size_t step, size_t row, size_t n, const float* observations,
                                const uint32_t* mask_bits, const int64_t* actions, const float* log_probabilities,
                                const float* values, const int32_t* tables, const float* entropies, cudaStream_t st) {
    t8b_rollout& s = *r;
    if (step >= s.horizon || row + n > s.envs) raise(T8B_ERANGE, "rollout rows exceed the buffer");
    const size_t at = step * s.envs + row;
    const auto copy = [&](void* to, const void* from, size_t bytes, const char* what) {
        check(cudaMemcpyAsync(to, from, bytes, cudaMemcpyDeviceToDevice, st), what);
    };
    copy(s.observations.data() + at * s.width, observations + row * s.width, sizeof(float) * n * s.width, "observations");
    copy(s.mask_bits.data() + at * 12, mask_bits + row * 12, sizeof(uint32_t) * n * 12, "masks");
    copy(s.actions.data() + at, actions + row, sizeof(int64_t) * n, "actions");
    copy(s.log_probs.data() + at, log_probabilities + row, sizeof(float) * n, "log-probabilities");
    copy(s.values.data() + at, values + row, sizeof(float) * n, "values");
    copy(s.tables.data() + at, tables + row, sizeof(int32_t) * n, "tables");
    copy(s.entropies.data() + at, entropies + row, sizeof(float) * n, "entropies");
    s.bytes_current[step] = 0;
    s.entropy_recorded[step] = 1;
}

void rollout_record_outcome_rows(t8b_rollout* r, size_t step, size_t row, size_t n, const float* rewards,
                                 const uint8_t* terminated, const uint8_t* truncated, const float* next_values,
                                 float reward_scale, cudaStream_t st) {
    t8b_rollout& s = *r;
    if (step >= s.horizon || row + n > s.envs) raise(T8B_ERANGE, "rollout rows exceed the buffer");
    const size_t at = step * s.envs + row;
    launch("k_record_outcome", k_record_outcome, blocks(n, 256), 256, 0, st, s.rewards.data() + at,
           s.terminated.data() + at, s.truncated.data() + at, s.next_values.data() + at, rewards + row,
           terminated + row, truncated + row, next_values + row, reward_scale, n);
    check(cudaGetLastError(), "record outcome");
}

}  // namespace t8b::internal

extern "C" {

int t8b_rollout_compute_gae(t8b_rollout* r, float gamma, float gae_lambda, int normalize, void* stream) {
    return with_rollout(r, [&](t8b_rollout& s) {
        if (!std::isfinite(gamma) || !std::isfinite(gae_lambda) ||
            !(gamma >= 0.0f && gamma <= 1.0f && gae_lambda >= 0.0f && gae_lambda <= 1.0f)) {
            raise(T8B_EINVAL, "gamma and gae_lambda must be in [0, 1]");
        }
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const unsigned grid = blocks(s.envs, kGaeFights);
        if (s.partial.size() < 2 * static_cast<size_t>(grid)) s.partial.allocate(2 * static_cast<size_t>(grid));
        launch("k_gae", k_gae, grid, kGaeThreads, 0, st, s.rewards.data(), s.values.data(), s.terminated.data(), s.truncated.data(),
                                            s.next_values.data(), s.envs, s.horizon, gamma, gae_lambda, s.advantages.data(),
                                            s.returns.data(), s.partial.data());
        check(cudaGetLastError(), "GAE");
        if (normalize) {
            launch("k_pair_total", k_pair_total, 1, 32, 0, st, s.partial.data(), static_cast<int>(grid), s.stats.data());
            launch("k_set_count", k_set_count, 1, 32, 0, st, s.stats.data(), static_cast<double>(s.samples));
            if (s.comm_active()) s.comm.allreduce_sum_f64(s.stats.data(), 3, stream, s.comm.user);
            launch("k_normalize", k_normalize, blocks(s.samples, 256), 256, 0, st, s.advantages.data(), s.samples, s.stats.data());
            check(cudaGetLastError(), "normalize advantages");
        }
    });
}

// normalize_rewards (src/ppo.cu:2365-2406)
int t8b_rollout_normalize_rewards(t8b_rollout* r, float gamma, float clip, void* stream, float* std_out) {
    return with_rollout(r, [&](t8b_rollout& s) {
        if (!std::isfinite(gamma) || gamma < 0.0f || gamma > 1.0f) raise(T8B_EINVAL, "return normalization gamma must be in [0, 1]");
        if (!std::isfinite(clip) || clip <= 0.0f) raise(T8B_EINVAL, "return normalization clip must be finite and positive");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        launch("k_discounted", k_discounted, blocks(s.envs, 256), 256, 0, st, s.rewards.data(), s.terminated.data(), s.truncated.data(), s.envs,
                                                          s.horizon, gamma, s.discounted.data(), s.return_samples.data());
        s.moments(s.return_samples.data(), s.samples, st, stream);
        double sums[3];
        s.stats.download(sums, 3, st);
        const double batch_count = sums[2];
        const double batch_mean = sums[0] / batch_count;
        const double batch_m2 = std::max(0.0, sums[1] - sums[0] * batch_mean);
        if (!std::isfinite(batch_mean) || !std::isfinite(batch_m2)) {
            raise(T8B_ENONFINITE, "discounted returns became non-finite during return normalization");
        }
        const double running = static_cast<double>(s.return_count);
        const double total = running + batch_count;
        const double delta = batch_mean - s.return_mean;
        s.return_variance = (s.return_variance * running + batch_m2 + delta * delta * running * batch_count / total) / total;
        s.return_mean += delta * batch_count / total;
        s.return_count += static_cast<uint64_t>(batch_count);
        const float deviation = static_cast<float>(std::sqrt(s.return_variance + 1e-8));
        launch("k_scale_rewards", k_scale_rewards, blocks(s.samples, 256), 256, 0, st, s.rewards.data(), s.samples, 1.0f / deviation, clip);
        check(cudaGetLastError(), "scale rewards");
        if (std_out) *std_out = deviation;
    });
}

int t8b_rollout_mean_reward(t8b_rollout* r, void* stream, double* out) {
    return with_rollout(r, [&](t8b_rollout& s) {
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        s.moments(s.rewards.data(), s.samples, st, stream);
        double sums[3];
        s.stats.download(sums, 3, st);
        *out = sums[0] / sums[2];
    });
}

int t8b_rollout_return_normalizer_state(t8b_rollout* r, uint64_t* count, double* mean, double* variance,
                                        float* discounted_returns) {
    return with_rollout(r, [&](t8b_rollout& s) {
        if (count) *count = s.return_count;
        if (mean) *mean = s.return_mean;
        if (variance) *variance = s.return_variance;
        if (discounted_returns) s.discounted.download(discounted_returns, s.envs, nullptr);
    });
}

int t8b_rollout_restore_return_normalizer_state(t8b_rollout* r, uint64_t count, double mean, double variance,
                                                const float* discounted_returns) {
    return with_rollout(r, [&](t8b_rollout& s) {
        if (!std::isfinite(mean) || !std::isfinite(variance) || variance < 0.0) {
            raise(T8B_EINVAL, "return normalizer state is invalid for this rollout buffer");
        }
        for (size_t i = 0; i < s.envs; ++i) {
            if (!std::isfinite(discounted_returns[i])) raise(T8B_EINVAL, "return normalizer state is invalid for this rollout buffer");
        }
        s.discounted.upload(discounted_returns, s.envs, nullptr);
        check(cudaStreamSynchronize(nullptr), "restore return normalizer");
        s.return_count = count;
        s.return_mean = mean;
        s.return_variance = variance;
    });
}

int t8b_rollout_set_comm(t8b_rollout* r, const t8b_comm_t* comm) {
    return with_rollout(r, [&](t8b_rollout& s) { s.comm = comm ? *comm : t8b_comm_t{}; });
}

int t8b_rollout_synchronize(t8b_rollout* r, void* stream) {
    return with_rollout(r, [&](t8b_rollout&) { check(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "synchronize rollout"); });
}

int t8b_ppo_output_gradient(const float* outputs, const uint8_t* masks, const int64_t* actions,
                            const float* old_log_probabilities, const float* old_values, const float* advantages,
                            const float* returns, size_t n, int action_count, const t8b_ppo_config_t* config,
                            float* gradients, double* metric_sums, void* stream) {
    return guarded([&] {
        if (!outputs || !masks || !actions || !old_log_probabilities || !old_values || !advantages || !returns ||
            !gradients || !config || n == 0) {
            raise(T8B_EINVAL, "invalid PPO objective input");
        }
        if (action_count < 2 || action_count > 32 * kMaxLogitSlots) raise(T8B_EINVAL, "action_count must be 2..512");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        const unsigned grid = objective_grid(n);
        double* partial = nullptr;
        if (metric_sums) {
            // per-block metric partials from the library's stream-ordered pool: no device-wide
            // synchronisation, and the memory returns to the pool (not the driver) when freed
            check(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&partial),
                                          sizeof(double) * static_cast<size_t>(grid) * ppo::kMetrics, scratch_pool(), st),
                  "PPO objective partials");
        }
        const unsigned rows = launch_objective(st, grid, outputs, masks, actions, old_log_probabilities, old_values,
                                               advantages, returns, n, action_count, *config, gradients, partial);
        const cudaError_t launched = cudaGetLastError();
        if (metric_sums) {
            if (launched == cudaSuccess) {
                launch("k_sum_rows_f64", ppo::k_sum_rows_f64, ppo::kMetrics, 256, 0, st, partial, static_cast<int>(rows),
                       ppo::kMetrics, metric_sums, 0);
            }
            check(cudaFreeAsync(partial, st), "PPO objective partials");
        }
        check(launched, "PPO objective");
        check(cudaGetLastError(), "PPO objective metrics");
    });
}

// The raw-logits PPO objective without allocating device memory, for callers that cannot call
// cudaMalloc: a host whose memory manager owns all of the GPU's memory and forbids allocations
// outside it, or a training loop that must not pay the device-wide synchronisation cudaMalloc
// and cudaFree imply in the middle of a step. The per-block metric partials live in the static
// 4 MiB device array above instead of a buffer allocated per call. The first call on a device
// looks up the array's device address (cudaGetSymbolAddress); make that first call before any
// stream capture. Every call shares the one array, so calls that overlap on the GPU (two
// streams, two host threads) race on it; each call overwrites the partials it reads, so nothing
// needs clearing between calls. At most 524,288 samples per call. It returns once the work is
// queued, so results are ordered on `stream` only. The address is kept per device index, for the device's primary
// context: `stream` must belong to the current device.
int t8b_ppo_output_gradient_static(const float* outputs, const uint8_t* masks, const int64_t* actions,
                                   const float* old_log_probabilities, const float* old_values, const float* advantages,
                                   const float* returns, size_t n, int action_count, const t8b_ppo_config_t* config,
                                   float* gradients, double* metric_sums, void* stream) {
    return guarded([&] {
        if (!outputs || !masks || !actions || !old_log_probabilities || !old_values || !advantages || !returns ||
            !gradients || !config || n == 0) {
            raise(T8B_EINVAL, "invalid PPO objective input");
        }
        if (n > kStaticObjectiveSamples) {
            raise(T8B_EINVAL, "n exceeds the static scratch of this entry point (at most 524288 samples)");
        }
        if (action_count < 2 || action_count > 32 * kMaxLogitSlots) raise(T8B_EINVAL, "action_count must be 2..512");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        double* scratch = metric_sums ? objective_scratch() : nullptr;
        const unsigned grid = objective_grid(n);
        const unsigned rows = launch_objective(st, grid, outputs, masks, actions, old_log_probabilities, old_values,
                                               advantages, returns, n, action_count, *config, gradients, scratch);
        check(cudaGetLastError(), "PPO objective");
        if (metric_sums) {
            launch("k_sum_rows_f64", ppo::k_sum_rows_f64, ppo::kMetrics, 256, 0, st, scratch, static_cast<int>(rows), ppo::kMetrics,
                                                               metric_sums, 0);
            check(cudaGetLastError(), "PPO objective metrics");
        }
    });
}

}  // extern "C"
