// SIMT kernels of the policy and PPO update around the tcgen05 GEMMs: input preparation
// (normalisation, minibatch gather), the parametric scorer fused with masked sampling or with
// the clipped PPO objective and its gradient, the tanh/bias epilogues of the GEMMs, split-K and
// bias-gradient reductions, the global gradient norm and Adam. Every reduction that feeds
// weights or control decisions runs in a fixed order, so an update is bit-reproducible.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "gemm.cuh"

namespace t8b {
namespace ppo {
namespace {  // internal linkage: every translation unit gets its own kernels

constexpr int kWarps = 8;  // warps per block of the warp-per-sample kernels
constexpr int kMaskWords = 12;
constexpr int kCandidates = 368;
constexpr int kMetrics = 8;  // policy loss, value loss, entropy, KL, clip fraction, grad norm, decisions, decision entropy

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ uint64_t splitmix(uint64_t v) {
    v += 0x9e3779b97f4a7c15ull;
    v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
    v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
    return v ^ (v >> 31);
}
// uniform01 (src/ppo.cu:224-230)
__device__ __forceinline__ float uniform01(uint64_t seed, uint64_t step, uint64_t lane) {
    const uint64_t bits = splitmix(seed ^ splitmix(step) ^ splitmix(lane));
    return static_cast<float>(static_cast<double>(bits >> 40) + 0.5) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ------------------------------------------------------------------ inputs
// Normalised (src/ppo.cu:132-145), clipped, bf16, zero-padded rows of the layer-1 operand;
// with `perm` the rows are gathered (src/ppo.cu:383-421) and the minibatch side data follows.
struct Prep {
    const float* obs;
    int width, padded;  // observation floats, padded operand row
    const float* mean;
    const float* istd;
    float clip;
    int normalize;
    const uint32_t* perm;  // null: identity
    size_t offset, count;
    __nv_bfloat16* x;
    // minibatch side data (null when preparing an inference batch)
    const uint32_t* src_bits;
    const uint8_t* src_bytes;  // [samples][action_count]
    int action_count;          // candidates per sample (the mask row of src_bytes)
    uint32_t* bits;
    const int64_t* src_actions;
    int32_t* actions;
    const float* src_old_lp;
    float* old_lp;
    const float* src_old_v;
    float* old_v;
    const float* src_adv;
    float* adv;
    const float* src_ret;
    float* ret;
    const int32_t* src_tables;
    int32_t* tables;
    const double* adv_stats;  // [mean, inverse std] applied to advantages when non-null
};

__global__ void k_prep(Prep p) {
    const int lane = threadIdx.x & 31;
    const size_t i = static_cast<size_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    if (i >= p.count) return;
    const size_t src = p.perm ? p.perm[p.offset + i] : p.offset + i;
    const float* row = p.obs + src * static_cast<size_t>(p.width);
    __nv_bfloat16* out = p.x + i * static_cast<size_t>(p.padded);
    // the row's first 256 columns: every load issued before the first use
    constexpr int kHeld = 8;
    float held[kHeld];
#pragma unroll
    for (int k = 0; k < kHeld; ++k) {
        const int j = lane + 32 * k;
        held[k] = j < p.width ? row[j] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kHeld; ++k) {
        const int j = lane + 32 * k;
        if (j >= p.padded) break;
        float v = held[k];
        if (j < p.width && p.normalize) v = fminf(p.clip, fmaxf(-p.clip, (v - p.mean[j]) * p.istd[j]));
        out[j] = __float2bfloat16_rn(v);
    }
    for (int j = lane + 32 * kHeld; j < p.padded; j += 32) {
        float v = 0.0f;
        if (j < p.width) {
            v = row[j];
            if (p.normalize) v = fminf(p.clip, fmaxf(-p.clip, (v - p.mean[j]) * p.istd[j]));
        }
        out[j] = __float2bfloat16_rn(v);
    }
    if (p.bits != nullptr) {
        if (lane < kMaskWords) {
            uint32_t w;
            if (p.src_bits) {
                w = p.src_bits[src * kMaskWords + lane];
            } else {
                w = 0;
                const uint8_t* m = p.src_bytes + src * p.action_count + lane * 32;
                for (int b = 0; b < 32 && lane * 32 + b < p.action_count; ++b) w |= (m[b] != 0 ? 1u : 0u) << b;
            }
            p.bits[i * kMaskWords + lane] = w;
        }
        if (lane == 0) {
            p.actions[i] = static_cast<int32_t>(p.src_actions[src]);
            p.old_lp[i] = p.src_old_lp[src];
            p.old_v[i] = p.src_old_v[src];
            float a = p.src_adv[src];
            if (p.adv_stats) a = static_cast<float>((static_cast<double>(a) - p.adv_stats[0]) * p.adv_stats[1]);
            p.adv[i] = a;
            p.ret[i] = p.src_ret[src];
            p.tables[i] = p.src_tables ? p.src_tables[src] : 0;
        }
    }
}

// The minibatch gather of update_ppo: k_prep's work for kGatherRows consecutive minibatch rows
// per warp. The rows' source indices come from one load per lane, and every row's loads are
// issued before any is used, so a warp keeps several random rows in flight; lane r carries row
// r's per-sample scalars. The same arithmetic as k_prep, element for element.
constexpr int kGatherRows = 4;
constexpr int kGatherHeld = 8;  // columns a lane holds per row (the first 256 of the row)

__global__ void __launch_bounds__(32 * kWarps) k_gather(Prep p) {
    const int lane = threadIdx.x & 31;
    const size_t first = (static_cast<size_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5)) * kGatherRows;
    if (first >= p.count) return;
    size_t mine = 0;
    if (lane < kGatherRows && first + lane < p.count) mine = p.perm ? p.perm[p.offset + first + lane] : p.offset + first + lane;
    size_t src[kGatherRows];
    bool live[kGatherRows];
#pragma unroll
    for (int r = 0; r < kGatherRows; ++r) {
        src[r] = __shfl_sync(0xffffffffu, mine, r);
        live[r] = first + r < p.count;
    }
    float held[kGatherRows][kGatherHeld];
#pragma unroll
    for (int r = 0; r < kGatherRows; ++r) {
        const float* row = p.obs + src[r] * static_cast<size_t>(p.width);
#pragma unroll
        for (int k = 0; k < kGatherHeld; ++k) {
            const int j = lane + 32 * k;
            held[r][k] = live[r] && j < p.width ? row[j] : 0.0f;
        }
    }
    uint32_t words[kGatherRows];
#pragma unroll
    for (int r = 0; r < kGatherRows; ++r) {
        words[r] = 0;
        if (live[r] && lane < kMaskWords) {
            if (p.src_bits) {
                words[r] = p.src_bits[src[r] * kMaskWords + lane];
            } else {
                const uint8_t* m = p.src_bytes + src[r] * p.action_count + lane * 32;
                for (int b = 0; b < 32 && lane * 32 + b < p.action_count; ++b) words[r] |= (m[b] != 0 ? 1u : 0u) << b;
            }
        }
    }
    const bool carries = lane < kGatherRows && first + lane < p.count;
    int32_t action = 0, table = 0;
    float old_lp = 0.0f, old_v = 0.0f, advantage = 0.0f, ret = 0.0f;
    if (carries) {
        action = static_cast<int32_t>(p.src_actions[mine]);
        old_lp = p.src_old_lp[mine];
        old_v = p.src_old_v[mine];
        advantage = p.src_adv[mine];
        ret = p.src_ret[mine];
        table = p.src_tables ? p.src_tables[mine] : 0;
    }
#pragma unroll
    for (int r = 0; r < kGatherRows; ++r) {
        if (!live[r]) break;
        __nv_bfloat16* out = p.x + (first + r) * static_cast<size_t>(p.padded);
#pragma unroll
        for (int k = 0; k < kGatherHeld; ++k) {
            const int j = lane + 32 * k;
            if (j >= p.padded) break;
            float v = held[r][k];
            if (j < p.width && p.normalize) v = fminf(p.clip, fmaxf(-p.clip, (v - p.mean[j]) * p.istd[j]));
            out[j] = __float2bfloat16_rn(v);
        }
        const float* row = p.obs + src[r] * static_cast<size_t>(p.width);
        for (int j = lane + 32 * kGatherHeld; j < p.padded; j += 32) {
            float v = 0.0f;
            if (j < p.width) {
                v = row[j];
                if (p.normalize) v = fminf(p.clip, fmaxf(-p.clip, (v - p.mean[j]) * p.istd[j]));
            }
            out[j] = __float2bfloat16_rn(v);
        }
        if (lane < kMaskWords) p.bits[(first + r) * kMaskWords + lane] = words[r];
    }
    if (carries) {
        const size_t i = first + lane;
        p.actions[i] = action;
        p.old_lp[i] = old_lp;
        p.old_v[i] = old_v;
        float a = advantage;
        if (p.adv_stats) a = static_cast<float>((static_cast<double>(a) - p.adv_stats[0]) * p.adv_stats[1]);
        p.adv[i] = a;
        p.ret[i] = ret;
        p.tables[i] = table;
    }
}

// ------------------------------------------------------------------ GEMM epilogues
// A bf16 chunk (the warp's 32 rows x 32 columns) is staged in one of two 2 KB tiles of the warp's
// scratch (at 4096 and 6144, alternating chunk by chunk), each lane writing its row's 64 bytes
// with the 16-byte pieces rotated as the 64-byte TMA swizzle lays them out (tc::staged_piece), and
// leaves as one TMA store issued by lane 0 through `map` (a [rows][ld] bf16 tensor, 32 x 32
// boxes, 64-byte swizzle; rows past the tensor are not written). A tile is restaged once the
// store that last read it has finished reading. A warp whose rows all lie at or past row m (the
// padding of the last row tile) stores nothing and lets its earlier stores finish reading first.
constexpr int kTmaStoreScratch = 8704;  // prefetch 4096 + two staging tiles + 512
__device__ __forceinline__ void store_rows_bf16(const tc::EpiCtx& x, const uint32_t* packed, const CUtensorMap* map,
                                                int m) {
    unsigned char* stage = x.scratch + 4096 + (x.chunk & 1) * 2048;
    if (x.row0 >= m) {
        if (x.lane == 0) tc::bulk_wait_read();
        __syncwarp();
        return;
    }
    if (x.lane == 0) tc::bulk_wait_read_all_but_one();
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        *reinterpret_cast<uint4*>(stage + tc::staged_piece(x.lane, q, 4)) =
            make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (x.lane == 0) {
        tc::tma_store(map, stage, x.col0, x.row0);
        tc::bulk_commit();
    }
}

// The chunk's 32 bias values, fetched asynchronously into the scratch at `at` (one 128 B
// buffer per prefetch buffer); columns at or past `valid` read as zero.
__device__ __forceinline__ void prefetch_bias(const tc::EpiCtx& x, const float* bias, int valid, int at) {
    float* dst = reinterpret_cast<float*>(x.scratch + at + x.buffer * 128);
    const bool ok = x.col0 + x.lane < valid;
    tc::cp_async4(dst + x.lane, ok ? bias + x.col0 + x.lane : bias, ok);
    tc::cp_async_commit();
}
__device__ __forceinline__ void wait_prefetch(const tc::EpiCtx& x) {
    if (x.more) tc::cp_async_wait<1>(); else tc::cp_async_wait<0>();
    __syncwarp();
}

// Hidden layer forward: h = tanh(acc + b) as bf16 [rows][ld].
struct EpiTanh {
    static constexpr int kEpilogueWarps = 8;
    static constexpr int kScratchBytes = kTmaStoreScratch;
    const float* bias;
    CUtensorMap out;  // the bf16 [rows][ld] output (store_rows_bf16)
    int ld, m, cols;
    __device__ void prefetch(const tc::EpiCtx& x) const { prefetch_bias(x, bias, cols, 0); }
    __device__ void operator()(const tc::EpiCtx& x, const float* v) const {
        wait_prefetch(x);
        const float4* b = reinterpret_cast<const float4*>(x.scratch + x.buffer * 128);
        uint32_t packed[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 bq = b[q];
            __nv_bfloat162 lo = __floats2bfloat162_rn(tanh_fast(v[4 * q] + bq.x), tanh_fast(v[4 * q + 1] + bq.y));
            __nv_bfloat162 hi = __floats2bfloat162_rn(tanh_fast(v[4 * q + 2] + bq.z), tanh_fast(v[4 * q + 3] + bq.w));
            packed[2 * q] = *reinterpret_cast<uint32_t*>(&lo);
            packed[2 * q + 1] = *reinterpret_cast<uint32_t*>(&hi);
        }
        store_rows_bf16(x, packed, &out, m);
    }
};

// Output layer: o = acc + b for the valid columns (zero beyond), fp32 [rows][ld].
struct EpiBias {
    static constexpr int kEpilogueWarps = 8;
    static constexpr int kScratchBytes = tc::kEpiWarpBytes;
    const float* bias;
    float* out;
    int ld, m, valid;
    __device__ void prefetch(const tc::EpiCtx& x) const { prefetch_bias(x, bias, valid, 6144); }
    __device__ void operator()(const tc::EpiCtx& x, const float* v) const {
        wait_prefetch(x);
        const float4* b = reinterpret_cast<const float4*>(x.scratch + 6144 + x.buffer * 128);
        unsigned char* stage = x.scratch;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 bq = b[q];
            const int c = x.col0 + 4 * q;
            const float4 o = make_float4(c < valid ? v[4 * q] + bq.x : 0.0f, c + 1 < valid ? v[4 * q + 1] + bq.y : 0.0f,
                                         c + 2 < valid ? v[4 * q + 2] + bq.z : 0.0f, c + 3 < valid ? v[4 * q + 3] + bq.w : 0.0f);
            *reinterpret_cast<float4*>(stage + tc::staged_piece(x.lane, q, 8)) = o;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (x.lane >> 3), q = x.lane & 7;
            const float4 piece = *reinterpret_cast<const float4*>(stage + tc::staged_piece(r, q, 8));
            if (x.row0 + r < m) *reinterpret_cast<float4*>(out + static_cast<size_t>(x.row0 + r) * ld + x.col0 + q * 4) = piece;
        }
        __syncwarp();
    }
};

// Backward through tanh: dz = g (1 - h^2) as bf16, and per (row tile, lane quarter) column
// sums of dz (the bias gradient, reduced later in a fixed order). The h chunk is prefetched
// with cp.async into one of two 2 KB buffers while the previous chunk is processed.
struct EpiTanhGrad {
    static constexpr int kEpilogueWarps = 8;
    static constexpr int kScratchBytes = kTmaStoreScratch;
    const __nv_bfloat16* h;
    CUtensorMap out;  // the bf16 [rows][ld] gradient (store_rows_bf16)
    float* colsum;
    int ld, m;
    __device__ void prefetch(const tc::EpiCtx& x) const {
        unsigned char* buf = x.scratch + x.buffer * 2048;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = i * 8 + (x.lane >> 2), q = x.lane & 3;
            const bool valid = x.row0 + r < m;
            const __nv_bfloat16* src = valid ? h + static_cast<size_t>(x.row0 + r) * ld + x.col0 + q * 8 : h;
            tc::cp_async16(buf + tc::staged_piece(r, q, 4), src, valid);
        }
        tc::cp_async_commit();
    }
    __device__ void operator()(const tc::EpiCtx& x, const float* v) const {
        wait_prefetch(x);
        const unsigned char* buf = x.scratch + x.buffer * 2048;
        const bool live = x.row < m;
        float g[32];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint4 piece = *reinterpret_cast<const uint4*>(buf + tc::staged_piece(x.lane, q, 4));
            const uint32_t w[4] = {piece.x, piece.y, piece.z, piece.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
                g[8 * q + 2 * k] = live ? v[8 * q + 2 * k] * (1.0f - f.x * f.x) : 0.0f;
                g[8 * q + 2 * k + 1] = live ? v[8 * q + 2 * k + 1] * (1.0f - f.y * f.y) : 0.0f;
            }
        }
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            __nv_bfloat162 pair = __floats2bfloat162_rn(g[2 * i], g[2 * i + 1]);
            packed[i] = *reinterpret_cast<uint32_t*>(&pair);
        }
        store_rows_bf16(x, packed, &out, m);
        // Transpose-reduce across the warp: after 5 halving steps lane c holds column c's sum.
#pragma unroll
        for (int width = 16; width >= 1; width >>= 1) {
            const bool upper = (x.lane & width) != 0;
#pragma unroll
            for (int i = 0; i < width; ++i) {
                const float send = upper ? g[i] : g[i + width];
                const float keep = upper ? g[i + width] : g[i];
                g[i] = keep + __shfl_xor_sync(0xffffffffu, send, width);
            }
        }
        colsum[(static_cast<size_t>(x.tm) * 4 + x.quarter) * ld + x.col0 + x.lane] = g[0];
    }
};

// Split-K partial of a weight gradient: part[split][row][col] (fp32).
struct EpiSplit {
    static constexpr int kEpilogueWarps = 4;
    static constexpr int kScratchBytes = 0;
    __device__ void prefetch(const tc::EpiCtx&) const {}
    float* part;
    int m, n;
    __device__ void operator()(const tc::EpiCtx& x, const float* v) const {
        if (x.row >= m) return;
        float* out = part + (static_cast<size_t>(x.split) * m + x.row) * n + x.col0;
#pragma unroll
        for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(out + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
};

// grad[r][c] (reference layout, rows x cols, cols <= part cols) = sum over splits in order;
// transpose: the partial is [cols][rows] (the weight gradient came out transposed).
__global__ void k_reduce_split(const float* part, int splits, int part_rows, int part_cols, float* grad, int rows,
                               int cols, int transpose) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * cols) return;
    const int r = i / cols, c = i % cols;
    const size_t at = transpose ? static_cast<size_t>(c) * part_cols + r : static_cast<size_t>(r) * part_cols + c;
    const size_t stride = static_cast<size_t>(part_rows) * part_cols;
    float sum = 0.0f;
    for (int s = 0; s < splits; ++s) sum += part[s * stride + at];
    grad[i] = sum;
}

// Bias gradient = column sums of the per-32-row partials, in row order.
__global__ void k_reduce_columns(const float* partial, int rows, int ld, int cols, float* grad) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    float sum = 0.0f;
    for (int r = 0; r < rows; ++r) sum += partial[static_cast<size_t>(r) * ld + c];
    grad[c] = sum;
}

// Column sums of a [rows][ld] fp32 matrix in two fixed-order levels: each block sums 32 columns
// over one row chunk (8 interleaved sub-rows, combined in order), then one pass over the chunks.
constexpr int kColumnChunks = 128;
__global__ void k_column_partials(const float* in, int rows, int ld, int cols, float* partial) {
    __shared__ float part[8][33];
    const int c = blockIdx.x * 32 + threadIdx.x;
    const int per = (rows + gridDim.y - 1) / gridDim.y;
    const int begin = blockIdx.y * per;
    const int end = min(rows, begin + per);
    float s = 0.0f;
    if (c < cols) {
        for (int r = begin + threadIdx.y; r < end; r += 8) s += in[static_cast<size_t>(r) * ld + c];
    }
    part[threadIdx.y][threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.y == 0 && c < cols) {
        float t = 0.0f;
        for (int k = 0; k < 8; ++k) t += part[k][threadIdx.x];
        partial[static_cast<size_t>(blockIdx.y) * cols + c] = t;
    }
}

__global__ void k_scale(float* v, size_t n, float factor) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) v[i] *= factor;
}

// ------------------------------------------------------------------ scorer + sampler
// parametric_policy_output_kernel + masked_sample_kernel (src/ppo.cu:316-348, 232-306): one warp
// per sample; scores q . F[table, a] / sqrt(F) only where needed, masked softmax, inverse-CDF
// sample, log-probability, value and entropy.
struct Sample {
    const float* out;  // [n][ld]: q (feature_size), value
    int ld, feature_size;
    int action_count;       // candidates per sample (at most 368)
    const float* features;  // [tables][action_count][feature_size]
    int table_count;
    const int32_t* tables;
    const uint32_t* bits;   // [n][12] or null
    const uint8_t* bytes;   // [n][action_count] or null
    size_t count;
    uint64_t seed, step, lane_offset;
    int deterministic;
    unsigned parts;  // blocks per table group (k_sample's grid is groups x parts)
    float* logits;  // [n][368] or null
    int64_t* actions;
    float* log_probs;
    float* values;
    float* entropies;
};

// Feature sizes the scorer kernels are built for: the full-move tables' 32
// (kFullMoveFeatureSize, include/t8_v2/full_move_roster.hpp:21) and 48.
constexpr int kFeatures = 32;
constexpr int kMaxFeatures = 48;
constexpr int kMaxTableBytes = kCandidates * kMaxFeatures * 4;

// Chunk k (4 floats) of candidate c's feature row in the staged table: chunks are rotated by
// the row (an xor for 8 chunks, a cyclic shift otherwise) so that lanes reading different rows
// at the same chunk spread over the banks.
template <int F>
__device__ __forceinline__ int staged_slot(int c, int k) {
    constexpr int chunks = F / 4;
    return c * chunks + (chunks == 8 ? (k ^ (c & 7)) : (k + c) % chunks);
}
template <int F>
__device__ __forceinline__ float4 staged_chunk(const float4* table, int c, int k) {
    return table[staged_slot<F>(c, k)];
}
// q . F[a] in feature order, then scaled (src/ppo.cu:340-346).
template <int F>
__device__ __forceinline__ float staged_score(const float* q, const float4* table, int c, float scale) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < F / 4; ++k) {
        const float4 f = staged_chunk<F>(table, c, k);
        s += q[4 * k] * f.x;
        s += q[4 * k + 1] * f.y;
        s += q[4 * k + 2] * f.z;
        s += q[4 * k + 3] * f.w;
    }
    return s * scale;
}

// 32 per-lane vectors -> lane f holds the warp sum of element f.
__device__ __forceinline__ float transpose_sum32(float* g, int lane) {
#pragma unroll
    for (int width = 16; width >= 1; width >>= 1) {
        const bool upper = (lane & width) != 0;
#pragma unroll
        for (int i = 0; i < width; ++i) {
            const float send = upper ? g[i] : g[i + width];
            const float keep = upper ? g[i + width] : g[i];
            g[i] = keep + __shfl_xor_sync(0xffffffffu, send, width);
        }
    }
    return g[0];
}

// The legal candidates of one sample, ascending, compacted into `list` by ballots (12 words
// held by every lane); returns how many. Nothing legal: candidate 0 alone (src/ppo.cu:254-258).
__device__ __forceinline__ int compact_legal(const uint32_t* words, bool any, int lane, int16_t* list) {
    int count = 0;
    if (!any) {
        if (lane == 0) list[0] = 0;
        count = 1;
    } else {
#pragma unroll
        for (int w = 0; w < kMaskWords; ++w) {
            const uint32_t bits = words[w];
            if ((bits >> lane) & 1u) list[count + __popc(bits & ((1u << lane) - 1u))] = static_cast<int16_t>(w * 32 + lane);
            count += __popc(bits);
        }
    }
    __syncwarp();
    return count;
}

// Position of candidate c in the compacted list.
__device__ __forceinline__ int legal_rank(const uint32_t* words, bool any, int c) {
    if (!any) return 0;
    int rank = 0;
#pragma unroll
    for (int w = 0; w < kMaskWords; ++w) {
        if (w < (c >> 5)) rank += __popc(words[w]);
    }
    return rank + __popc(words[(c >> 5) % kMaskWords] & ((1u << (c & 31)) - 1u));
}

// k_sample's shape: 16 warps per block; a block gathers up to kSampleFound of its samples before
// scoring them, checking kSampleUnroll table indices per thread per gathering round.
constexpr int kSampleWarps = 16;
constexpr int kSampleFound = 4096;
constexpr int kSampleUnroll = 4;

// Dynamic shared memory of k_sample: the block's feature table, then the gathered sample indices.
inline size_t sample_smem(int features) {
    return static_cast<size_t>(features) * kCandidates * sizeof(float) + kSampleFound * sizeof(uint32_t);
}

// One sample's global inputs, loaded a sample ahead: lane w < 12 holds packed mask word w
// (bits) or each lane its candidate's mask byte per word (bytes), and the output row's q and
// value (lane f: elements f and 32 + f).
struct SampleInputs {
    uint32_t raw[kMaskWords];
    float q_lo, q_hi;
};

__device__ __forceinline__ void load_sample(const Sample& p, size_t i, int lane, SampleInputs& in) {
    const float* o = p.out + i * p.ld;
    in.q_lo = lane <= p.feature_size ? o[lane] : 0.0f;
    in.q_hi = lane + 32 <= p.feature_size ? o[lane + 32] : 0.0f;
    if (p.bits) {
        in.raw[0] = lane < kMaskWords ? p.bits[i * kMaskWords + lane] : 0u;
    } else {
#pragma unroll
        for (int w = 0; w < kMaskWords; ++w) {
            const int c = w * 32 + lane;
            in.raw[w] = c < p.action_count ? p.bytes[i * p.action_count + c] : 0u;
        }
    }
}

// One sample, one warp: the scores of the legal candidates, the masked softmax, the
// inverse-CDF draw (argmax when deterministic), log-probability, value and entropy.
template <int F>
__device__ __forceinline__ void sample_one(const Sample& p, size_t i, int lane, const SampleInputs& in, float* q,
                                           int16_t* list, float* sc, const float4* table, bool bad_table) {
    q[lane] = in.q_lo;
    if (lane + 32 <= p.feature_size) q[lane + 32] = in.q_hi;
    __syncwarp();
    const float scale = rsqrtf(static_cast<float>(p.feature_size));
    uint32_t words[kMaskWords];
    bool any = false;
#pragma unroll
    for (int w = 0; w < kMaskWords; ++w) {
        words[w] = p.bits ? __shfl_sync(0xffffffffu, in.raw[0], w) : __ballot_sync(0xffffffffu, in.raw[w] != 0u);
        any = any || words[w] != 0;
    }
    if (p.logits) {
        for (int c = lane; c < p.action_count; c += 32) {
            p.logits[i * p.action_count + c] =
                bad_table ? __int_as_float(0x7fc00000) : staged_score<F>(q, table, c, scale);
        }
    }
    const int count = compact_legal(words, any, lane, list);
    // scores of the legal candidates; argmax = largest score, then the lowest candidate
    float best = -3.402823466e38f;
    int best_j = kCandidates;
    for (int j = lane; j < count; j += 32) {
        const float s = bad_table ? __int_as_float(0x7fc00000) : staged_score<F>(q, table, list[j], scale);
        sc[j] = s;
        if (s > best || best_j == kCandidates) {
            best = s;
            best_j = j;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, off);
        const int oj = __shfl_xor_sync(0xffffffffu, best_j, off);
        if (ob > best || (ob == best && oj < best_j)) {
            best = ob;
            best_j = oj;
        }
    }
    __syncwarp();
    const float maximum = best;
    float local = 0.0f;
    for (int j = lane; j < count; j += 32) local += expf(sc[j] - maximum);
    const float sum = fmaxf(warp_sum(local), 1e-20f);
    int selected_j = best_j;
    if (!p.deterministic) {
        // inverse CDF in candidate order (src/ppo.cu:271-284)
        const float target = uniform01(p.seed, p.step, i + p.lane_offset) * sum;
        float running = 0.0f;
        int found = -1;
        for (int base = 0; base < count && found < 0; base += 32) {
            const int j = base + lane;
            const float e = j < count ? expf(sc[j] - maximum) : 0.0f;
            float x = e;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, off);
                if (lane >= off) x += y;
            }
            const uint32_t hit = __ballot_sync(0xffffffffu, j < count && target <= running + x);
            if (hit) found = base + __ffs(hit) - 1;
            running += __shfl_sync(0xffffffffu, x, 31);
        }
        if (found >= 0) selected_j = found;
    }
    const float log_sum = logf(sum) + maximum;
    float entropy = 0.0f;
    for (int j = lane; j < count; j += 32) {
        const float lp = sc[j] - log_sum;
        entropy -= expf(lp) * lp;
    }
    entropy = warp_sum(entropy);
    if (lane == 0) {
        p.actions[i] = list[selected_j];
        p.log_probs[i] = sc[selected_j] - log_sum;
        p.values[i] = bad_table ? __int_as_float(0x7fc00000) : q[p.feature_size];
        p.entropies[i] = entropy;
    }
    __syncwarp();
}

// The forward's sampler (src/ppo.cu:238-300), one warp per sample. Each block owns one feature
// table (p.parts blocks per table, sample i going to part i % p.parts; with tables given, one
// more group takes the samples whose table index is out of range and gives them NaN scores):
// it stages the table in shared memory once (staged_slot layout) and gathers its samples by
// scanning the table indices, so scoring reads shared memory instead of streaming every
// sample's feature rows from L2. A warp loads its next sample's inputs while it scores the
// current one.
template <int F>
__global__ void __launch_bounds__(32 * kSampleWarps) k_sample(Sample p) {
    extern __shared__ __align__(16) unsigned char dynamic_smem[];
    float4* table = reinterpret_cast<float4*>(dynamic_smem);
    uint32_t* found = reinterpret_cast<uint32_t*>(table + kCandidates * (F / 4));
    __shared__ float qs[kSampleWarps][64];
    __shared__ int16_t lists[kSampleWarps][kCandidates];
    __shared__ float scores[kSampleWarps][kCandidates];
    __shared__ unsigned found_count;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int group = static_cast<int>(blockIdx.x / p.parts);
    const size_t part = blockIdx.x % p.parts;
    const bool bad_group = p.tables != nullptr && group == p.table_count;
    if (!bad_group) {
        const float4* src = reinterpret_cast<const float4*>(p.features + static_cast<size_t>(group) * p.action_count * F);
        for (int idx = threadIdx.x; idx < p.action_count * (F / 4); idx += blockDim.x) {
            table[staged_slot<F>(idx / (F / 4), idx % (F / 4))] = __ldg(src + idx);
        }
    }
    if (threadIdx.x == 0) found_count = 0;
    __syncthreads();
    // this part's samples are i = part + t * parts, t < per_part
    const size_t per_part = p.count > part ? (p.count - part + p.parts - 1) / p.parts : 0;
    const size_t round = static_cast<size_t>(blockDim.x) * kSampleUnroll;
    size_t t0 = 0;
    for (;;) {
        while (t0 < per_part && found_count + round <= kSampleFound) {
            size_t index[kSampleUnroll];
            int key[kSampleUnroll];
#pragma unroll
            for (int u = 0; u < kSampleUnroll; ++u) {
                const size_t t = t0 + threadIdx.x + static_cast<size_t>(u) * blockDim.x;
                index[u] = part + t * p.parts;
                key[u] = -1;
                if (t < per_part) {
                    const int table_index = p.tables ? p.tables[index[u]] : 0;
                    key[u] = p.tables && (table_index < 0 || table_index >= p.table_count) ? p.table_count : table_index;
                }
            }
#pragma unroll
            for (int u = 0; u < kSampleUnroll; ++u) {
                if (key[u] == group) found[atomicAdd(&found_count, 1u)] = static_cast<uint32_t>(index[u]);
            }
            t0 += round;
            __syncthreads();
        }
        const unsigned count = found_count;
        SampleInputs next;
        if (static_cast<unsigned>(warp) < count) load_sample(p, found[warp], lane, next);
        for (unsigned j = warp; j < count; j += kSampleWarps) {
            const SampleInputs current = next;
            if (j + kSampleWarps < count) load_sample(p, found[j + kSampleWarps], lane, next);
            sample_one<F>(p, found[j], lane, current, qs[warp], lists[warp], scores[warp], table, bad_group);
        }
        __syncthreads();
        if (t0 >= per_part) break;
        if (threadIdx.x == 0) found_count = 0;
        __syncthreads();
    }
}

// ------------------------------------------------------------------ minibatch grouping
// Each minibatch of an epoch's permutation is stably reordered by feature table (the
// minibatch is the same set of samples; only the row order inside it changes), so the
// objective kernel can stage one table per block. Three passes over 1024-row blocks:
// per-block table counts, per-minibatch offsets, and a scatter whose ranks come from warp
// matches in row order, so the result is deterministic.
constexpr int kBuckets = 43;     // feature tables 0..41, then samples with no valid table
constexpr int kGroupRows = 1024;  // rows per block of the grouping kernels

struct Group {
    const uint32_t* perm;    // [samples] the epoch's order
    const int32_t* tables;   // [samples] feature table per rollout sample (null: table 0)
    int table_count;
    size_t samples, minibatch;
    int blocks_per_slice;
    uint32_t* counts;        // [blocks][kBuckets]; turned into each block's first row per table
    uint32_t* sorted;        // [samples] the epoch's order, each minibatch grouped by table
    int32_t* bucket_start;   // [minibatches][kBuckets + 1] row offsets inside each minibatch
};

__device__ __forceinline__ bool group_range(const Group& p, size_t& slice_start, size_t& start, size_t& end) {
    const size_t slice = blockIdx.x / p.blocks_per_slice;
    slice_start = slice * p.minibatch;
    const size_t slice_end = min(slice_start + p.minibatch, p.samples);
    start = slice_start + static_cast<size_t>(blockIdx.x % p.blocks_per_slice) * kGroupRows;
    end = min(start + kGroupRows, slice_end);
    return start < end;
}

__device__ __forceinline__ int bucket_of(const Group& p, size_t row) {
    if (!p.tables) return 0;
    const int t = p.tables[p.perm[row]];
    return t >= 0 && t < p.table_count ? t : kBuckets - 1;
}

__global__ void k_group_count(Group p) {
    __shared__ uint32_t hist[kBuckets];
    for (int t = threadIdx.x; t < kBuckets; t += blockDim.x) hist[t] = 0;
    __syncthreads();
    size_t slice_start, start, end;
    if (group_range(p, slice_start, start, end)) {
        for (size_t r = start + threadIdx.x; r < end; r += blockDim.x) atomicAdd(&hist[bucket_of(p, r)], 1u);
    }
    __syncthreads();
    for (int t = threadIdx.x; t < kBuckets; t += blockDim.x) p.counts[static_cast<size_t>(blockIdx.x) * kBuckets + t] = hist[t];
}

// One block per minibatch, one thread per table.
__global__ void k_group_offsets(Group p) {
    __shared__ uint32_t total[kBuckets];
    const size_t first = static_cast<size_t>(blockIdx.x) * p.blocks_per_slice;
    const int t = threadIdx.x;
    if (t < kBuckets) {
        uint32_t sum = 0;
        for (int b = 0; b < p.blocks_per_slice; ++b) sum += p.counts[(first + b) * kBuckets + t];
        total[t] = sum;
    }
    __syncthreads();
    if (t < kBuckets) {
        uint32_t base = 0;
        for (int u = 0; u < t; ++u) base += total[u];
        int32_t* starts = p.bucket_start + static_cast<size_t>(blockIdx.x) * (kBuckets + 1);
        starts[t] = static_cast<int32_t>(base);
        if (t == kBuckets - 1) starts[kBuckets] = static_cast<int32_t>(base + total[t]);
        uint32_t running = base;
        for (int b = 0; b < p.blocks_per_slice; ++b) {
            uint32_t* c = p.counts + (first + b) * kBuckets + t;
            const uint32_t n = *c;
            *c = running;
            running += n;
        }
    }
}

__global__ void k_group_scatter(Group p) {
    constexpr int kRuns = kGroupRows / 32;
    __shared__ uint32_t base[kRuns][kBuckets];
    for (int i = threadIdx.x; i < kRuns * kBuckets; i += blockDim.x) (&base[0][0])[i] = 0;
    __syncthreads();
    size_t slice_start, start, end;
    const bool any = group_range(p, slice_start, start, end);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const uint32_t below = (1u << lane) - 1u;
    if (any) {
        for (int g = warp; g < kRuns; g += warps) {
            const size_t r = start + static_cast<size_t>(g) * 32 + lane;
            const bool live = r < end;
            const uint32_t active = __ballot_sync(0xffffffffu, live);
            if (live) {
                const int b = bucket_of(p, r);
                const uint32_t same = __match_any_sync(active, b);
                if ((same & below) == 0) base[g][b] = __popc(same);
            }
        }
    }
    __syncthreads();
    if (any && threadIdx.x < kBuckets) {
        uint32_t running = p.counts[static_cast<size_t>(blockIdx.x) * kBuckets + threadIdx.x];
        for (int g = 0; g < kRuns; ++g) {
            const uint32_t n = base[g][threadIdx.x];
            base[g][threadIdx.x] = running;
            running += n;
        }
    }
    __syncthreads();
    if (any) {
        for (int g = warp; g < kRuns; g += warps) {
            const size_t r = start + static_cast<size_t>(g) * 32 + lane;
            const bool live = r < end;
            const uint32_t active = __ballot_sync(0xffffffffu, live);
            if (live) {
                const int b = bucket_of(p, r);
                const uint32_t same = __match_any_sync(active, b);
                p.sorted[slice_start + base[g][b] + __popc(same & below)] = p.perm[r];
            }
        }
    }
}

// ------------------------------------------------------------------ PPO objective
// ppo_output_gradient_kernel + parametric_policy_gradient_kernel (src/ppo.cu:453-565, 350-381):
// one warp per sample; the clipped policy objective, the clipped value loss and the entropy
// bonus; d(objective)/d(q, value) written as the bf16 gradient row of the output layer.
struct Loss {
    const float* out;  // [n][ld]
    int ld, feature_size;
    int action_count;  // candidates per sample (at most 368)
    const float* features;
    int table_count;
    const int32_t* tables;
    const uint32_t* bits;
    const int32_t* actions;
    const float* old_lp;
    const float* old_v;
    const float* adv;
    const float* ret;
    size_t count;
    float inv_batch;  // 1 / minibatch size
    float clip, value_clip, value_coef, entropy_coef;
    __nv_bfloat16* dout;  // [n][ld_grad]
    int ld_grad;
    double* block_metrics;  // [blocks][kMetrics]
    float* out_colsum;      // [blocks][ld_grad]: bias gradient partials of the output layer
    float* sample_entropy;  // first epoch: entropy per rollout sample (or null)
    uint8_t* sample_decision;
    const uint32_t* perm;
    size_t offset;
    const int32_t* bucket_start;  // [kBuckets + 1] first row of each table's rows in the minibatch
};

// Rows of one feature table that a k_loss block scores; the block's table sits in shared
// memory, so each candidate row is read from L2 once per block instead of once per sample.
constexpr int kLossRows = 256;

// The minibatch rows are grouped by feature table (k_group_*); block b takes the b-th run of at
// most kLossRows rows of one table, counted over the tables in order. Blocks past the last run
// only write zero partials.
template <int F>
__global__ void __launch_bounds__(32 * kWarps, 3) k_loss(Loss p) {
    extern __shared__ float4 table[];  // action_count x F floats, see staged_slot
    __shared__ float qs[kWarps][64];
    __shared__ float grads[kWarps][64];
    __shared__ float colsum[kWarps][64];
    __shared__ double metric[kWarps][kMetrics];
    __shared__ int16_t lists[kWarps][kCandidates];
    __shared__ float scores[kWarps][kCandidates];
    __shared__ int run[3];  // bucket, first row, end row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        int b = static_cast<int>(blockIdx.x);
        run[0] = -1;
        run[1] = run[2] = 0;
        for (int t = 0; t < kBuckets; ++t) {
            const int lo = p.bucket_start[t], hi = p.bucket_start[t + 1];
            const int runs = (hi - lo + kLossRows - 1) / kLossRows;
            if (b < runs) {
                run[0] = t;
                run[1] = lo + b * kLossRows;
                run[2] = min(lo + (b + 1) * kLossRows, hi);
                break;
            }
            b -= runs;
        }
    }
    __syncthreads();
    const int bucket = run[0];
    const bool bad_table = bucket < 0 || bucket >= p.table_count;
    if (!bad_table) {
        const float4* src = reinterpret_cast<const float4*>(p.features + static_cast<size_t>(bucket) * p.action_count * F);
        for (int i = threadIdx.x; i < p.action_count * (F / 4); i += blockDim.x) {
            table[staged_slot<F>(i / (F / 4), i % (F / 4))] = __ldg(src + i);
        }
    }
    float col_lo = 0.0f, col_hi = 0.0f;
    if (lane < kMetrics) metric[warp][lane] = 0.0;
    for (int f = lane; f < 64; f += 32) grads[warp][f] = 0.0f;
    __syncthreads();
    const float scale = rsqrtf(static_cast<float>(p.feature_size));
    for (int row = run[1] + warp; bucket >= 0 && row < run[2]; row += kWarps) {
        const size_t i = static_cast<size_t>(row);
        // the sample's scalars load with its output row, one exposed latency per sample
        const int32_t action_in = p.actions[i];
        const float old_lp_in = p.old_lp[i], advantage_in = p.adv[i], ret_in = p.ret[i], old_v_in = p.old_v[i];
        const float* o = p.out + i * p.ld;
        for (int f = lane; f <= p.feature_size; f += 32) qs[warp][f] = o[f];
        __syncwarp();
        float q[F];
#pragma unroll
        for (int f = 0; f < F; ++f) q[f] = qs[warp][f];
        uint32_t words[kMaskWords];
        bool any = false;
#pragma unroll
        for (int w = 0; w < kMaskWords; ++w) {
            words[w] = p.bits[i * kMaskWords + w];
            any = any || words[w] != 0;
        }
        int16_t* list = lists[warp];
        float* sc = scores[warp];
        const int count = compact_legal(words, any, lane, list);
        float local_max = -3.402823466e38f;
        for (int j = lane; j < count; j += 32) {
            const float s = bad_table ? __int_as_float(0x7fc00000) : staged_score<F>(q, table, list[j], scale);
            sc[j] = s;
            local_max = fmaxf(local_max, s);
        }
        const float maximum = warp_max(local_max);
        __syncwarp();
        float local = 0.0f;
        for (int j = lane; j < count; j += 32) local += expf(sc[j] - maximum);
        const float sum = fmaxf(warp_sum(local), 1e-20f);
        const float log_sum = logf(sum) + maximum;
        const int selected = any ? action_in : 0;
        const float new_lp = sc[legal_rank(words, any, selected)] - log_sum;
        const float log_ratio = new_lp - old_lp_in;
        const float ratio = expf(log_ratio);
        const float advantage = advantage_in;
        const float unclipped = ratio * advantage;
        const float clipped = fminf(1.0f + p.clip, fmaxf(1.0f - p.clip, ratio)) * advantage;
        const bool use_unclipped = unclipped <= clipped;
        const float policy_loss = -fminf(unclipped, clipped);
        const float lp_grad = use_unclipped ? -advantage * ratio : 0.0f;
        float entropy = 0.0f;
        for (int j = lane; j < count; j += 32) {
            const float lp = sc[j] - log_sum;
            entropy -= expf(lp) * lp;
        }
        entropy = warp_sum(entropy);
        // d(objective)/d(score) of each legal candidate folded into d/dq
        float dq_local[F];
#pragma unroll
        for (int f = 0; f < F; ++f) dq_local[f] = 0.0f;
        if (!bad_table) {
            for (int j = lane; j < count; j += 32) {
                const int c = list[j];
                const float lp = sc[j] - log_sum;
                const float prob = expf(lp);
                float g = (lp_grad * ((c == selected ? 1.0f : 0.0f) - prob)) * p.inv_batch;
                g += p.entropy_coef * prob * (lp + entropy) * p.inv_batch;
#pragma unroll
                for (int k = 0; k < F / 4; ++k) {
                    const float4 f = staged_chunk<F>(table, c, k);
                    dq_local[4 * k] += g * f.x;
                    dq_local[4 * k + 1] += g * f.y;
                    dq_local[4 * k + 2] += g * f.z;
                    dq_local[4 * k + 3] += g * f.w;
                }
            }
        }
        const float total = transpose_sum32(dq_local, lane);
        grads[warp][lane] = bad_table ? __int_as_float(0x7fc00000) : total * scale;
        if constexpr (F > 32) {
            float high[32];
#pragma unroll
            for (int f = 0; f < 32; ++f) high[f] = f + 32 < F ? dq_local[f + 32] : 0.0f;
            const float upper = transpose_sum32(high, lane);
            if (lane + 32 < F) grads[warp][32 + lane] = bad_table ? __int_as_float(0x7fc00000) : upper * scale;
        }
        const float value = qs[warp][p.feature_size];
        const float error = value - ret_in;
        float vgrad = error;
        float vloss = 0.5f * error * error;
        if (p.value_clip > 0.0f) {
            const float delta = value - old_v_in;
            const float clipped_value = old_v_in + fminf(p.value_clip, fmaxf(-p.value_clip, delta));
            const float cerr = clipped_value - ret_in;
            const float closs = 0.5f * cerr * cerr;
            if (closs > vloss) {
                vloss = closs;
                vgrad = fabsf(delta) <= p.value_clip ? cerr : 0.0f;
            }
        }
        if (lane == 0) {
            grads[warp][p.feature_size] = p.value_coef * vgrad * p.inv_batch;
            double* m = metric[warp];
            m[0] += policy_loss;
            m[1] += vloss;
            m[2] += entropy;
            m[3] += (ratio - 1.0f) - log_ratio;
            m[4] += fabsf(ratio - 1.0f) > p.clip ? 1.0f : 0.0f;
            m[6] += count > 1 ? 1.0f : 0.0f;
            m[7] += count > 1 ? entropy : 0.0f;
            if (p.sample_entropy) {
                const size_t sample = p.perm[p.offset + i];
                p.sample_entropy[sample] = entropy;
                p.sample_decision[sample] = count > 1 ? 1 : 0;
            }
        }
        __syncwarp();
        col_lo += grads[warp][lane];
        col_hi += grads[warp][32 + lane];
        for (int f = lane; f < p.ld_grad; f += 32) p.dout[i * p.ld_grad + f] = __float2bfloat16_rn(grads[warp][f]);
        __syncwarp();
    }
    colsum[warp][lane] = col_lo;
    colsum[warp][32 + lane] = col_hi;
    __syncthreads();
    // block partials in warp order (deterministic)
    if (threadIdx.x < p.ld_grad) {
        float sum = 0.0f;
        for (int w = 0; w < kWarps; ++w) sum += colsum[w][threadIdx.x];
        p.out_colsum[static_cast<size_t>(blockIdx.x) * p.ld_grad + threadIdx.x] = sum;
    }
    if (threadIdx.x < kMetrics) {
        double sum = 0.0;
        for (int w = 0; w < kWarps; ++w) sum += metric[w][threadIdx.x];
        p.block_metrics[static_cast<size_t>(blockIdx.x) * kMetrics + threadIdx.x] = sum;
    }
}

// Fixed-order sum of [rows][cols] doubles into out[cols] (+= when accumulate).
__global__ void k_sum_rows_f64(const double* in, int rows, int cols, double* out, int accumulate) {
    __shared__ double part[256];
    const int c = blockIdx.x;
    double s = 0.0;
    for (int r = threadIdx.x; r < rows; r += blockDim.x) s += in[static_cast<size_t>(r) * cols + c];
    part[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[c] = (accumulate ? out[c] : 0.0) + part[0];
}

// ------------------------------------------------------------------ norm + Adam
// Squared gradient norm: per-block partial sums over fixed chunks, then one fixed-order sum.
__global__ void k_square_partials(const float* g, size_t n, double* partial) {
    __shared__ double part[256];
    double s = 0.0;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const double v = g[i];
        s += v * v;
    }
    part[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) partial[blockIdx.x] = part[0];
}

__global__ void k_norm_finish(const double* partial, int blocks, double* norm_sq, double* metrics) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    double s = 0.0;
    for (int b = 0; b < blocks; ++b) s += partial[b];
    *norm_sq = s;
    metrics[5] += sqrt(s);
}

// One tensor's view in the flat parameter vector, with the bf16 operand copies to refresh.
struct TensorSpec {
    size_t offset;
    int rows, cols;            // reference layout [rows][cols] (a bias has rows = 1)
    __nv_bfloat16* copy;       // [rows][copy_ld] operand copy or null
    int copy_ld;
    __nv_bfloat16* copy_t;     // [cols][copy_t_ld] transposed operand copy or null
    int copy_t_ld;
};

constexpr int kMaxTensors = 20;
struct AdamSpec {
    TensorSpec t[kMaxTensors];
    int count;
};

// adam_kernel (src/ppo.cu:710-736) over the whole flat vector, fused with the bf16 casts.
__global__ void k_adam(float* params, const float* grads, float* m1, float* m2, size_t n, const double* norm_sq,
                       float max_norm, float lr, float beta1, float beta2, float eps, float bc1, float bc2, AdamSpec spec,
                       int update) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float p = params[i];
    if (update) {
        const float norm = sqrtf(static_cast<float>(*norm_sq));
        if (isfinite(norm)) {
            const float scale = norm > max_norm ? max_norm / fmaxf(norm, 1e-12f) : 1.0f;
            const float g = grads[i] * scale;
            const float m = beta1 * m1[i] + (1.0f - beta1) * g;
            const float v = beta2 * m2[i] + (1.0f - beta2) * g * g;
            m1[i] = m;
            m2[i] = v;
            p -= lr * (m / bc1) / (sqrtf(v / bc2) + eps);
            params[i] = p;
        }
    }
    int t = 0;
    while (t + 1 < spec.count && spec.t[t + 1].offset <= i) ++t;
    const TensorSpec& ts = spec.t[t];
    const size_t local = i - ts.offset;
    const int r = static_cast<int>(local / ts.cols), c = static_cast<int>(local % ts.cols);
    const __nv_bfloat16 b = __float2bfloat16_rn(p);
    if (ts.copy) ts.copy[static_cast<size_t>(r) * ts.copy_ld + c] = b;
    if (ts.copy_t) ts.copy_t[static_cast<size_t>(c) * ts.copy_t_ld + r] = b;
}

// ------------------------------------------------------------------ rollout scan, observation normaliser
// One pass over the rollout before update_ppo: validate_rollout_kernel's checks (src/ppo.cu:423-451:
// finite observations, log-probabilities, values, advantages and returns; each action legal in its
// mask, or 0 with no legal candidate) and, when `moments` is non-null, the batch moments of every
// observation feature per chunk of samples ([chunks][width][3]: count, mean, M2), which the
// normaliser merges after the update (src/ppo.cu:1663-1667). Grid x: the feature groups of 32,
// then one group checking the chunk's samples; grid y: the chunks. A thread owns one feature
// over an eighth of a chunk and sums (x - K) and (x - K)^2 in double, K the first value it reads
// (shifted sums, no division per element); the eighths merge in order (Chan et al.).
struct Scan {
    const float* obs;
    int width;
    size_t samples, chunk;
    double* moments;
    const uint8_t* bytes;
    const uint32_t* bits;
    int actions_per_sample;
    const int64_t* actions;
    const float* lp;
    const float* v;
    const float* adv;
    const float* ret;
    int* invalid;
};

__global__ void __launch_bounds__(256) k_scan(Scan p) {
    const int groups = (p.width + 31) / 32;
    const size_t begin = static_cast<size_t>(blockIdx.y) * p.chunk;
    const size_t end = begin + p.chunk < p.samples ? begin + p.chunk : p.samples;
    if (static_cast<int>(blockIdx.x) == groups) {
        bool ok = true;
        for (size_t s = begin + threadIdx.x; s < end; s += blockDim.x) {
            bool finite = isfinite(p.lp[s]) && isfinite(p.v[s]) && isfinite(p.adv[s]) && isfinite(p.ret[s]);
            bool any = false, chosen = false;
            const int64_t a = p.actions[s];
            for (int w = 0; w < kMaskWords; ++w) {
                uint32_t word = 0;
                if (p.bits) {
                    word = p.bits[s * kMaskWords + w];
                } else {
                    for (int b = 0; b < 32 && w * 32 + b < p.actions_per_sample; ++b) {
                        word |= (p.bytes[s * p.actions_per_sample + w * 32 + b] != 0 ? 1u : 0u) << b;
                    }
                }
                any = any || word != 0;
                if (a >= w * 32 && a < w * 32 + 32) chosen = (word >> (a - w * 32)) & 1u;
            }
            const bool valid = a >= 0 && a < p.actions_per_sample && ((any && chosen) || (!any && a == 0));
            ok = ok && finite && valid;
        }
        if (!ok) atomicExch(p.invalid, 1);
        return;
    }
    const int lane = threadIdx.x & 31;
    const int sub = threadIdx.x >> 5;  // 8 eighths of the chunk per block
    const int feature = static_cast<int>(blockIdx.x) * 32 + lane;
    __shared__ double sm_mean[8][32], sm_m2[8][32], sm_n[8];
    const size_t span = end > begin ? end - begin : 0;
    const size_t per = (span + 7) / 8;
    const size_t b = begin + sub * per < end ? begin + sub * per : end;
    const size_t e = b + per < end ? b + per : end;
    bool finite = true;
    double shift = 0.0, s1 = 0.0, s2 = 0.0, t1 = 0.0, t2 = 0.0;
    if (feature < p.width && e > b) {
        const float* col = p.obs + feature;
        const size_t w = static_cast<size_t>(p.width);
        shift = col[b * w];
        size_t s = b;
        for (; s + 2 <= e; s += 2) {
            const float x0 = col[s * w], x1 = col[(s + 1) * w];
            finite = finite && isfinite(x0) && isfinite(x1);
            const double d0 = static_cast<double>(x0) - shift, d1 = static_cast<double>(x1) - shift;
            s1 += d0;
            s2 += d0 * d0;
            t1 += d1;
            t2 += d1 * d1;
        }
        if (s < e) {
            const float x = col[s * w];
            finite = finite && isfinite(x);
            const double d = static_cast<double>(x) - shift;
            s1 += d;
            s2 += d * d;
        }
    }
    if (!finite) atomicExch(p.invalid, 1);
    if (p.moments == nullptr) return;
    const double n = e > b ? static_cast<double>(e - b) : 0.0;
    double mean = 0.0, m2 = 0.0;
    if (n > 0.0) {
        const double sum = s1 + t1;
        mean = shift + sum / n;
        m2 = fmax((s2 + t2) - sum * sum / n, 0.0);
    }
    sm_mean[sub][lane] = mean;
    sm_m2[sub][lane] = m2;
    if (lane == 0) sm_n[sub] = n;
    __syncthreads();
    if (sub == 0 && feature < p.width) {
        double count = 0.0, mu = 0.0, q = 0.0;
        for (int k = 0; k < 8; ++k) {
            const double nk = sm_n[k];
            if (nk == 0.0) continue;
            const double total = count + nk;
            const double delta = sm_mean[k][lane] - mu;
            q += sm_m2[k][lane] + delta * delta * count * nk / total;
            mu += delta * nk / total;
            count = total;
        }
        double* slot = p.moments + (static_cast<size_t>(blockIdx.y) * p.width + feature) * 3;
        slot[0] = count;
        slot[1] = mu;
        slot[2] = q;
    }
}

// merge_observation_moments_kernel + refresh_inverse_standard_deviation_kernel (src/ppo.cu:183-215).
__global__ void k_obs_merge(const double* chunks, int chunk_count, int width, double running_count, float* mean,
                            float* variance, float* istd, float epsilon, double* batch_out) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= width) return;
    double n = 0.0, mu = 0.0, q = 0.0;
    for (int k = 0; k < chunk_count; ++k) {
        const double* slot = chunks + (static_cast<size_t>(k) * width + f) * 3;
        if (slot[0] == 0.0) continue;
        const double total = n + slot[0];
        const double delta = slot[1] - mu;
        q += slot[2] + delta * delta * n * slot[0] / total;
        mu += delta * slot[0] / total;
        n = total;
    }
    if (batch_out) {
        batch_out[3 * f] = n;
        batch_out[3 * f + 1] = mu;
        batch_out[3 * f + 2] = q;
    }
    if (mean == nullptr) return;
    const double total = running_count + n;
    const double delta = mu - static_cast<double>(mean[f]);
    const double m2 = static_cast<double>(variance[f]) * running_count + q + delta * delta * running_count * n / total;
    mean[f] = static_cast<float>(static_cast<double>(mean[f]) + delta * n / total);
    variance[f] = static_cast<float>(m2 / total);
    istd[f] = 1.0f / sqrtf(variance[f] + epsilon);
}

__global__ void k_refresh_istd(const float* variance, float* istd, int width, float epsilon) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f < width) istd[f] = 1.0f / sqrtf(variance[f] + epsilon);
}

}  // namespace
}  // namespace ppo
}  // namespace t8b
