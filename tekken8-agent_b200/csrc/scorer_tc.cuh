// The PPO objective's parametric scorer on the tensor cores, for 32-feature tables (the
// full-move roster's): parametric_policy_gradient_kernel + ppo_output_gradient_kernel
// (src/ppo.cu:350-381, 453-565) over a minibatch whose rows are grouped by feature table.
//
// One CTA per SM walks a contiguous range of 128-row tiles, each of one table:
//   scores S = Q . T^T on tcgen05 (M = 128 rows, N = 256 + 112 candidates, K = 32 features) into
//     tensor memory, in tf32 with both operands split into a tf32 high part and a tf32 remainder
//     (Qh.Th + Qh.Tl + Ql.Th: about 22 significant bits per product, fp32 accumulation);
//   the objective on the accumulator: each thread owns one row (its TMEM lane) and half of the
//     candidates (8 warps: lane quarter = warp & 3, column half = warp >> 2), so the masked
//     softmax, entropy and clipped ratio need no shuffles; the two halves of a row meet in
//     shared memory;
//   the score gradient G (tf32) is written back over the scores in tensor memory, and
//     dq = G . T runs as a second tcgen05 MMA with A read from tensor memory and B the table's
//     transpose (tf32, K-major, staged beside the table: a tf32 B operand read MN-major from
//     the table's own rows gave zeros on B200);
//   the epilogue writes the bf16 gradient row d(objective)/d(q, value), and per tile the fp32
//     column sums (the output bias gradient) and the metric sums, both in row order.
// The table is staged (tf32 high and remainder, and the transpose, 128B swizzle) only when the
// tile's table changes. Waits on the MMAs are bounded: a stall sets the error flag and the CTA stops.
#pragma once

#include "ppo_kernels.cuh"

namespace t8b {
namespace ppo {

constexpr int kTcRows = 128;          // rows per tile: the MMA's M, one TMEM lane each
constexpr int kTcCandidates = 368;    // score columns (23 x 16)
constexpr int kTcTableBytes = kTcCandidates * 128;  // one 128-byte swizzle row per candidate
constexpr int kTcQBytes = kTcRows * 128;
constexpr int kTcTransposeBytes = 12 * 4096;  // 32 feature rows x 384 candidates: 12 atoms of 32
constexpr int kTcThreads = 256;
constexpr int kTcTmemColumns = 512;   // scores / score gradients [0, 384), dq [384, 416)
constexpr int kTcDq = 384;
constexpr int kTcStage = 33;          // staged gradient row: 32 query columns + the value column
constexpr int kTcOffTlo = kTcTableBytes;
constexpr int kTcOffTt = 2 * kTcTableBytes;
constexpr int kTcOffQhi = kTcOffTt + kTcTransposeBytes;
constexpr int kTcOffQlo = kTcOffQhi + kTcQBytes;
constexpr int kTcOffStage = kTcOffQlo + kTcQBytes;
constexpr int kTcOffMetric = kTcOffStage + kTcRows * kTcStage * 4;
constexpr int kTcOffPart = kTcOffMetric + kTcRows * kMetrics * 4;
constexpr int kTcOffBar = kTcOffPart + 4 * 2 * kTcRows * 4;
constexpr int kTcSmemBytes = kTcOffBar + 64 + 1024;  // + alignment of the dynamic base to 1024
constexpr float kLog2e = 1.4426950408889634f;

// Byte offset of 16-byte chunk k of row r in a 128B-swizzled block of 128-byte rows (1024-aligned).
__device__ __forceinline__ uint32_t sw128(int r, int k) {
    return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((k ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint32_t tf32_bits(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
// x = hi + lo with both parts tf32: hi rounds x, lo rounds the exact remainder.
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    hi = tf32_bits(x);
    lo = tf32_bits(x - __uint_as_float(hi));
}
__device__ __forceinline__ void st_shared4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// Four floats split into the high and remainder blocks at the same swizzled offset.
__device__ __forceinline__ void stage_split(uint32_t hi_base, uint32_t lo_base, uint32_t at, float4 x) {
    uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
    split_tf32(x.x, h0, l0);
    split_tf32(x.y, h1, l1);
    split_tf32(x.z, h2, l2);
    split_tf32(x.w, h3, l3);
    st_shared4(hi_base + at, h0, h1, h2, h3);
    st_shared4(lo_base + at, l0, l1, l2, l3);
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// kind::tf32 instruction descriptor: fp32 accumulate, tf32 A and B, M = 128; B MN-major when asked.
__host__ __device__ constexpr uint32_t tf32_desc(int n, bool b_mn) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(b_mn) << 16) |
        (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(tc::BM >> 4) << 24);
}
__device__ __forceinline__ void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// A read from tensor memory (K-major: row = lane, one tf32 element per column).
__device__ __forceinline__ void mma_tf32_tmem_a(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_store32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,"
        "%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_store_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Tile `tile` of a minibatch grouped by table (bucket_start[kBuckets + 1]): the tables' runs cut
// into 128-row tiles, counted over the tables in order; bucket -1 past the last.
__device__ __forceinline__ void tc_tile(const int32_t* bucket_start, int tile, int& bucket, int& first, int& end) {
    bucket = -1;
    first = end = 0;
    for (int t = 0; t < kBuckets; ++t) {
        const int lo = bucket_start[t], hi = bucket_start[t + 1];
        const int tiles = (hi - lo + kTcRows - 1) / kTcRows;
        if (tile < tiles) {
            bucket = t;
            first = lo + tile * kTcRows;
            end = min(first + kTcRows, hi);
            return;
        }
        tile -= tiles;
    }
}

// Tiles a minibatch of n rows can take (every table's run rounded up to whole tiles): the
// rows of the per-tile partial arrays.
__host__ __device__ constexpr size_t tc_tiles(size_t n) { return (n + kTcRows - 1) / kTcRows + kBuckets; }

__global__ void __launch_bounds__(kTcThreads, 1) k_loss_tc(Loss p, int tiles, int* error) {
    extern __shared__ __align__(1024) unsigned char tc_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
    float* stage = reinterpret_cast<float*>(base + kTcOffStage);       // [128][33]
    float* row_metric = reinterpret_cast<float*>(base + kTcOffMetric);  // [128][8]
    float* part = reinterpret_cast<float*>(base + kTcOffPart);          // [4 quantities][2 halves][128 rows]
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + kTcOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t t_hi = tc::smem_addr(base), t_lo = t_hi + kTcOffTlo, t_tr = t_hi + kTcOffTt;
    const uint32_t q_hi = t_hi + kTcOffQhi, q_lo = t_hi + kTcOffQlo;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;  // this thread's tile row (its TMEM lane)
    if (threadIdx.x == 0) {
        tc::bar_init(bar, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_addr(tmem_slot)),
                     "r"(kTcTmemColumns));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lanes = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    if (half == 1) {
        // columns 368..383 hold no score; keep them finite (zero) for the passes that read them
        uint32_t zero[32] = {};
        tmem_store32(lanes + 352, zero);
        tmem_store_wait();
    }
    const float scale = rsqrtf(32.0f);
    const float inv_batch = p.inv_batch;
    uint32_t phase = 0;
    int staged = -1;
    const int t0 = static_cast<int>(static_cast<long long>(tiles) * blockIdx.x / gridDim.x);
    const int t1 = static_cast<int>(static_cast<long long>(tiles) * (blockIdx.x + 1) / gridDim.x);
    for (int tile = t0; tile < t1; ++tile) {
        int bucket, first, end;
        tc_tile(p.bucket_start, tile, bucket, first, end);
        float* colsum_out = p.out_colsum + static_cast<size_t>(tile) * p.ld_grad;
        double* metric_out = p.block_metrics + static_cast<size_t>(tile) * kMetrics;
        if (bucket < 0) {  // past the last run: zero partials
            if (static_cast<int>(threadIdx.x) < p.ld_grad) colsum_out[threadIdx.x] = 0.0f;
            if (threadIdx.x < kMetrics) metric_out[threadIdx.x] = 0.0;
            continue;
        }
        const bool bad = bucket >= p.table_count;
        if (!bad && bucket != staged) {
            const float4* src = reinterpret_cast<const float4*>(p.features + static_cast<size_t>(bucket) * p.action_count * 32);
            for (int idx = threadIdx.x; idx < kTcCandidates * 8; idx += kTcThreads) {
                const int c = idx >> 3, k = idx & 7;
                const float4 x = c < p.action_count ? __ldg(src + idx) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                stage_split(t_hi, t_lo, sw128(c, k), x);
            }
            // the transpose: feature row f, candidates 32 j + 4 k .. + 3 (zero past the table)
            const float* table = p.features + static_cast<size_t>(bucket) * p.action_count * 32;
            for (int idx = threadIdx.x; idx < 32 * 96; idx += kTcThreads) {
                const int f = idx / 96, q = idx % 96, j = q >> 3, k = q & 7;
                const int c0 = j * 32 + 4 * k;
                uint32_t x[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) x[e] = c0 + e < p.action_count ? tf32_bits(__ldg(table + (c0 + e) * 32 + f)) : 0u;
                st_shared4(t_tr + static_cast<uint32_t>(j * 4096) + sw128(f, k), x[0], x[1], x[2], x[3]);
            }
            staged = bucket;
        }
        for (int idx = threadIdx.x; idx < kTcRows * 8; idx += kTcThreads) {
            const int row = idx >> 3, k = idx & 7;
            const int i = first + row;
            float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < end) x = *reinterpret_cast<const float4*>(p.out + static_cast<size_t>(i) * p.ld + 4 * k);
            stage_split(q_hi, q_lo, sw128(row, k), x);
        }
        proxy_fence_shared();
        tc::fence_before();
        __syncthreads();
        if (threadIdx.x == 0 && !bad) {
            tc::fence_after();
#pragma unroll
            for (int chunk = 0; chunk < 2; ++chunk) {
                const int n0 = chunk * 256;
                const uint32_t idesc = tf32_desc(chunk == 0 ? 256 : kTcCandidates - 256, false);
                const uint32_t d = tmem + static_cast<uint32_t>(n0);
                const uint32_t bh = t_hi + static_cast<uint32_t>(n0 * 128), bl = t_lo + static_cast<uint32_t>(n0 * 128);
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    mma_tf32(d, tc::sw128_desc(q_hi + s * 32, 16, 1024), tc::sw128_desc(bh + s * 32, 16, 1024), idesc, s > 0);
                }
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    mma_tf32(d, tc::sw128_desc(q_hi + s * 32, 16, 1024), tc::sw128_desc(bl + s * 32, 16, 1024), idesc, 1);
                }
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    mma_tf32(d, tc::sw128_desc(q_lo + s * 32, 16, 1024), tc::sw128_desc(bh + s * 32, 16, 1024), idesc, 1);
                }
            }
            tc::commit(bar);
        }
        // the row's inputs load while the MMAs run
        const int i_row = first + r;
        const bool valid = i_row < end;
        const size_t i = static_cast<size_t>(valid ? i_row : first);
        uint32_t words[kMaskWords];
        {
            const uint4* b4 = reinterpret_cast<const uint4*>(p.bits + i * kMaskWords);
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const uint4 w = b4[q];
                words[4 * q] = w.x;
                words[4 * q + 1] = w.y;
                words[4 * q + 2] = w.z;
                words[4 * q + 3] = w.w;
            }
        }
        bool any = false;
#pragma unroll
        for (int w = 0; w < kMaskWords; ++w) any = any || words[w] != 0;
        if (!any) words[0] = 1u;  // nothing legal: candidate 0 alone (src/ppo.cu:254-258)
        int count = 0;
#pragma unroll
        for (int w = 0; w < kMaskWords; ++w) count += __popc(words[w]);
        const int action_in = p.actions[i];
        const float old_lp_in = p.old_lp[i], advantage = p.adv[i], ret_in = p.ret[i], old_v_in = p.old_v[i];
        const float value = p.out[i * p.ld + 32];
        const int selected = any ? action_in : 0;
        const int sel_chunk = selected >> 5, sel_bit = selected & 31;
        const int j0 = half * 6;
        float v[32];

        // pass 1: the largest legal raw dot product of this half
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
        if (!bad) {
            if (!tc::bar_wait(bar, phase, abort)) *abort = 1;
            tc::fence_after();
#pragma unroll 1
            for (int j = j0; j < j0 + 6; ++j) {
                tc::tmem_load32(lanes + static_cast<uint32_t>(j * 32), v);
                const uint32_t w = words[j];
#pragma unroll
                for (int b = 0; b < 32; b += 4) {
                    mx0 = fmaxf(mx0, (w >> b) & 1u ? v[b] : -INFINITY);
                    mx1 = fmaxf(mx1, (w >> (b + 1)) & 1u ? v[b + 1] : -INFINITY);
                    mx2 = fmaxf(mx2, (w >> (b + 2)) & 1u ? v[b + 2] : -INFINITY);
                    mx3 = fmaxf(mx3, (w >> (b + 3)) & 1u ? v[b + 3] : -INFINITY);
                }
            }
            phase ^= 1u;
        }
        part[(0 * 2 + half) * kTcRows + r] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        __syncthreads();
        const float maximum = fmaxf(part[0 * kTcRows + r], part[1 * kTcRows + r]) * scale;

        // pass 2: sum of exp(s - max), sum of exp(s - max) (s - max), and the chosen score
        const float k_exp = scale * kLog2e, m_exp = maximum * kLog2e;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f, u0 = 0.0f, u1 = 0.0f, u2 = 0.0f, u3 = 0.0f;
        float chosen_half = __int_as_float(0x7fc00000);
        if (!bad) {
#pragma unroll 1
            for (int j = j0; j < j0 + 6; ++j) {
                tc::tmem_load32(lanes + static_cast<uint32_t>(j * 32), v);
                const uint32_t w = words[j];
#pragma unroll
                for (int b = 0; b < 32; ++b) {
                    const bool legal = (w >> b) & 1u;
                    const float e = legal ? ex2(fmaf(v[b], k_exp, -m_exp)) : 0.0f;
                    const float u = legal ? fmaf(v[b], scale, -maximum) : 0.0f;
                    if ((b & 3) == 0) { s0 += e; u0 = fmaf(e, u, u0); }
                    if ((b & 3) == 1) { s1 += e; u1 = fmaf(e, u, u1); }
                    if ((b & 3) == 2) { s2 += e; u2 = fmaf(e, u, u2); }
                    if ((b & 3) == 3) { s3 += e; u3 = fmaf(e, u, u3); }
                }
                if (j == sel_chunk) {
#pragma unroll
                    for (int b = 0; b < 32; ++b) chosen_half = b == sel_bit ? v[b] * scale : chosen_half;
                }
                __syncwarp();  // reconverge before the next warp-collective tensor-memory load
            }
        }
        part[(2 + half) * kTcRows + r] = (s0 + s1) + (s2 + s3);
        part[(4 + half) * kTcRows + r] = (u0 + u1) + (u2 + u3);
        part[(6 + half) * kTcRows + r] = chosen_half;
        __syncthreads();
        const float exp_sum = part[2 * kTcRows + r] + part[3 * kTcRows + r];
        const float weighted = part[4 * kTcRows + r] + part[5 * kTcRows + r];
        const float chosen = bad ? __int_as_float(0x7fc00000) : part[(6 + (sel_chunk >= 6 ? 1 : 0)) * kTcRows + r];
        const float sum = fmaxf(exp_sum, 1e-20f);
        const float log_sum = bad ? __int_as_float(0x7fc00000) : logf(sum) + maximum;
        // entropy = -sum p (s - log_sum) = log(sum) - sum e (s - max) / sum (p = e / sum)
        const float entropy = bad ? __int_as_float(0x7fc00000) : logf(sum) - weighted / sum;
        const float new_lp = chosen - log_sum;
        const float log_ratio = new_lp - old_lp_in;
        const float ratio = expf(log_ratio);
        const float unclipped = ratio * advantage;
        const float clipped = fminf(1.0f + p.clip, fmaxf(1.0f - p.clip, ratio)) * advantage;
        const bool use_unclipped = unclipped <= clipped;
        const float policy_loss = -fminf(unclipped, clipped);
        const float lp_grad = use_unclipped ? -advantage * ratio : 0.0f;

        // pass 3: d(objective)/d(score) = (lp_grad (onehot - p) + entropy_coef p (log p + entropy)) / batch,
        // written as tf32 over the scores
        if (!bad) {
            const float a_scale = inv_batch / sum;
            const float e_scale = p.entropy_coef * scale;
            const float bias = p.entropy_coef * (entropy - log_sum) - lp_grad;
            const float onehot = lp_grad * inv_batch;
#pragma unroll 1
            for (int j = j0; j < j0 + 6; ++j) {
                tc::tmem_load32(lanes + static_cast<uint32_t>(j * 32), v);
                const uint32_t w = words[j];
                float g[32];
#pragma unroll
                for (int b = 0; b < 32; ++b) {
                    const float e = ex2(fmaf(v[b], k_exp, -m_exp));
                    const float t = fmaf(v[b], e_scale, bias);
                    g[b] = (w >> b) & 1u ? (e * a_scale) * t : 0.0f;
                }
                if (j == sel_chunk) {
#pragma unroll
                    for (int b = 0; b < 32; ++b) g[b] += b == sel_bit ? onehot : 0.0f;
                }
                __syncwarp();
                uint32_t bits[32];
#pragma unroll
                for (int b = 0; b < 32; ++b) bits[b] = tf32_bits(g[b]);
                tmem_store32(lanes + static_cast<uint32_t>(j * 32), bits);
            }
            tmem_store_wait();
        }
        tc::fence_before();
        __syncthreads();
        if (threadIdx.x == 0 && !bad) {
            tc::fence_after();
            constexpr uint32_t idesc = tf32_desc(32, false);
#pragma unroll 4
            for (int s = 0; s < kTcCandidates / 8; ++s) {
                mma_tf32_tmem_a(tmem + kTcDq, tmem + static_cast<uint32_t>(s * 8),
                                tc::sw128_desc(t_tr + static_cast<uint32_t>((s >> 2) * 4096 + (s & 3) * 32), 16, 1024),
                                idesc, s > 0);
            }
            tc::commit(bar);
        }

        // the row's outputs (the column-half 0 warps)
        const float error_v = value - ret_in;
        float vgrad = error_v;
        float vloss = 0.5f * error_v * error_v;
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
        const float value_grad = p.value_coef * vgrad * inv_batch;
        if (!bad) {
            if (!tc::bar_wait(bar, phase, abort)) *abort = 1;
            tc::fence_after();
            phase ^= 1u;
        }
        if (half == 0) {
            if (!bad) {
                tc::tmem_load32(lanes + kTcDq, v);
#pragma unroll
                for (int f = 0; f < 32; ++f) v[f] *= scale;
            } else {
#pragma unroll
                for (int f = 0; f < 32; ++f) v[f] = __int_as_float(0x7fc00000);
            }
            float* st = stage + r * kTcStage;
            float* mt = row_metric + r * kMetrics;
            if (valid) {
#pragma unroll
                for (int f = 0; f < 32; ++f) st[f] = v[f];
                st[32] = value_grad;
                uint32_t packed[32];
#pragma unroll
                for (int f = 0; f < 32; f += 2) {
                    const __nv_bfloat162 two = __floats2bfloat162_rn(v[f], v[f + 1]);
                    packed[f / 2] = *reinterpret_cast<const uint32_t*>(&two);
                }
                {
                    const __nv_bfloat162 two = __floats2bfloat162_rn(value_grad, 0.0f);
                    packed[16] = *reinterpret_cast<const uint32_t*>(&two);
                }
#pragma unroll
                for (int f = 17; f < 32; ++f) packed[f] = 0u;
                uint4* row_out = reinterpret_cast<uint4*>(p.dout + i * p.ld_grad);
#pragma unroll
                for (int q = 0; q < 8; ++q) row_out[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
                mt[0] = policy_loss;
                mt[1] = vloss;
                mt[2] = entropy;
                mt[3] = (ratio - 1.0f) - log_ratio;
                mt[4] = fabsf(ratio - 1.0f) > p.clip ? 1.0f : 0.0f;
                mt[5] = 0.0f;
                mt[6] = count > 1 ? 1.0f : 0.0f;
                mt[7] = count > 1 ? entropy : 0.0f;
                if (p.sample_entropy) {
                    const size_t sample = p.perm[p.offset + i];
                    p.sample_entropy[sample] = entropy;
                    p.sample_decision[sample] = count > 1 ? 1 : 0;
                }
            } else {
#pragma unroll
                for (int f = 0; f < kTcStage; ++f) st[f] = 0.0f;
#pragma unroll
                for (int m = 0; m < kMetrics; ++m) mt[m] = 0.0f;
            }
        }
        tc::fence_before();
        __syncthreads();
        // per-tile partials in row order (deterministic)
        if (static_cast<int>(threadIdx.x) < p.ld_grad) {
            float total = 0.0f;
            if (threadIdx.x < kTcStage) {
                for (int row = 0; row < kTcRows; ++row) total += stage[row * kTcStage + threadIdx.x];
            }
            colsum_out[threadIdx.x] = total;
        } else if (threadIdx.x >= 128 && threadIdx.x < 128 + kMetrics) {
            const int m = threadIdx.x - 128;
            double total = 0.0;
            for (int row = 0; row < kTcRows; ++row) total += static_cast<double>(row_metric[row * kMetrics + m]);
            metric_out[m] = total;
        }
        if (*abort) break;
    }
    if (*abort && threadIdx.x == 0 && error != nullptr) atomicExch(error, 1);
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemColumns));
    }
}

}  // namespace ppo
}  // namespace t8b
