// The PPO objective's parametric scorer on the tensor cores, for 32-feature tables (the
// full-move roster's): parametric_policy_gradient_kernel + ppo_output_gradient_kernel
// (src/ppo.cu:350-381, 453-565) over a minibatch whose rows are grouped by feature table.
//
// One CTA per SM walks a contiguous range of 128-row tiles, each of one table:
//   scores S = Q . T^T on tcgen05 (M = 128 rows, N = 256 + 112 candidates, K = 32 features) into
//     tensor memory, in tf32 with both operands split into a tf32 high part and a tf32 remainder
//     (Qh.Th + Qh.Tl + Ql.Th: about 22 significant bits per product, fp32 accumulation);
//   the objective on the accumulator: each thread owns one row (its TMEM lane) and a quarter of
//     the candidates (16 warps: lane quarter = warp & 3, column slice = warp >> 2, three 32-column
//     chunks each), so the masked softmax, entropy and clipped ratio need no shuffles; the four
//     slices of a row meet in shared memory, combined in slice order;
//   the score gradient G (tf32) is written back over the scores in tensor memory, and
//     dq = G . T runs as a second tcgen05 MMA with A read from tensor memory and B the table's
//     transpose (tf32, K-major, staged beside the table: a tf32 B operand read MN-major from
//     the table's own rows gave zeros on B200);
//   the epilogue writes the bf16 gradient row d(objective)/d(q, value), and per tile the fp32
//     column sums (the output bias gradient) and the metric sums, both in row order.
// The table (tf32 high parts and remainders, and the transpose, 128B swizzle) is copied from its
// prebuilt image (k_table_images) only when the tile's table changes. Waits on the MMAs are bounded: a stall sets the error flag and the CTA stops.
#pragma once

#include "ppo_kernels.cuh"

namespace t8b {
namespace ppo {

constexpr int kTcRows = 128;          // rows per tile: the MMA's M, one TMEM lane each
constexpr int kTcCandidates = 368;    // score columns (23 x 16)
constexpr int kTcTableBytes = kTcCandidates * 128;  // one 128-byte swizzle row per candidate
constexpr int kTcQBytes = kTcRows * 128;
constexpr int kTcTransposeBytes = 12 * 4096;  // 32 feature rows x 384 candidates: 12 atoms of 32
constexpr int kTcSlices = 4;                // warps per lane quarter
constexpr int kTcChunks = 12 / kTcSlices;   // 32-column chunks per warp
constexpr int kTcThreads = 128 * kTcSlices;
static_assert(kTcChunks == 3, "the sampler's rolled chunk loops pick among three mask words");
constexpr int kTcTmemColumns = 512;   // scores / score gradients [0, 384), dq [384, 416)
constexpr int kTcDq = 384;
constexpr int kTcStage = 33;          // gradient columns of a row: 32 query columns + the value column
constexpr int kTcOffTlo = kTcTableBytes;
constexpr int kTcOffTt = 2 * kTcTableBytes;
constexpr int kTcOffQhi = kTcOffTt + kTcTransposeBytes;
constexpr int kTcOffQlo = kTcOffQhi + kTcQBytes;
constexpr int kTcOffPart = kTcOffQlo + kTcQBytes;
constexpr int kTcOffSums = kTcOffPart + 4 * kTcSlices * kTcRows * 4;  // column and metric partials
constexpr int kTcOffBar = kTcOffSums + 1024;
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

// A feature table's shared-memory image, built once when the tables are installed and copied
// verbatim into a 1024-aligned shared-memory base (the 128B swizzle is a function of the offset
// within each 1024-byte block): the tf32 high parts and remainders of the [368][32] table as
// K-major rows, then the transpose's tf32 high parts as [32][384] K-major atoms of 32 candidates.
constexpr int kTcImageBytes = 2 * kTcTableBytes + kTcTransposeBytes;  // 143,360
constexpr int kTcImageChunks = kTcImageBytes / 16;

__global__ void k_table_images(const float* features, int action_count, int tables, uint4* images) {
    const int table = blockIdx.y;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (table >= tables) return;
    unsigned char* image = reinterpret_cast<unsigned char*>(images) + static_cast<size_t>(table) * kTcImageBytes;
    const float* t = features + static_cast<size_t>(table) * action_count * 32;
    if (idx < kTcCandidates * 8) {
        const int c = idx >> 3, k = idx & 7;
        uint32_t hi[4] = {}, lo[4] = {};
        if (c < action_count) {
#pragma unroll
            for (int e = 0; e < 4; ++e) split_tf32(t[c * 32 + 4 * k + e], hi[e], lo[e]);
        }
        *reinterpret_cast<uint4*>(image + sw128(c, k)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(image + kTcTableBytes + sw128(c, k)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    } else if (idx < kTcCandidates * 8 + 32 * 96) {
        const int q0 = idx - kTcCandidates * 8;
        const int f = q0 / 96, q = q0 % 96, j = q >> 3, k = q & 7;
        const int c0 = j * 32 + 4 * k;
        uint32_t x[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = c0 + e < action_count ? tf32_bits(t[(c0 + e) * 32 + f]) : 0u;
        *reinterpret_cast<uint4*>(image + 2 * kTcTableBytes + j * 4096 + sw128(f, k)) = make_uint4(x[0], x[1], x[2], x[3]);
    }
}

// Copies `bytes` of a table image into shared memory at `dst` (all threads of the block).
__device__ __forceinline__ void copy_image(uint32_t dst, const uint4* image, int bytes, int threads) {
    for (int idx = threadIdx.x; idx < bytes / 16; idx += threads) {
        const uint4 v = __ldg(image + idx);
        st_shared4(dst + static_cast<uint32_t>(idx * 16), v.x, v.y, v.z, v.w);
    }
}

__global__ void __launch_bounds__(kTcThreads, 1) k_loss_tc(Loss p, const uint4* images, int tiles, int* error) {
    extern __shared__ __align__(1024) unsigned char tc_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
    float* part = reinterpret_cast<float*>(base + kTcOffPart);          // [4 quantities][slices][128 rows]
    float* column_part = reinterpret_cast<float*>(base + kTcOffSums);   // [4 quarters][33]
    double* metric_part = reinterpret_cast<double*>(base + kTcOffSums + 33 * 4 * 4 + 48);  // [4 quarters][8]
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + kTcOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t t_hi = tc::smem_addr(base), t_lo = t_hi + kTcOffTlo, t_tr = t_hi + kTcOffTt;
    const uint32_t q_hi = t_hi + kTcOffQhi, q_lo = t_hi + kTcOffQlo;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quarter = warp & 3, slice = warp >> 2;
    const int r = quarter * 32 + lane;  // this thread's tile row (its TMEM lane)
    const int j0 = slice * kTcChunks;   // this warp's first 32-column chunk
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
    if (slice == kTcSlices - 1) {
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
            copy_image(t_hi, images + static_cast<size_t>(bucket) * kTcImageChunks, kTcImageBytes, kTcThreads);
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
        uint32_t mine[kTcChunks];  // this warp's three mask words
        bool any;
        int count;
        {
            const uint4* b4 = reinterpret_cast<const uint4*>(p.bits + i * kMaskWords);
            const uint4 a = b4[0], b = b4[1], c = b4[2];
            const uint32_t w[kMaskWords] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w};
            any = false;
            count = 0;
#pragma unroll
            for (int k = 0; k < kMaskWords; ++k) {
                any = any || w[k] != 0;
                count += __popc(w[k]);
            }
#pragma unroll
            for (int c2 = 0; c2 < kTcChunks; ++c2) {
                uint32_t pick = w[c2];
#pragma unroll
                for (int sl = 1; sl < kTcSlices; ++sl) pick = slice == sl ? w[sl * kTcChunks + c2] : pick;
                mine[c2] = pick;
            }
            if (!any) {  // nothing legal: candidate 0 alone (src/ppo.cu:254-258)
                count = 1;
                if (slice == 0) mine[0] = 1u;
            }
        }
        const int action_in = p.actions[i];
        const float old_lp_in = p.old_lp[i], advantage = p.adv[i], ret_in = p.ret[i], old_v_in = p.old_v[i];
        const float value = p.out[i * p.ld + 32];
        const int selected = any ? action_in : 0;
        const int sel_chunk = selected >> 5, sel_bit = selected & 31;
        float v[32];

        // pass 1 (online, per slice): the largest legal score m, sum of exp(s - m), sum of
        // exp(s - m) (s - m), rescaled whenever a chunk raises m; and the chosen score
        float m_slice = -INFINITY, s_slice = 0.0f, u_slice = 0.0f;
        float chosen_slice = __int_as_float(0x7fc00000);
        if (!bad) {
            if (!tc::bar_wait(bar, phase, abort)) *abort = 1;
            tc::fence_after();
#pragma unroll
            for (int c2 = 0; c2 < kTcChunks; ++c2) {
                tc::tmem_load32(lanes + static_cast<uint32_t>((j0 + c2) * 32), v);
                const uint32_t w = mine[c2];
                float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
                for (int b = 0; b < 32; b += 4) {
                    mx0 = fmaxf(mx0, (w >> b) & 1u ? v[b] : -INFINITY);
                    mx1 = fmaxf(mx1, (w >> (b + 1)) & 1u ? v[b + 1] : -INFINITY);
                    mx2 = fmaxf(mx2, (w >> (b + 2)) & 1u ? v[b + 2] : -INFINITY);
                    mx3 = fmaxf(mx3, (w >> (b + 3)) & 1u ? v[b + 3] : -INFINITY);
                }
                const float chunk_max = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * scale;
                if (chunk_max > m_slice) {
                    if (s_slice > 0.0f) {
                        const float f = ex2((m_slice - chunk_max) * kLog2e);
                        u_slice = f * fmaf(m_slice - chunk_max, s_slice, u_slice);
                        s_slice *= f;
                    }
                    m_slice = chunk_max;
                }
                const float k_exp = scale * kLog2e, m_exp = m_slice * kLog2e;
                float s0 = 0.0f, s1 = 0.0f, u0 = 0.0f, u1 = 0.0f;
#pragma unroll
                for (int b = 0; b < 32; ++b) {
                    const bool legal = (w >> b) & 1u;
                    const float e = legal ? ex2(fmaf(v[b], k_exp, -m_exp)) : 0.0f;
                    const float u = legal ? fmaf(v[b], scale, -m_slice) : 0.0f;
                    if (b & 1) { s1 += e; u1 = fmaf(e, u, u1); } else { s0 += e; u0 = fmaf(e, u, u0); }
                }
                s_slice += s0 + s1;
                u_slice += u0 + u1;
                if (j0 + c2 == sel_chunk) {
#pragma unroll
                    for (int b = 0; b < 32; ++b) chosen_slice = b == sel_bit ? v[b] * scale : chosen_slice;
                }
                __syncwarp();  // reconverge before the next warp-collective tensor-memory load
            }
            phase ^= 1u;
        }
        part[(0 * kTcSlices + slice) * kTcRows + r] = m_slice;
        part[(1 * kTcSlices + slice) * kTcRows + r] = s_slice;
        part[(2 * kTcSlices + slice) * kTcRows + r] = u_slice;
        part[(3 * kTcSlices + slice) * kTcRows + r] = chosen_slice;
        __syncthreads();
        float maximum = part[r];
#pragma unroll
        for (int sl = 1; sl < kTcSlices; ++sl) maximum = fmaxf(maximum, part[sl * kTcRows + r]);
        // the slices' sums moved to the common maximum, added in slice order
        float exp_sum = 0.0f, weighted = 0.0f;
#pragma unroll
        for (int sl = 0; sl < kTcSlices; ++sl) {
            const float m = part[sl * kTcRows + r], sm = part[(kTcSlices + sl) * kTcRows + r];
            if (sm > 0.0f) {
                const float f = ex2((m - maximum) * kLog2e);
                exp_sum += f * sm;
                weighted += f * fmaf(m - maximum, sm, part[(2 * kTcSlices + sl) * kTcRows + r]);
            }
        }
        const float k_exp = scale * kLog2e, m_exp = maximum * kLog2e;
        const int owner = sel_chunk / kTcChunks;
        const float chosen = bad || owner >= kTcSlices ? __int_as_float(0x7fc00000) : part[(3 * kTcSlices + owner) * kTcRows + r];
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
#pragma unroll
            for (int c2 = 0; c2 < kTcChunks; ++c2) {
                const uint32_t at = lanes + static_cast<uint32_t>((j0 + c2) * 32);
                tc::tmem_load32(at, v);
                const uint32_t w = mine[c2];
#pragma unroll
                for (int b = 0; b < 32; ++b) {
                    const float e = ex2(fmaf(v[b], k_exp, -m_exp));
                    const float t = fmaf(v[b], e_scale, bias);
                    v[b] = (w >> b) & 1u ? (e * a_scale) * t : 0.0f;
                }
                if (j0 + c2 == sel_chunk) {
#pragma unroll
                    for (int b = 0; b < 32; ++b) v[b] += b == sel_bit ? onehot : 0.0f;
                }
                __syncwarp();
                uint32_t* bits = reinterpret_cast<uint32_t*>(v);
#pragma unroll
                for (int b = 0; b < 32; ++b) bits[b] = tf32_bits(v[b]);
                tmem_store32(at, bits);
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

        // the row's outputs (the slice-0 warps)
        if (slice == 0) {
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
                tc::tmem_load32(lanes + kTcDq, v);
#pragma unroll
                for (int f = 0; f < 32; ++f) v[f] *= scale;
            } else {
#pragma unroll
                for (int f = 0; f < 32; ++f) v[f] = __int_as_float(0x7fc00000);
            }
            float mt[kMetrics] = {policy_loss, vloss, entropy, (ratio - 1.0f) - log_ratio,
                                  fabsf(ratio - 1.0f) > p.clip ? 1.0f : 0.0f, 0.0f, count > 1 ? 1.0f : 0.0f,
                                  count > 1 ? entropy : 0.0f};
            float value_column = value_grad;
            if (valid) {
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
                if (p.sample_entropy) {
                    const size_t sample = p.perm[p.offset + i];
                    p.sample_entropy[sample] = entropy;
                    p.sample_decision[sample] = count > 1 ? 1 : 0;
                }
            } else {
#pragma unroll
                for (int f = 0; f < 32; ++f) v[f] = 0.0f;
                value_column = 0.0f;
#pragma unroll
                for (int m = 0; m < kMetrics; ++m) mt[m] = 0.0f;
            }
            // this quarter's 32 rows summed per column (fixed butterflies): the fp32 gradient
            // columns (the output bias gradient) and the metrics in fp64
            const float column = transpose_sum32(v, lane);
            const float value_total = warp_sum(value_column);
            column_part[quarter * kTcStage + lane] = column;
            if (lane == 0) column_part[quarter * kTcStage + 32] = value_total;
#pragma unroll
            for (int m = 0; m < kMetrics; ++m) {
                double x = static_cast<double>(mt[m]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
                if (lane == m) metric_part[quarter * kMetrics + m] = x;
            }
        }
        if (!bad) phase ^= 1u;  // every thread tracks the barrier's phase; only the slice-0 warps waited
        tc::fence_before();
        __syncthreads();
        // per-tile partials: the four quarters in order
        const int t = threadIdx.x;
        if (t < p.ld_grad) {
            colsum_out[t] = t < kTcStage ? (column_part[t] + column_part[kTcStage + t]) +
                                               (column_part[2 * kTcStage + t] + column_part[3 * kTcStage + t])
                                         : 0.0f;
        } else if (t >= 256 && t < 256 + kMetrics) {
            const int m = t - 256;
            metric_out[m] = (metric_part[m] + metric_part[kMetrics + m]) + (metric_part[2 * kMetrics + m] + metric_part[3 * kMetrics + m]);
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

// The forward's sampler on the tensor cores (masked_sample_kernel, src/ppo.cu:238-300, with the
// parametric scores of src/ppo.cu:316-348), for 32-feature tables: one CTA per (feature table,
// part), grid = groups x parts in one wave. A CTA copies its table's image once, gathers its
// samples (part k of a group takes the samples of its table in the k-th of `parts` contiguous
// ranges of the batch; out-of-range table indices form one more group that gets NaN scores)
// into a row list, 8,192 table indices per round, and scores them 128 rows at a time: S = Q . T^T in tensor memory (the tf32 split of
// k_loss_tc), then per row the largest legal score (the lowest candidate on ties), the masked
// softmax sums, the inverse-CDF draw against the reference's uniform in candidate order (each
// column slice scans its candidates from the sum of the slices before it; the lowest slice
// that reaches the target wins, and the argmax stands in when none does), log-probability,
// value and entropy.
constexpr int kTsUnroll = 16;                      // table indices a thread checks per gathering round
constexpr int kTsList = kTcThreads * kTsUnroll;    // gathered rows per round (one round's worth)
constexpr int kTsOffQhi = 2 * kTcTableBytes;
constexpr int kTsOffQlo = kTsOffQhi + kTcQBytes;
constexpr int kTsOffList = kTsOffQlo + kTcQBytes;
constexpr int kTsOffPart = kTsOffList + kTsList * 4;
constexpr int kTsParts = 6;  // max, argmax, sum, weighted sum, drawn candidate, drawn score
constexpr int kTsOffBar = kTsOffPart + kTsParts * kTcSlices * kTcRows * 4;
constexpr int kTsSmemBytes = kTsOffBar + 64 + 1024;

__global__ void __launch_bounds__(kTcThreads, 1) k_sample_tc(Sample p, const uint4* images, int parts, int* error) {
    extern __shared__ __align__(1024) unsigned char tc_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
    uint32_t* list = reinterpret_cast<uint32_t*>(base + kTsOffList);
    float* part = reinterpret_cast<float*>(base + kTsOffPart);  // [kTsParts][slices][128]
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + kTsOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    unsigned* found = reinterpret_cast<unsigned*>(tmem_slot + 2);
    const uint32_t t_hi = tc::smem_addr(base), t_lo = t_hi + kTcOffTlo;
    const uint32_t q_hi = t_hi + kTsOffQhi, q_lo = t_hi + kTsOffQlo;
    const auto at = [&](int quantity, int sl, int row) -> float& { return part[(quantity * kTcSlices + sl) * kTcRows + row]; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quarter = warp & 3, slice = warp >> 2;
    const int r = quarter * 32 + lane;
    const int j0 = slice * kTcChunks;
    const int group = static_cast<int>(blockIdx.x) / parts;
    const size_t part_id = static_cast<size_t>(blockIdx.x) % static_cast<size_t>(parts);
    const bool bad = p.tables != nullptr && group == p.table_count;
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
    if (slice == kTcSlices - 1) {
        uint32_t zero[32] = {};
        tmem_store32(lanes + 352, zero);
        tmem_store_wait();
    }
    const float scale = rsqrtf(32.0f);
    const float nan = __int_as_float(0x7fc00000);
    uint32_t phase = 0;
    const size_t range_end = p.count * (part_id + 1) / parts;
    size_t next = p.count * part_id / parts;
    bool staged = bad;  // the table image is copied before the first tile (a CTA without samples skips it)
    for (;;) {
        if (threadIdx.x == 0) *found = 0;
        __syncthreads();
        if (next < range_end) {
            // one round: indices next + 2048 q + 4 t + e (q, e < 4), all loads issued first
            int key[kTsUnroll];
#pragma unroll
            for (int u = 0; u < kTsUnroll; ++u) {
                const size_t i = next + static_cast<size_t>((u >> 2) * (4 * kTcThreads) + 4 * threadIdx.x + (u & 3));
                key[u] = -1;
                if (i < range_end) {
                    key[u] = 0;
                    if (p.tables) {
                        const int table_index = p.tables[i];
                        key[u] = table_index < 0 || table_index >= p.table_count ? p.table_count : table_index;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < kTsUnroll; ++u) {
                const size_t i = next + static_cast<size_t>((u >> 2) * (4 * kTcThreads) + 4 * threadIdx.x + (u & 3));
                if (key[u] == group) list[atomicAdd(found, 1u)] = static_cast<uint32_t>(i);
            }
            next += kTsList;
        }
        __syncthreads();
        const int count = static_cast<int>(*found);
        for (int first = 0; first < count && !*abort; first += kTcRows) {
            const int rows = min(kTcRows, count - first);
            if (!staged) {
                copy_image(t_hi, images + static_cast<size_t>(group) * kTcImageChunks, 2 * kTcTableBytes, kTcThreads);
                staged = true;
            }
            for (int idx = threadIdx.x; idx < kTcRows * 8; idx += kTcThreads) {
                const int row = idx >> 3, k = idx & 7;
                float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (row < rows) x = *reinterpret_cast<const float4*>(p.out + static_cast<size_t>(list[first + row]) * p.ld + 4 * k);
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
            const bool valid = r < rows;
            const size_t i = list[first + (valid ? r : 0)];
            uint32_t mine[kTcChunks];
            bool any = false;
            if (p.bits) {
                const uint4* b4 = reinterpret_cast<const uint4*>(p.bits + i * kMaskWords);
                const uint4 a = b4[0], b = b4[1], c = b4[2];
                const uint32_t w[kMaskWords] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w};
#pragma unroll
                for (int k = 0; k < kMaskWords; ++k) any = any || w[k] != 0;
#pragma unroll
                for (int c2 = 0; c2 < kTcChunks; ++c2) {
                    uint32_t pick = w[c2];
#pragma unroll
                    for (int sl = 1; sl < kTcSlices; ++sl) pick = slice == sl ? w[sl * kTcChunks + c2] : pick;
                    mine[c2] = pick;
                }
            } else {
                const uint8_t* bytes = p.bytes + i * p.action_count;
#pragma unroll
                for (int c2 = 0; c2 < kTcChunks; ++c2) {
                    uint32_t w = 0;
                    for (int b = 0; b < 32; ++b) {
                        const int c = (j0 + c2) * 32 + b;
                        if (c < p.action_count && bytes[c] != 0) w |= 1u << b;
                    }
                    mine[c2] = w;
                }
                at(0, slice, r) = (mine[0] | mine[1] | mine[2]) != 0 ? 1.0f : 0.0f;
                __syncthreads();
#pragma unroll
                for (int sl = 0; sl < kTcSlices; ++sl) any = any || at(0, sl, r) != 0.0f;
                __syncthreads();
            }
            if (!any && slice == 0) mine[0] = 1u;  // nothing legal: candidate 0 alone (src/ppo.cu:254-258)
            const float value = p.out[i * p.ld + 32];
            float v[32];

            // pass 1 (online, per slice): the largest legal score and its lowest candidate, the sums
            // of exp(s - max) and exp(s - max) (s - max) rescaled whenever a chunk raises the
            // maximum; the scores out when asked
            float best = -INFINITY, s_slice = 0.0f, u_slice = 0.0f;
            int best_c = -1;
            if (!bad) {
                if (!tc::bar_wait(bar, phase, abort)) *abort = 1;
                tc::fence_after();
                phase ^= 1u;
            }
            // the chunk loops stay rolled: a sampler CTA scores two or three tiles, and unrolled
            // code mostly misses in the instruction cache
#pragma unroll 1
            for (int c2 = 0; c2 < kTcChunks; ++c2) {
                const int j = j0 + c2;
                if (!bad) tc::tmem_load32(lanes + static_cast<uint32_t>(j * 32), v);
                const uint32_t w = c2 == 0 ? mine[0] : (c2 == 1 ? mine[1] : mine[2]);
                const float previous = best;
#pragma unroll
                for (int b = 0; b < 32; ++b) {
                    const float sc = bad ? nan : v[b] * scale;
                    if (((w >> b) & 1u) && (best_c < 0 || sc > best)) {
                        best = sc;
                        best_c = j * 32 + b;
                    }
                }
                if (!bad) {
                    if (best > previous && s_slice > 0.0f) {
                        const float f = ex2((previous - best) * kLog2e);
                        u_slice = f * fmaf(previous - best, s_slice, u_slice);
                        s_slice *= f;
                    }
                    const float k_exp = scale * kLog2e, m_exp = best * kLog2e;
                    float s0 = 0.0f, s1 = 0.0f, u0 = 0.0f, u1 = 0.0f;
#pragma unroll
                    for (int b = 0; b < 32; ++b) {
                        const bool legal = (w >> b) & 1u;
                        const float e = legal ? ex2(fmaf(v[b], k_exp, -m_exp)) : 0.0f;
                        const float u = legal ? fmaf(v[b], scale, -best) : 0.0f;
                        if (b & 1) { s1 += e; u1 = fmaf(e, u, u1); } else { s0 += e; u0 = fmaf(e, u, u0); }
                    }
                    s_slice += s0 + s1;
                    u_slice += u0 + u1;
                }
                if (p.logits && valid) {
                    float* out = p.logits + i * p.action_count;
#pragma unroll
                    for (int b = 0; b < 32; ++b) {
                        const int c = j * 32 + b;
                        if (c < p.action_count) out[c] = bad ? nan : v[b] * scale;
                    }
                }
                __syncwarp();
            }
            at(0, slice, r) = best;
            at(1, slice, r) = __int_as_float(best_c);
            at(2, slice, r) = s_slice;
            at(3, slice, r) = u_slice;
            __syncthreads();
            float maximum = nan;
            int chosen = -1;
#pragma unroll
            for (int sl = 0; sl < kTcSlices; ++sl) {
                const int c = __float_as_int(at(1, sl, r));
                const float m = at(0, sl, r);
                if (c >= 0 && (chosen < 0 || m > maximum)) {
                    maximum = m;
                    chosen = c;
                }
            }
            if (chosen < 0) chosen = 0;
            const float k_exp = scale * kLog2e, m_exp = maximum * kLog2e;
            // the slices' sums moved to the common maximum; prefix = the slices before this one
            float exp_sum = 0.0f, weighted = 0.0f, prefix = 0.0f;
#pragma unroll
            for (int sl = 0; sl < kTcSlices; ++sl) {
                const float sm = at(2, sl, r);
                if (sm > 0.0f) {
                    const float m = at(0, sl, r);
                    const float f = ex2((m - maximum) * kLog2e);
                    if (sl < slice) prefix += f * sm;
                    exp_sum += f * sm;
                    weighted += f * fmaf(m - maximum, sm, at(3, sl, r));
                }
            }
            const float sum = fmaxf(exp_sum, 1e-20f);
            float score = maximum;  // the chosen candidate's score

            // pass 3: the inverse-CDF draw
            if (!p.deterministic && !bad) {
                const float target = uniform01(p.seed, p.step, i + p.lane_offset) * sum;
                float running = prefix;
                int hit = -1;
                float hit_score = 0.0f;
#pragma unroll 1
                for (int c2 = 0; c2 < kTcChunks; ++c2) {
                    tc::tmem_load32(lanes + static_cast<uint32_t>((j0 + c2) * 32), v);
                    const uint32_t w = c2 == 0 ? mine[0] : (c2 == 1 ? mine[1] : mine[2]);
#pragma unroll
                    for (int b = 0; b < 32; ++b) {
                        const bool legal = (w >> b) & 1u;
                        running += legal ? ex2(fmaf(v[b], k_exp, -m_exp)) : 0.0f;
                        if (legal && hit < 0 && target <= running) {
                            hit = (j0 + c2) * 32 + b;
                            hit_score = v[b] * scale;
                        }
                    }
                }
                at(4, slice, r) = __int_as_float(hit);
                at(5, slice, r) = hit_score;
                __syncthreads();
#pragma unroll
                for (int sl = kTcSlices - 1; sl >= 0; --sl) {
                    const int h = __float_as_int(at(4, sl, r));
                    if (h >= 0) {
                        chosen = h;
                        score = at(5, sl, r);
                    }
                }
            }
            if (slice == 0 && valid) {
                const float log_sum = logf(sum) + maximum;
                p.actions[i] = chosen;
                p.log_probs[i] = bad ? nan : score - log_sum;
                p.values[i] = bad ? nan : value;
                p.entropies[i] = bad ? nan : logf(sum) - weighted / sum;
            }
            tc::fence_before();
            __syncthreads();
        }
        if (next >= range_end || *abort) break;
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
