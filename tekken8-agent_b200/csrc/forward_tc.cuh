// The policy's inference forward in one tcgen05 kernel: for a tile of 128 observations, the
// normalised bf16 layer-1 operand (k_prep's arithmetic), both tanh hidden layers and the output
// layer (q, value), with the activations held in shared memory between the layers instead of
// making a round trip through HBM. It computes forward_network (src/ppo.cu:1248-1290: the
// normalise kernel, a GEMM and bias_tanh_kernel per hidden layer, a GEMM and bias_kernel for the
// output layer) for GpuActorCritic::forward (src/ppo.cu:1499-1525).
//
// One persistent CTA per SM, 320 threads:
//   warp 0     TMA producer: one elected thread streams the weights through a ring of three
//              32 KB stages (a 256-row half of a hidden layer's 64-wide k-block, or the output
//              layer's 64 x 64 k-block), in the order the MMA issuer consumes them;
//   warp 1     MMA issuer: per layer, tcgen05.mma (M = 128, N = 256 per half, K = 16) from the
//              activation tile in shared memory and a weight stage into tensor memory (512
//              columns: the layer's two halves), then one commit to acc_full;
//   warps 2-9  the 128 rows' observations (staged as fp32 by cp.async in the atoms layer 1 does
//              not read, the normaliser of the lane's columns in registers) -> normalised,
//              clipped bf16 operand; after each hidden layer, tensor memory -> bias + tanh ->
//              bf16 written back over the activation tile (the layer's MMAs have finished
//              reading it); after the output layer, tensor memory -> bias -> fp32 [rows][64]
//              (zero past the valid columns).
// The activation tile (128 rows x up to 512 columns of bf16) is eight 16 KB atoms in the
// layout a 128B-swizzled TMA load would produce, so the MMA descriptors are the GEMM's.
// Each accumulator half sees the same k-block and K-step order as the separate GEMMs, so the
// outputs are bit-identical to that path. Every wait is bounded: a stall sets the error flag and
// the CTA drains and returns.
#pragma once

#include "gemm.cuh"
#include "ppo_kernels.cuh"

namespace t8b {
namespace ppo {

constexpr int kFwRows = 128;
constexpr int kFwHidden = 512;
constexpr int kFwAtomBytes = kFwRows * 128;                 // 64 bf16 columns of the tile
constexpr int kFwActBytes = kFwAtomBytes * (kFwHidden / 64);  // 128 KB
constexpr int kFwStageBytes = 256 * 64 * 2;                 // 32 KB
constexpr int kFwOutStageBytes = 64 * 64 * 2;               // the output layer's k-block, 8 KB
constexpr int kFwStages = 3;
constexpr int kFwEpiWarps = 8;
constexpr int kFwThreads = 64 + 32 * kFwEpiWarps;
constexpr int kFwHeldCols = 256;  // staged inputs: the normaliser of at most 256 columns in registers
constexpr int kFwSmemBytes = 1024 + kFwActBytes + kFwStages * kFwStageBytes + 256;

struct Forward {
    const float* obs;  // [n][width]
    int width;         // observation floats
    int in_blocks;     // layer-1 k-blocks (padded operand row / 64, at most 8)
    const float* mean;
    const float* istd;
    float clip;
    int normalize;
    const float* b1;
    const float* b2;
    const float* b_out;
    int outputs;  // valid output columns (query + value)
    float* out;   // [n][64]
    int n;
    int* error;
};

// Byte offset of element (r, c) of the activation tile: atom c / 64, 128B-swizzled rows.
__device__ __forceinline__ uint32_t fw_at(int r, int c) {
    return static_cast<uint32_t>((c >> 6) * kFwAtomBytes + (r >> 3) * 1024 + (r & 7) * 128 +
                                 ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}

__device__ __forceinline__ float fw_input(const Forward& p, const float* row, int j, bool live) {
    float v = 0.0f;
    if (live && j < p.width) {
        v = row[j];
        if (p.normalize) v = fminf(p.clip, fmaxf(-p.clip, (v - p.mean[j]) * p.istd[j]));
    }
    return v;
}

// Two 32-column loads of this thread's TMEM lane (at a0 and a1) under one wait: v[0..31], v[32..63].
__device__ __forceinline__ void fw_tmem_load64(uint32_t a0, uint32_t a1, float* v) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(a0), "r"(a1)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(kFwThreads, 1)
    k_forward_tc(const __grid_constant__ CUtensorMap map_w1, const __grid_constant__ CUtensorMap map_w2,
                 const __grid_constant__ CUtensorMap map_out, Forward p) {
    extern __shared__ __align__(1024) unsigned char raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    unsigned char* act = base;
    unsigned char* stages = base + kFwActBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(stages + kFwStages * kFwStageBytes);
    uint64_t* empty = full + kFwStages;
    uint64_t* act_ready = empty + kFwStages;
    uint64_t* acc_full = act_ready + 1;
    uint64_t* rows_staged = acc_full + 1;  // the epilogue warps' cp.async copies of a tile's rows have landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rows_staged + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = (p.n + kFwRows - 1) / kFwRows;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kFwStages; ++i) {
            tc::bar_init(full + i, 1);
            tc::bar_init(empty + i, 1);
        }
        tc::bar_init(act_ready, 32 * kFwEpiWarps);
        tc::bar_init(acc_full, 1);
        tc::bar_init(rows_staged, 32 * kFwEpiWarps);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_addr(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    auto stop = [&]() {
        *abort = 1;
        if (p.error) atomicExch(p.error, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            auto load = [&](const CUtensorMap* map, int x, int y, uint32_t bytes) {
                if (!tc::bar_wait(empty + stage, phase ^ 1u, abort)) {
                    stop();
                    return false;
                }
                tc::bar_expect(full + stage, bytes);
                tc::tma_load(stages + stage * kFwStageBytes, map, full + stage, x, y);
                if (++stage == kFwStages) {
                    stage = 0;
                    phase ^= 1u;
                }
                return true;
            };
            for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
                bool ok = true;
                for (int kb = 0; ok && kb < p.in_blocks; ++kb) {
                    for (int h = 0; ok && h < 2; ++h) ok = load(&map_w1, kb * 64, h * 256, kFwStageBytes);
                }
                for (int kb = 0; ok && kb < kFwHidden / 64; ++kb) {
                    for (int h = 0; ok && h < 2; ++h) ok = load(&map_w2, kb * 64, h * 256, kFwStageBytes);
                }
                for (int kb = 0; ok && kb < kFwHidden / 64; ++kb) ok = load(&map_out, kb * 64, 0, kFwOutStageBytes);
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_hidden = tc::instr_desc(256, false, false);
            constexpr uint32_t idesc_out = tc::instr_desc(64, false, false);
            const uint32_t a0 = tc::smem_addr(act);
            int stage = 0;
            uint32_t phase = 0, ready = 0;
            // the four K = 16 steps of one k-block: activation atom `atom` x the current stage
            auto consume = [&](uint32_t d, int atom, uint32_t idesc, bool first) {
                if (!tc::bar_wait(full + stage, phase, abort)) {
                    stop();
                    return false;
                }
                tc::fence_after();
                const uint32_t a = a0 + static_cast<uint32_t>(atom * kFwAtomBytes);
                const uint32_t b = tc::smem_addr(stages + stage * kFwStageBytes);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    tc::mma(d, tc::sw128_desc(a + k * 32, 16, 1024), tc::sw128_desc(b + k * 32, 16, 1024), idesc,
                            (!first || k > 0) ? 1u : 0u);
                }
                tc::commit(empty + stage);
                if (++stage == kFwStages) {
                    stage = 0;
                    phase ^= 1u;
                }
                return true;
            };
            auto wait_ready = [&]() {
                if (!tc::bar_wait(act_ready, ready, abort)) {
                    stop();
                    return false;
                }
                ready ^= 1u;
                tc::fence_after();
                return true;
            };
            for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
                bool ok = wait_ready();
                for (int kb = 0; ok && kb < p.in_blocks; ++kb) {
                    for (int h = 0; ok && h < 2; ++h) ok = consume(tmem + h * 256, kb, idesc_hidden, kb == 0);
                }
                if (!ok) break;
                tc::commit(acc_full);
                ok = wait_ready();
                for (int kb = 0; ok && kb < kFwHidden / 64; ++kb) {
                    for (int h = 0; ok && h < 2; ++h) ok = consume(tmem + h * 256, kb, idesc_hidden, kb == 0);
                }
                if (!ok) break;
                tc::commit(acc_full);
                ok = wait_ready();
                for (int kb = 0; ok && kb < kFwHidden / 64; ++kb) ok = consume(tmem, kb, idesc_out, kb == 0);
                if (!ok) break;
                tc::commit(acc_full);
            }
        }
    } else {
        const int e = warp - 2;           // epilogue warp 0..7
        const int quarter = warp & 3;     // TMEM lane quarter this warp may read
        const int half = e >> 2;          // alternate 32-column chunks
        const int r = quarter * 32 + lane;  // this lane's row of the tile in the epilogues
        const int in_cols = p.in_blocks * 64;
        uint32_t acc_phase = 0, staged_phase = 0;
        const uint32_t t = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        auto handoff = [&]() {
            tc::fence_before();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc::bar_arrive(act_ready);
        };
        auto wait_acc = [&]() {
            if (!tc::bar_wait(acc_full, acc_phase, abort)) {
                stop();
                return false;
            }
            acc_phase ^= 1u;
            tc::fence_after();
            return true;
        };
        // the observation rows of a tile are staged as fp32 in the atoms layer 1 does not read
        const bool staged = kFwRows * p.width * 4 <= (kFwHidden / 64 - p.in_blocks) * kFwAtomBytes &&
            in_cols <= kFwHeldCols;
        float* stage_rows = reinterpret_cast<float*>(act + p.in_blocks * kFwAtomBytes);
        // this lane's columns j = lane + 32 k of the normaliser, loaded once
        float mean[kFwHeldCols / 32], istd[kFwHeldCols / 32];
#pragma unroll
        for (int k = 0; k < kFwHeldCols / 32; ++k) {
            const int j = lane + 32 * k;
            const bool in = p.normalize && j < p.width;
            mean[k] = in ? p.mean[j] : 0.0f;
            istd[k] = in ? p.istd[j] : 0.0f;
        }
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
            const int row0 = tile * kFwRows;
            const int rows = min(kFwRows, p.n - row0);
            if (staged) {
                const float* src = p.obs + static_cast<size_t>(row0) * p.width;
                const int total = rows * p.width;
                for (int i = e * 32 + lane; i < total; i += 32 * kFwEpiWarps) tc::cp_async4(stage_rows + i, src + i, true);
                tc::cp_async_commit();
                tc::cp_async_wait<0>();
                // every epilogue thread's rows have landed (a bounded wait: a warp that left the
                // loop after an abort cannot hold the others)
                tc::bar_arrive(rows_staged);
                if (!tc::bar_wait(rows_staged, staged_phase, abort)) {
                    stop();
                    break;
                }
                staged_phase ^= 1u;
#pragma unroll 1
                for (int rr = e; rr < kFwRows; rr += kFwEpiWarps) {
                    const float* row = stage_rows + rr * p.width;
#pragma unroll
                    for (int k = 0; k < kFwHeldCols / 32; ++k) {
                        const int j = lane + 32 * k;
                        if (j < in_cols) {
                            float v = 0.0f;
                            if (rr < rows && j < p.width) {
                                v = row[j];
                                if (p.normalize) v = fminf(p.clip, fmaxf(-p.clip, (v - mean[k]) * istd[k]));
                            }
                            *reinterpret_cast<__nv_bfloat16*>(act + fw_at(rr, j)) = __float2bfloat16_rn(v);
                        }
                    }
                }
            } else {
            // layer-1 operand: warp e takes rows e, e + 8, ...; two rows' loads in flight
#pragma unroll 1
            for (int rr = e; rr < kFwRows; rr += 16) {
                const int g0 = row0 + rr, g1 = g0 + 8;
                const float* row_a = p.obs + static_cast<size_t>(g0) * p.width;
                const float* row_b = p.obs + static_cast<size_t>(g1) * p.width;
                float va[8], vb[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int j = lane + 32 * k;
                    va[k] = j < in_cols ? fw_input(p, row_a, j, g0 < p.n) : 0.0f;
                    vb[k] = j < in_cols ? fw_input(p, row_b, j, g1 < p.n) : 0.0f;
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int j = lane + 32 * k;
                    if (j < in_cols) {
                        *reinterpret_cast<__nv_bfloat16*>(act + fw_at(rr, j)) = __float2bfloat16_rn(va[k]);
                        *reinterpret_cast<__nv_bfloat16*>(act + fw_at(rr + 8, j)) = __float2bfloat16_rn(vb[k]);
                    }
                }
                for (int j = lane + 256; j < in_cols; j += 32) {
                    *reinterpret_cast<__nv_bfloat16*>(act + fw_at(rr, j)) = __float2bfloat16_rn(fw_input(p, row_a, j, g0 < p.n));
                    *reinterpret_cast<__nv_bfloat16*>(act + fw_at(rr + 8, j)) =
                        __float2bfloat16_rn(fw_input(p, row_b, j, g1 < p.n));
                }
            }
            }
            handoff();
            // hidden layers: tanh(acc + b) as bf16 over the activation tile
            bool ok = true;
            for (int l = 0; ok && l < 2; ++l) {
                if (!(ok = wait_acc())) break;
                const float* bias = l == 0 ? p.b1 : p.b2;
                // chunks c and c + 2 (this warp's alternate 32-column chunks) per TMEM wait
#pragma unroll 1
                for (int c = half; c < kFwHidden / 32; c += 4) {
                    float v[64];
                    fw_tmem_load64(t + static_cast<uint32_t>(c * 32), t + static_cast<uint32_t>((c + 2) * 32), v);
#pragma unroll
                    for (int s = 0; s < 2; ++s) {
                        const int col = (c + 2 * s) * 32;
                        const float4* b = reinterpret_cast<const float4*>(bias + col);
                        uint32_t packed[16];
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 bq = __ldg(b + q);
                            const float* x = v + 32 * s + 4 * q;
                            __nv_bfloat162 lo = __floats2bfloat162_rn(tanh_fast(x[0] + bq.x), tanh_fast(x[1] + bq.y));
                            __nv_bfloat162 hi = __floats2bfloat162_rn(tanh_fast(x[2] + bq.z), tanh_fast(x[3] + bq.w));
                            packed[2 * q] = *reinterpret_cast<uint32_t*>(&lo);
                            packed[2 * q + 1] = *reinterpret_cast<uint32_t*>(&hi);
                        }
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            *reinterpret_cast<uint4*>(act + fw_at(r, col + q * 8)) =
                                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
                        }
                    }
                }
                handoff();
            }
            if (!ok || !wait_acc()) {
                stop();
                break;
            }
            // output layer: acc + b for the valid columns, zero beyond
            {
                float v[32];
                tc::tmem_load32(t + static_cast<uint32_t>(half * 32), v);
                const int g = row0 + r;
                if (g < p.n) {
                    float* dst = p.out + static_cast<size_t>(g) * 64 + half * 32;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int c = half * 32 + 4 * q;
                        const float4 o = make_float4(c < p.outputs ? v[4 * q] + __ldg(p.b_out + c) : 0.0f,
                                                     c + 1 < p.outputs ? v[4 * q + 1] + __ldg(p.b_out + c + 1) : 0.0f,
                                                     c + 2 < p.outputs ? v[4 * q + 2] + __ldg(p.b_out + c + 2) : 0.0f,
                                                     c + 3 < p.outputs ? v[4 * q + 3] + __ldg(p.b_out + c + 3) : 0.0f);
                        *reinterpret_cast<float4*>(dst + 4 * q) = o;
                    }
                }
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 2) {
        tc::fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

}  // namespace ppo
}  // namespace t8b
