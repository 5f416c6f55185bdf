// tcgen05 GEMM for sm_100a: C[M,N] (+)= A[M,K] . B[N,K]^T in bf16 with fp32 accumulation in
// tensor memory, fed by TMA, with the epilogue fused by a functor.
//
// One persistent CTA per SM, 192 or 320 threads:
//   warp 0     TMA producer: one elected thread loads A and B k-blocks (64 wide) into a ring of
//              shared-memory stages (128B swizzle), arriving on full[stage];
//   warp 1     MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16) per 16-wide slice and
//              commits each stage back to empty[stage]; the accumulator of a finished tile is
//              committed to acc_full[buffer];
//   warps 2-5 or 2-9  epilogue: tcgen05.ld of their 32 TMEM lanes (lane quarter = warp % 4), 32
//              columns at a time (with 8 warps, the two of a quarter take alternate chunks), handed to the
//              epilogue functor with a 6.5 KB warp-private shared-memory
//              scratch (for staging a 32 x 32 chunk so global rows are read whole, and so a bf16
//              chunk leaves as one TMA store);
//              the functor's prefetch of chunk c + 1 is issued before chunk c is loaded from
//              tensor memory; then acc_empty[buffer] frees the buffer.
// Two accumulator buffers of BN columns let the epilogue of tile i overlap the MMAs of tile i+1.
// Operands are K-major (row-major [rows][K]) or MN-major (row-major [K][rows]); the MN-major form
// lets weight gradients read activations [samples][features] directly with the samples as K.
// Work items are (m tile, n tile, k split); a split-K item writes a partial the caller reduces.
// Every wait is bounded: a stall sets the error flag, the CTA drains and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace t8b {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;
// Epilogue warps: a functor's kEpilogueWarps, 4 (one per lane quarter of the accumulator) or 8
// (two per quarter, alternating 32-column chunks).
template <class Epi>
constexpr int threads_for() { return 64 + 32 * Epi::kEpilogueWarps; }
constexpr uint32_t kSpinLimit = 1u << 24;

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void bar_expect(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Waits for the phase with the given parity; false after the spin limit or an abort.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                         uint32_t limit = kSpinLimit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (bar_try(bar, parity)) return true;
        if (*abort) return false;
    }
    return false;
}

__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

// Tiled TMA store of a shared-memory tile to the tensor map's box at (x, y) (rows and columns past
// the tensor are not written), in this thread's bulk async-group.
__device__ __forceinline__ void tma_store(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
                 "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// this thread's bulk stores have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// all but the most recent of this thread's bulk stores have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_all_but_one() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// this thread's bulk stores are complete
__device__ __forceinline__ void bulk_wait() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,"
        "%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, 128B swizzle (sm_100 descriptor version 1).
// K-major: 8-row groups of 128 B rows, group stride (SBO) 1024 B; 16-wide K steps advance
// the start address by 32 B inside the swizzle span. MN-major: 64-element MN atoms of 8 KB
// (LBO) holding 64 K rows, 8-row groups 1024 B apart (SBO); K steps advance 2048 B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((addr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16) |
        (static_cast<uint64_t>(sbo >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, M = 128.
__host__ __device__ constexpr uint32_t instr_desc(int n, bool a_mn, bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn) << 15) | (static_cast<uint32_t>(b_mn) << 16) |
        (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

// What an epilogue functor sees for one 32 x 32 chunk of a tile (one warp, 32 rows).
struct EpiCtx {
    int row;      // this lane's row (row0 + lane)
    int row0;     // first of the warp's 32 rows
    int col0;     // first of the chunk's 32 columns
    int split, tm, quarter, lane;
    unsigned char* scratch;  // warp-private, Epi::kScratchBytes
    int buffer;   // prefetch buffer (0 or 1) holding this chunk's inputs
    bool more;    // the next chunk's prefetch has been issued after this one's
    int chunk;    // chunks this warp has handed to the functor before this one (all tiles)
};
// Shared-memory scratch per epilogue warp of the epilogues that stage chunks (a functor's
// kScratchBytes; multiples of 512 keep every warp's staging tile aligned for the 64B swizzle).
constexpr int kEpiWarpBytes = 6656;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Byte offset of 16-byte piece q of row r in a 32-row tile with `pieces` pieces per row,
// rotated so that a warp writing one piece of 8 consecutive rows, or reading whole rows 8 at
// a time, touches every bank once.
__device__ __forceinline__ int staged_piece(int r, int q, int pieces) {
    return pieces == 4 ? r * 64 + ((q ^ ((r >> 1) & 3)) << 4) : r * (pieces * 16) + ((q ^ (r & 7)) << 4);
}

struct Shape {
    int m, n, k;        // GEMM extents (m rows of A and C, n rows of B, k reduction)
    int tiles_m, tiles_n, splits;
    int k_blocks;       // ceil(k / 64)
    int* error;         // set to 1 on a stalled wait
};

template <int BN, int EW, int SCRATCH>
struct Layout {
    static constexpr int kABytes = BM * BK * 2;
    static constexpr int kBBytes = BN * BK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kEpiBytes = EW * SCRATCH;
    // stages fill what the 227 KB of a CTA leaves after the epilogue scratch and barriers
    static constexpr int kStageBudget = 232448 - 1024 - 256 - kEpiBytes;
    static constexpr int kStages = kStageBudget / kStageBytes > 8 ? 8 : kStageBudget / kStageBytes;
    static constexpr int kTmemCols = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
    static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kEpiBytes + 256;
};

template <int BN, bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(threads_for<Epi>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Shape s,
                const __grid_constant__ Epi epi) {
    constexpr int EW = Epi::kEpilogueWarps;
    static_assert(EW == 4 || EW == 8, "4 or 8 epilogue warps");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
    static_assert(!B_MN || BN % 64 == 0, "MN-major B tiles are whole 64-wide atoms");
    static_assert(Epi::kScratchBytes % 512 == 0, "warp scratch in 512-byte units");
    using L = Layout<BN, EW, Epi::kScratchBytes>;
    extern __shared__ __align__(1024) unsigned char raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    unsigned char* stages = base;
    unsigned char* epi_scratch = base + L::kStages * L::kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(epi_scratch + L::kEpiBytes);
    uint64_t* empty = full + L::kStages;
    uint64_t* acc_full = empty + L::kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < L::kStages; ++i) {
            bar_init(full + i, 1);
            bar_init(empty + i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            bar_init(acc_full + i, 1);
            bar_init(acc_empty + i, EW * 32);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(L::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = s.tiles_m * s.tiles_n * s.splits;

    auto decode = [&](int work, int& tm, int& tn, int& kb0, int& kb1, int& split) {
        tn = work % s.tiles_n;
        const int rest = work / s.tiles_n;
        tm = rest % s.tiles_m;
        split = rest / s.tiles_m;
        kb0 = static_cast<int>((static_cast<long long>(s.k_blocks) * split) / s.splits);
        kb1 = static_cast<int>((static_cast<long long>(s.k_blocks) * (split + 1)) / s.splits);
    };
    auto stop = [&]() {
        *abort = 1;
        if (s.error) atomicExch(s.error, 1);
    };

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int work = blockIdx.x; work < total && !*abort; work += gridDim.x) {
                int tm, tn, kb0, kb1, split;
                decode(work, tm, tn, kb0, kb1, split);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!bar_wait(empty + stage, phase ^ 1u, abort)) {
                        stop();
                        break;
                    }
                    unsigned char* a = stages + stage * L::kStageBytes;
                    unsigned char* b = a + L::kABytes;
                    bar_expect(full + stage, L::kStageBytes);
                    if (A_MN) {
                        for (int j = 0; j < BM / 64; ++j) tma_load(a + j * 8192, &map_a, full + stage, tm * BM + j * 64, kb * BK);
                    } else {
                        tma_load(a, &map_a, full + stage, kb * BK, tm * BM);
                    }
                    if (B_MN) {
                        for (int j = 0; j < BN / 64; ++j) tma_load(b + j * 8192, &map_b, full + stage, tn * BN + j * 64, kb * BK);
                    } else {
                        tma_load(b, &map_b, full + stage, kb * BK, tn * BN);
                    }
                    if (++stage == L::kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = instr_desc(BN, A_MN, B_MN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int work = blockIdx.x; work < total && !*abort; work += gridDim.x) {
                int tm, tn, kb0, kb1, split;
                decode(work, tm, tn, kb0, kb1, split);
                if (!bar_wait(acc_empty + acc, acc_phase ^ 1u, abort)) {
                    stop();
                    break;
                }
                fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(acc * BN);
                bool ok = true;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!bar_wait(full + stage, phase, abort)) {
                        stop();
                        ok = false;
                        break;
                    }
                    fence_after();
                    const uint32_t a = smem_addr(stages + stage * L::kStageBytes);
                    const uint32_t b = a + L::kABytes;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint64_t da = A_MN ? sw128_desc(a + k * 2048, 8192, 1024) : sw128_desc(a + k * 32, 16, 1024);
                        const uint64_t db = B_MN ? sw128_desc(b + k * 2048, 8192, 1024) : sw128_desc(b + k * 32, 16, 1024);
                        mma(d, da, db, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
                    }
                    commit(empty + stage);
                    if (++stage == L::kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                commit(acc_full + acc);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
    } else {
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;  // which alternate 32-column chunks this warp takes (EW = 8)
        constexpr int stride = EW / 4;
        unsigned char* scratch = epi_scratch + (warp - 2) * Epi::kScratchBytes;
        int acc = 0;
        uint32_t acc_phase = 0;
        int chunks = 0;
        float v[32];
        for (int work = blockIdx.x; work < total && !*abort; work += gridDim.x) {
            int tm, tn, kb0, kb1, split;
            decode(work, tm, tn, kb0, kb1, split);
            EpiCtx x;
            x.row0 = tm * BM + quarter * 32;
            x.row = x.row0 + lane;
            x.split = split;
            x.tm = tm;
            x.quarter = quarter;
            x.lane = lane;
            x.scratch = scratch;
            x.col0 = tn * BN + half * 32;
            x.buffer = 0;
            epi.prefetch(x);
            if (!bar_wait(acc_full + acc, acc_phase, abort)) {
                stop();
                break;
            }
            fence_after();
            const uint32_t t = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
            const bool empty_k = kb1 <= kb0;
#pragma unroll 1
            for (int c = half, n = 0; c < BN / 32; c += stride, ++n) {
                x.more = c + stride < BN / 32;
                if (x.more) {
                    EpiCtx next = x;
                    next.col0 = tn * BN + (c + stride) * 32;
                    next.buffer = (n + 1) & 1;
                    epi.prefetch(next);
                }
                tmem_load32(t + static_cast<uint32_t>(c * 32), v);
                if (empty_k) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.0f;
                }
                x.col0 = tn * BN + c * 32;
                x.buffer = n & 1;
                x.chunk = chunks++;
                epi(x, v);
            }
            fence_before();
            bar_arrive(acc_empty + acc);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        bulk_wait();  // an epilogue's TMA stores (issued by lane 0) have landed
    }
    fence_before();
    __syncthreads();
    if (warp == 2) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::kTmemCols));
    }
}

}  // namespace tc
}  // namespace t8b
