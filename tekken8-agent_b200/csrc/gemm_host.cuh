// Host side of the tcgen05 GEMM: TMA descriptors (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the library needs no libcuda link) and the launcher.
#pragma once

#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "gemm.cuh"

namespace t8b {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult result{};
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &result) == cudaSuccess &&
            result == cudaDriverEntryPointSuccess) {
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        }
    });
    if (encode == nullptr) raise(T8B_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    return encode;
}

// Row-major bf16 matrix [outer][inner] with `pitch` elements per row, viewed through boxes of
// box_inner x box_outer elements with 128B swizzle (box_inner * 2 must be 128), or the 64B swizzle
// of the epilogues' 32 x 32 store tiles.
inline CUtensorMap make_map(const void* base, uint64_t inner, uint64_t outer, uint64_t pitch, uint32_t box_inner,
                            uint32_t box_outer, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (pitch * 2) % 16 != 0) {
        raise(T8B_EINVAL, "TMA operands need 16-byte aligned rows");
    }
    CUtensorMap map;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {pitch * 2};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t element[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                                            strides, box, element, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                            swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) raise(T8B_ECUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
    return map;
}

// The [rows][ld] bf16 output of a tanh epilogue, written 32 x 32 at a time (ppo::store_rows_bf16).
inline CUtensorMap make_store_map(void* base, int cols, int rows, int ld) {
    return make_map(base, static_cast<uint64_t>(cols), static_cast<uint64_t>(rows), static_cast<uint64_t>(ld), 32, 32,
                    CU_TENSOR_MAP_SWIZZLE_64B);
}

inline int sm_count() {
    static int count = 0;
    if (count == 0) {
        int device = 0;
        check(cudaGetDevice(&device), "cudaGetDevice");
        check(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device), "SM count");
    }
    return count;
}

// An operand: row-major bf16 [rows][k] (K-major) or [k][rows] (MN-major) with a row pitch.
struct Operand {
    const void* data;
    int rows, k;
    int pitch;
    bool mn_major;
};

// C[m][n] = A . B^T over k, epilogue `epi`; `splits` partitions the k blocks (split-K).
template <int BN, bool A_MN, bool B_MN, class Epi>
void gemm(const char* label, const Operand& a, const Operand& b, int splits, int* error, Epi epi, cudaStream_t stream) {
    using L = tc::Layout<BN, Epi::kEpilogueWarps, Epi::kScratchBytes>;
    if (a.k != b.k || a.mn_major != A_MN || b.mn_major != B_MN) raise(T8B_EINVAL, "GEMM operand mismatch");
    tc::Shape s{};
    s.m = a.rows;
    s.n = b.rows;
    s.k = a.k;
    s.tiles_m = (a.rows + tc::BM - 1) / tc::BM;
    s.tiles_n = (b.rows + BN - 1) / BN;
    s.k_blocks = (a.k + tc::BK - 1) / tc::BK;
    s.splits = splits < 1 ? 1 : (splits > s.k_blocks ? s.k_blocks : splits);
    s.error = error;
    const CUtensorMap ma = A_MN ? make_map(a.data, a.rows, a.k, a.pitch, 64, 64) : make_map(a.data, a.k, a.rows, a.pitch, 64, tc::BM);
    const CUtensorMap mb = B_MN ? make_map(b.data, b.rows, b.k, b.pitch, 64, 64) : make_map(b.data, b.k, b.rows, b.pitch, 64, BN);
    auto kernel = tc::gemm_kernel<BN, A_MN, B_MN, Epi>;
    static bool configured = false;
    if (!configured) {
        check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes), "GEMM smem");
        configured = true;
    }
    const int work = s.tiles_m * s.tiles_n * s.splits;
    const int grid = work < sm_count() ? work : sm_count();
    launch(label, kernel, grid, tc::threads_for<Epi>(), L::kSmemBytes, stream, ma, mb, s, epi);
    check(cudaGetLastError(), "GEMM launch");
}

}  // namespace t8b
