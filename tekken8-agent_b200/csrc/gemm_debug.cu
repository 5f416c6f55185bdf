// Test hook for the tcgen05 GEMM (no reference counterpart): C = A . B^T in fp32 through the
// split-K partial epilogue and a fixed-order reduction, for every tile width and operand major
// the policy uses.
#include "gemm_host.cuh"

namespace t8b {

// Split-K partials: part[split][row][col] (fp32), rows < m, cols < n.
struct EpiPartial {
    static constexpr int kEpilogueWarps = 4;
    static constexpr int kScratchBytes = 0;
    __device__ void prefetch(const tc::EpiCtx&) const {}
    float* part;
    int m, n;
    __device__ void operator()(const tc::EpiCtx& x, const float* v) const {
        const int row = x.row, col0 = x.col0;
        if (row >= m) return;
        float* out = part + (static_cast<size_t>(x.split) * m + row) * n + col0;
        if (col0 + 32 <= n && (n & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(out + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
            for (int i = 0; i < 32 && col0 + i < n; ++i) out[i] = v[i];
        }
    }
};

__global__ void k_reduce_splits(const float* part, float* out, size_t count, int splits) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float sum = 0.0f;
    for (int s = 0; s < splits; ++s) sum += part[static_cast<size_t>(s) * count + i];
    out[i] = sum;
}

template <int BN, bool A_MN, bool B_MN>
void debug_gemm(const void* a, const void* b, float* c, int m, int n, int k, int splits, cudaStream_t stream) {
    const Operand oa{a, m, k, A_MN ? m : k, A_MN};
    const Operand ob{b, n, k, B_MN ? n : k, B_MN};
    const int k_blocks = (k + tc::BK - 1) / tc::BK;
    const int used = splits < 1 ? 1 : (splits > k_blocks ? k_blocks : splits);
    Buffer<float> part(static_cast<size_t>(used) * m * n);
    Buffer<int> error(1);
    gemm<BN, A_MN, B_MN>("gemm_debug", oa, ob, used, error.data(), EpiPartial{part.data(), m, n}, stream);
    const size_t count = static_cast<size_t>(m) * n;
    launch("k_reduce_splits", k_reduce_splits, blocks(count, 256), 256, 0, stream, part.data(), c, count, used);
    check(cudaGetLastError(), "reduce splits");
    int flag = 0;
    error.download(&flag, 1, stream);
    if (flag) raise(T8B_ECUDA, "GEMM wait timed out");
}

}  // namespace t8b

extern "C" int t8b_debug_gemm(const void* a, int a_mn_major, const void* b, int b_mn_major, float* c, int m, int n,
                              int k, int bn, int splits, void* stream) {
    using namespace t8b;
    return guarded([&] {
        if (!a || !b || !c || m <= 0 || n <= 0 || k <= 0) raise(T8B_EINVAL, "GEMM arguments");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const int key = bn * 4 + (a_mn_major ? 2 : 0) + (b_mn_major ? 1 : 0);
        switch (key) {
            case 256 * 4 + 0: debug_gemm<256, false, false>(a, b, c, m, n, k, splits, s); break;
            case 256 * 4 + 3: debug_gemm<256, true, true>(a, b, c, m, n, k, splits, s); break;
            case 192 * 4 + 0: debug_gemm<192, false, false>(a, b, c, m, n, k, splits, s); break;
            case 192 * 4 + 3: debug_gemm<192, true, true>(a, b, c, m, n, k, splits, s); break;
            case 64 * 4 + 0: debug_gemm<64, false, false>(a, b, c, m, n, k, splits, s); break;
            case 64 * 4 + 3: debug_gemm<64, true, true>(a, b, c, m, n, k, splits, s); break;
            case 256 * 4 + 2: debug_gemm<256, true, false>(a, b, c, m, n, k, splits, s); break;
            default: raise(T8B_EINVAL, "unsupported GEMM tile/major combination");
        }
    });
}

namespace t8b {

// One thread waits on an mbarrier with the GEMM's bounded wait; with `arrive` the barrier's
// phase completes first, otherwise nothing ever arrives and the wait runs out after `limit`
// polls. status[0] = 1 when the wait gave up, 0 when it saw the phase.
__global__ void k_bounded_wait(int arrive, uint32_t limit, int* status) {
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x != 0) return;
    abort = 0;
    tc::bar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (arrive) tc::bar_arrive(&bar);
    const bool seen = tc::bar_wait(&bar, 0, &abort, limit);
    status[0] = seen ? 0 : 1;
}

}  // namespace t8b

extern "C" int t8b_debug_bounded_wait(int arrive, uint32_t spin_limit, int* timed_out) {
    using namespace t8b;
    return guarded([&] {
        if (!timed_out || spin_limit == 0) raise(T8B_EINVAL, "bounded wait arguments");
        Buffer<int> status(1);
        launch("k_bounded_wait", k_bounded_wait, 1, 32, 0, nullptr, arrive, spin_limit, status.data());
        check(cudaGetLastError(), "bounded wait");
        status.download(timed_out, 1, nullptr);
    });
}
