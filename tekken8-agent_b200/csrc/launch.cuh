// Every kernel of the library is launched through launch(): it counts launches (the count a
// benchmark reports) and, while profiling is on, brackets the launch with CUDA events on its
// stream so per-kernel device time can be read back without a profiler.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace t8b {

struct LaunchScope {
    LaunchScope(const char* name, cudaStream_t stream);
    ~LaunchScope();
    const char* name;
    cudaStream_t stream;
    cudaEvent_t start = nullptr;
};

template <typename Kernel, typename... Args>
inline void launch(const char* name, Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args... args) {
    LaunchScope scope(name, stream);
    kernel<<<grid, block, smem, stream>>>(args...);
}

}  // namespace t8b
