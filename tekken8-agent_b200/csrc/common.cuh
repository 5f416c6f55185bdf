// Shared host-side plumbing of the C ABI: status codes with a thread-local message, CUDA
// error checks that throw, and an owning device buffer.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "launch.cuh"
#include "t8b.h"

namespace t8b {

// Exceptions carry the C ABI status they map to.
struct Error : std::runtime_error {
    int code;
    Error(int status, const std::string& message) : std::runtime_error(message), code(status) {}
};

[[noreturn]] inline void raise(int status, const std::string& message) { throw Error(status, message); }

inline void check(cudaError_t result, const char* what) {
    if (result != cudaSuccess) raise(T8B_ECUDA, std::string(what) + ": " + cudaGetErrorString(result));
}

void set_last_error(const std::string& message);

// Runs body and converts any exception into a status code plus message.
template <typename Body>
int guarded(Body&& body) {
    try {
        body();
        return T8B_OK;
    } catch (const Error& error) {
        set_last_error(error.what());
        return error.code;
    } catch (const std::invalid_argument& error) {
        set_last_error(error.what());
        return T8B_EINVAL;
    } catch (const std::out_of_range& error) {
        set_last_error(error.what());
        return T8B_ERANGE;
    } catch (const std::exception& error) {
        set_last_error(error.what());
        return T8B_ECUDA;
    } catch (...) {
        set_last_error("unknown failure");
        return T8B_ECUDA;
    }
}

template <typename T>
class Buffer {
public:
    Buffer() = default;
    explicit Buffer(std::size_t count) { allocate(count); }
    ~Buffer() { release(); }
    Buffer(Buffer&& other) noexcept : data_(std::exchange(other.data_, nullptr)), count_(std::exchange(other.count_, 0)) {}
    Buffer& operator=(Buffer&& other) noexcept {
        if (this != &other) {
            release();
            data_ = std::exchange(other.data_, nullptr);
            count_ = std::exchange(other.count_, 0);
        }
        return *this;
    }
    Buffer(const Buffer&) = delete;
    Buffer& operator=(const Buffer&) = delete;

    void allocate(std::size_t count) {
        release();
        count_ = count;
        if (count > 0) {
            check(cudaMalloc(reinterpret_cast<void**>(&data_), sizeof(T) * count), "cudaMalloc");
            // The clear runs on the legacy stream, which a caller's non-blocking stream does not
            // wait for: it is complete before the buffer is handed out.
            check(cudaMemsetAsync(data_, 0, sizeof(T) * count, cudaStreamLegacy), "cudaMemset");
            check(cudaStreamSynchronize(cudaStreamLegacy), "cudaMemset");
        }
    }
    void upload(const T* host, std::size_t count, cudaStream_t stream) {
        if (count > count_) raise(T8B_EINVAL, "upload larger than the buffer");
        if (count > 0) check(cudaMemcpyAsync(data_, host, sizeof(T) * count, cudaMemcpyHostToDevice, stream), "upload");
    }
    void download(T* host, std::size_t count, cudaStream_t stream) const {
        if (count > count_) raise(T8B_EINVAL, "download larger than the buffer");
        if (count > 0) check(cudaMemcpyAsync(host, data_, sizeof(T) * count, cudaMemcpyDeviceToHost, stream), "download");
        check(cudaStreamSynchronize(stream), "synchronize download");
    }
    void zero(cudaStream_t stream) {
        if (count_ > 0) check(cudaMemsetAsync(data_, 0, sizeof(T) * count_, stream), "clear");
    }
    T* data() const noexcept { return data_; }
    std::size_t size() const noexcept { return count_; }

private:
    void release() noexcept {
        if (data_ != nullptr) cudaFree(data_);
        data_ = nullptr;
        count_ = 0;
    }
    T* data_ = nullptr;
    std::size_t count_ = 0;
};

inline unsigned blocks(std::size_t count, unsigned threads) {
    return static_cast<unsigned>((count + threads - 1) / threads);
}

}  // namespace t8b
