// Native data-parallel communicator: t8b_comm_t hooks backed by NCCL, for a C or C++ host (the
// reference's trainer is one) that drives one GPU per process and has no Python or torch.
//
// NCCL is opened at run time (dlopen of libnccl.so.2) when the first communicator is made, so a
// single-GPU user needs no NCCL, and a process that already loaded one (torch bundles its own)
// shares that copy instead of mapping a second. The hooks call ncclAllReduce (sum) on the
// library's stream, so the all-reduce is ordered with the kernels around it and the host never
// waits for it; the library calls them at the exchange points of a data-parallel PPO update
// (the minibatch gradient, the epoch KL, the rollout statistics), which every rank reaches in the
// same order.
#include "common.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <type_traits>

namespace t8b {
namespace {

struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

const Nccl& nccl() {
    static Nccl api;
    static std::string failure;
    static std::once_flag once;
    std::call_once(once, [] {
        void* handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (handle == nullptr) handle = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (handle == nullptr) {
            failure = std::string("cannot load NCCL (libnccl.so.2): ") + dlerror();
            return;
        }
        const auto symbol = [&](auto& slot, const char* name) {
            slot = reinterpret_cast<std::remove_reference_t<decltype(slot)>>(dlsym(handle, name));
            if (slot == nullptr && failure.empty()) failure = std::string("NCCL lacks ") + name;
        };
        symbol(api.get_unique_id, "ncclGetUniqueId");
        symbol(api.init_rank, "ncclCommInitRank");
        symbol(api.all_reduce, "ncclAllReduce");
        symbol(api.destroy, "ncclCommDestroy");
        symbol(api.async_error, "ncclCommGetAsyncError");
        symbol(api.error_string, "ncclGetErrorString");
    });
    if (!failure.empty()) raise(T8B_ECUDA, failure);
    return api;
}

void nccl_check(ncclResult_t result, const char* what) {
    if (result != ncclSuccess) raise(T8B_ECUDA, std::string(what) + ": " + nccl().error_string(result));
}

// A hook that fails has no status to return: it records the failure, which t8b_comm_status
// reports, and the collective is skipped on this rank (the others then wait in theirs until
// NCCL's own timeout, as with any rank that drops out).
struct Native {
    ncclComm_t comm = nullptr;
    int device = 0;
    std::string failure;
};

void reduce(Native* native, void* data, size_t count, ncclDataType_t type, void* stream) {
    if (count == 0 || !native->failure.empty()) return;
    const ncclResult_t r = nccl().all_reduce(data, data, count, type, ncclSum, native->comm,
                                             static_cast<cudaStream_t>(stream));
    if (r != ncclSuccess) native->failure = std::string("ncclAllReduce: ") + nccl().error_string(r);
}

void reduce_f32(float* data, size_t count, void* stream, void* user) {
    reduce(static_cast<Native*>(user), data, count, ncclFloat32, stream);
}

void reduce_f64(double* data, size_t count, void* stream, void* user) {
    reduce(static_cast<Native*>(user), data, count, ncclFloat64, stream);
}

}  // namespace
}  // namespace t8b

using namespace t8b;

extern "C" {

int t8b_comm_unique_id(void* id, size_t size) {
    return guarded([&] {
        if (id == nullptr || size < sizeof(ncclUniqueId)) raise(T8B_EINVAL, "the unique id needs 128 bytes");
        ncclUniqueId unique;
        nccl_check(nccl().get_unique_id(&unique), "ncclGetUniqueId");
        std::memcpy(id, &unique, sizeof unique);
    });
}

int t8b_comm_init(const void* id, size_t size, int world_size, int rank, t8b_comm_t* out) {
    return guarded([&] {
        if (id == nullptr || size < sizeof(ncclUniqueId) || out == nullptr) raise(T8B_EINVAL, "null argument");
        if (world_size < 1 || rank < 0 || rank >= world_size) raise(T8B_ERANGE, "rank outside the world");
        ncclUniqueId unique;
        std::memcpy(&unique, id, sizeof unique);
        auto native = std::make_unique<Native>();
        check(cudaGetDevice(&native->device), "cudaGetDevice");
        nccl_check(nccl().init_rank(&native->comm, world_size, unique, rank), "ncclCommInitRank");
        *out = t8b_comm_t{};
        out->allreduce_sum_f32 = reduce_f32;
        out->allreduce_sum_f64 = reduce_f64;
        out->user = native.release();
        out->world_size = world_size;
        out->rank = rank;
    });
}

int t8b_comm_status(const t8b_comm_t* comm) {
    return guarded([&] {
        if (comm == nullptr || comm->user == nullptr) raise(T8B_EINVAL, "null communicator");
        auto* native = static_cast<Native*>(comm->user);
        if (!native->failure.empty()) raise(T8B_ECUDA, native->failure);
        ncclResult_t pending = ncclSuccess;
        nccl_check(nccl().async_error(native->comm, &pending), "ncclCommGetAsyncError");
        nccl_check(pending, "NCCL communicator");
    });
}

int t8b_comm_allreduce_sum_f32(const t8b_comm_t* comm, float* data, size_t count, void* stream) {
    return guarded([&] {
        if (comm == nullptr || comm->user == nullptr) raise(T8B_EINVAL, "null communicator");
        reduce_f32(data, count, stream, comm->user);
        auto* native = static_cast<Native*>(comm->user);
        if (!native->failure.empty()) raise(T8B_ECUDA, native->failure);
    });
}

int t8b_comm_destroy(t8b_comm_t* comm) {
    return guarded([&] {
        if (comm == nullptr || comm->user == nullptr) return;
        auto* native = static_cast<Native*>(comm->user);
        const ncclResult_t r = nccl().destroy(native->comm);
        delete native;
        *comm = t8b_comm_t{};
        nccl_check(r, "ncclCommDestroy");
    });
}

}  // extern "C"
