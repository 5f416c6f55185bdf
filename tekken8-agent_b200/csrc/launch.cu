// Launch counting and optional per-kernel event timing behind t8b_launch_count,
// t8b_profile_enable and t8b_profile_report.
#include "common.cuh"
#include "launch.cuh"

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace t8b {
namespace {

struct Timing {
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
    double ms = 0.0;
    uint64_t launches = 0;
};

std::atomic<uint64_t> g_launches{0};
std::atomic<bool> g_profiling{false};
std::atomic<bool> g_filtered{false};
std::mutex g_lock;
std::string g_only;  // the one label bracketed while g_filtered
std::map<std::string, Timing> g_timings;
std::vector<cudaEvent_t> g_pool;

cudaEvent_t take_event() {
    if (!g_pool.empty()) {
        cudaEvent_t e = g_pool.back();
        g_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

}  // namespace

LaunchScope::LaunchScope(const char* n, cudaStream_t s) : name(n), stream(s) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (g_profiling.load(std::memory_order_relaxed)) {
        std::lock_guard<std::mutex> guard(g_lock);
        if (g_filtered.load(std::memory_order_relaxed) && g_only != name) return;
        start = take_event();
        cudaEventRecord(start, stream);
    }
}

LaunchScope::~LaunchScope() {
    if (start == nullptr) return;
    std::lock_guard<std::mutex> guard(g_lock);
    cudaEvent_t end = take_event();
    cudaEventRecord(end, stream);
    g_timings[name].pending.emplace_back(start, end);
}

}  // namespace t8b

extern "C" {

/* Launch count since load (every kernel of the library). */
uint64_t t8b_launch_count(void) { return t8b::g_launches.load(); }

/* Per-kernel event timing on (1) or off (0); turning it on clears earlier results. */
void t8b_profile_enable(int on) {
    std::lock_guard<std::mutex> guard(t8b::g_lock);
    if (on) t8b::g_timings.clear();
    t8b::g_profiling.store(on != 0);
}

/* Event bracketing for launches labelled `label` only (NULL: every launch). */
void t8b_profile_only(const char* label) {
    std::lock_guard<std::mutex> guard(t8b::g_lock);
    t8b::g_only = label != nullptr ? label : "";
    t8b::g_filtered.store(label != nullptr);
}

/* Synchronises the device, folds the recorded events into totals and writes one line per
 * kernel name, "name launches total_ms", into `text` (NUL-terminated). Returns the length
 * needed. */
size_t t8b_profile_report(char* text, size_t capacity) {
    cudaDeviceSynchronize();
    std::lock_guard<std::mutex> guard(t8b::g_lock);
    std::string out;
    for (auto& [name, timing] : t8b::g_timings) {
        for (auto& [a, b] : timing.pending) {
            float ms = 0.0f;
            if (cudaEventElapsedTime(&ms, a, b) == cudaSuccess) timing.ms += ms;
            t8b::g_pool.push_back(a);
            t8b::g_pool.push_back(b);
            ++timing.launches;
        }
        timing.pending.clear();
        out += name + " " + std::to_string(timing.launches) + " " + std::to_string(timing.ms) + "\n";
    }
    if (text != nullptr && capacity > 0) {
        const size_t n = out.size() < capacity - 1 ? out.size() : capacity - 1;
        out.copy(text, n);
        text[n] = 0;
    }
    return out.size() + 1;
}

}  // extern "C"
