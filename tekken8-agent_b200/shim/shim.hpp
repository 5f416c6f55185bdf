// The reference's C++ classes over the C ABI: shared pieces of the shim.
//
// The shim keeps the reference's headers (include/t8_v2/full_move_gpu.hpp, ppo.hpp) and
// replaces the implementation files behind them (src/full_move_gpu.cu and the GpuActorCritic /
// GpuRolloutBuffer part of src/ppo.cu) with calls into libt8b.so, so the programs built on those
// headers (the full-move trainer, arena and benchmark) compile unchanged. Status codes become
// the exceptions the reference throws (src/full_move_gpu.cu:17-21, src/ppo.cu:87-98):
// T8B_EINVAL std::invalid_argument, T8B_ERANGE std::out_of_range, T8B_ESTATE std::logic_error,
// anything else std::runtime_error.
#pragma once

#include "t8b.h"

#include <cstring>
#include <stdexcept>
#include <string>

namespace t8::v2::shim {

inline void ok(int status) {
    if (status == T8B_OK) return;
    const std::string message = t8b_last_error();
    switch (status) {
        case T8B_EINVAL: throw std::invalid_argument(message);
        case T8B_ERANGE: throw std::out_of_range(message);
        case T8B_ESTATE: throw std::logic_error(message);
        default: throw std::runtime_error(message);
    }
}

// Copies a std::string into a fixed, NUL-padded field (longer text is cut to the field).
template <std::size_t N>
void copy_text(char (&field)[N], const std::string& text) {
    std::memset(field, 0, N);
    std::memcpy(field, text.data(), text.size() < N ? text.size() : N);
}

}  // namespace t8::v2::shim
