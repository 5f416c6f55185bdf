// Library-internal entry points between the translation units (C++ linkage, not exported in
// include/t8b.h): the row-range and fight-group forms of the simulator, policy and rollout calls
// that the native rollout loop (trainer.cu) uses to run two halves of the fights on two streams.
#pragma once

#include <cuda_runtime.h>

#include "t8b.h"

namespace t8b::internal {

// Splits the simulator's fights into `groups` contiguous ranges (1: all fights, the default).
void sim_set_groups(t8b_sim* sim, int groups);
size_t sim_group_first(const t8b_sim* sim, int group);
size_t sim_group_count(const t8b_sim* sim, int group);
// env_step over one group's fights on `stream`; candidates are the batch's base pointers.
void sim_step_group(t8b_sim* sim, int group, const int64_t* learner, const int64_t* opponent, uint64_t seed,
                    uint64_t counter, bool reset, cudaStream_t stream);

// env_step over all fights (one group) on `stream` without the learner's masks, which
// sim_learner_masks then computes on another stream (they depend only on the new states).
void sim_step_without_masks(t8b_sim* sim, const int64_t* learner, const int64_t* opponent, uint64_t seed,
                            uint64_t counter, bool reset, cudaStream_t stream);
void sim_learner_masks(t8b_sim* sim, cudaStream_t stream);

// The policy's forward on rows [row, row + n) of a batch (base pointers in; outputs in those rows
// of the buffers `out` points at, with the same samples a whole-batch forward would draw).
// With `masks_ready`, the sampler (the only part that reads the masks) waits for that event, so
// the input preparation and the network's GEMMs run while the masks are still being computed.
void policy_forward_rows(t8b_policy* policy, size_t row, size_t n, const float* observations, const uint32_t* mask_bits,
                         const int32_t* tables, uint64_t seed, uint64_t step, int deterministic, cudaStream_t stream,
                         t8b_policy_output_t* out, cudaEvent_t masks_ready = nullptr);

// record_policy_device / record_outcome_device for environments [row, row + n) of one step.
void rollout_record_policy_rows(t8b_rollout* rollout, size_t step, size_t row, size_t n, const float* observations,
                                const uint32_t* mask_bits, const int64_t* actions, const float* log_probabilities,
                                const float* values, const int32_t* tables, const float* entropies, cudaStream_t stream);
void rollout_record_outcome_rows(t8b_rollout* rollout, size_t step, size_t row, size_t n, const float* rewards,
                                 const uint8_t* terminated, const uint8_t* truncated, const float* next_values,
                                 float reward_scale, cudaStream_t stream);

}  // namespace t8b::internal
