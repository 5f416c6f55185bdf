// The trainer's rollout loop (src/full_move_train.cpp:1374-1400) as one native call over the
// simulator, the policy and the rollout buffer, so no interpreter sits between the ~15 launches
// of a decision. With one process per GPU on a shared host, a per-decision Python loop can fall
// behind the GPU; this loop issues a decision in tens of microseconds.
//
// Per decision: the learner's forward (sampling, seed + 1), the previous decision's outcome with
// this forward's values as its bootstrap (for a fight whose round ended the bootstrap is the
// reset state's value, which GAE multiplies by zero: terminated and never truncated), the
// decision itself, the simulator step, and the reset of finished rounds. After the last
// decision one deterministic forward (seed + 3) gives the final bootstrap. With a frozen
// opponent policy its forward (seed + 2) runs on a second stream that overlaps the learner's.
// Every decision but the last steps and resets in one launch (the reset of t8b_sim_step_and_reset):
// nothing reads the terminal observations there, while the last decision's bootstrap forward
// does. The learner's masks of those steps are computed on a second stream while the next
// forward prepares its inputs and runs its GEMMs; its sampler waits for them.
//
//
// With T8B_ROLLOUT_GROUPS=2 in the environment (scripted opponents, at least 8,192 fights) the
// fights are split into two groups (contiguous halves) and each half's decision runs on a stream
// of its own, so one half's forward, sampler, masks and records can run beside the other half's
// frame step. Everything per fight is the same computation as in one stream (the sampler's
// uniforms are keyed by the fight's row), so the rollout is bit-identical. It is off by default:
// at 32,768 fights it measured 465.7 ms per iteration against 432.8 ms on one stream, because the
// frame step is bound by instruction fetch and the kernels sharing its SMs evict its code.
#include "common.cuh"
#include "internal.cuh"

#include <cstdlib>

namespace {

int rollout_groups(size_t fights, bool opponent) {
    const char* text = std::getenv("T8B_ROLLOUT_GROUPS");
    const int configured = text != nullptr ? std::atoi(text) : 1;
    if (opponent || fights < 8192) return 1;
    return configured == 2 ? 2 : 1;
}

// The grouped loop: per decision and group, on the group's stream, the learner's forward on the
// group's rows, the previous decision's outcome, the record and the group's step (with the reset
// of finished rounds); after the last decision the bootstrap forward per group, then one reset
// of finished rounds over all fights on the main stream.
void collect_grouped(t8b_sim* sim, t8b_policy* policy, t8b_rollout* rollout, uint64_t seed, uint64_t update,
                     size_t horizon, float reward_scale, cudaStream_t main) {
    using namespace t8b;
    const auto ok = [](int status) {
        if (status != T8B_OK) raise(status, t8b_last_error());
    };
    constexpr int kGroups = 2;
    internal::sim_set_groups(sim, kGroups);
    cudaStream_t streams[kGroups] = {};
    cudaEvent_t done[kGroups] = {};
    cudaEvent_t start = nullptr;
    struct Cleanup {
        cudaStream_t* streams;
        cudaEvent_t* done;
        cudaEvent_t* start;
        ~Cleanup() {
            for (int g = 0; g < kGroups; ++g) {
                if (done[g]) cudaEventDestroy(done[g]);
                if (streams[g]) cudaStreamDestroy(streams[g]);
            }
            if (*start) cudaEventDestroy(*start);
        }
    } cleanup{streams, done, &start};
    check(cudaEventCreateWithFlags(&start, cudaEventDisableTiming), "event");
    for (int g = 0; g < kGroups; ++g) {
        // blocking streams: the legacy stream (the uint8 mask expansion of the reference view)
        // waits for them
        check(cudaStreamCreate(&streams[g]), "group stream");
        check(cudaEventCreateWithFlags(&done[g], cudaEventDisableTiming), "event");
    }
    check(cudaEventRecord(start, main), "event");
    for (int g = 0; g < kGroups; ++g) check(cudaStreamWaitEvent(streams[g], start, 0), "wait");
    const int32_t* tables = t8b_sim_learner_feature_tables(sim);
    const float* obs = t8b_sim_learner_observations(sim);
    const uint32_t* bits = t8b_sim_learner_mask_bits(sim);
    for (size_t step = 0; step < horizon; ++step) {
        const uint64_t counter = update * horizon + step;
        for (int g = 0; g < kGroups; ++g) {
            const size_t row = internal::sim_group_first(sim, g), n = internal::sim_group_count(sim, g);
            cudaStream_t st = streams[g];
            t8b_policy_output_t out{};
            internal::policy_forward_rows(policy, row, n, obs, bits, tables, seed + 1, counter, 0, st, &out);
            if (step > 0) {
                internal::rollout_record_outcome_rows(rollout, step - 1, row, n, t8b_sim_rewards(sim),
                                                      t8b_sim_terminated(sim), t8b_sim_truncated(sim), out.values,
                                                      reward_scale, st);
            }
            internal::rollout_record_policy_rows(rollout, step, row, n, obs, bits, out.actions, out.log_probabilities,
                                                 out.values, tables, out.entropies, st);
            internal::sim_step_group(sim, g, out.actions, nullptr, seed, counter + 1, step + 1 < horizon, st);
            if (step + 1 == horizon) {
                t8b_policy_output_t last{};
                internal::policy_forward_rows(policy, row, n, obs, bits, tables, seed + 3, counter, 1, st, &last);
                internal::rollout_record_outcome_rows(rollout, step, row, n, t8b_sim_rewards(sim),
                                                      t8b_sim_terminated(sim), t8b_sim_truncated(sim), last.values,
                                                      reward_scale, st);
            }
        }
    }
    for (int g = 0; g < kGroups; ++g) {
        check(cudaEventRecord(done[g], streams[g]), "event");
        check(cudaStreamWaitEvent(main, done[g], 0), "wait");
    }
    ok(t8b_sim_reset_done(sim, seed, update * horizon + horizon));
}

}  // namespace

extern "C" int t8b_collect_rollout(t8b_sim* sim, t8b_policy* policy, t8b_rollout* rollout, t8b_policy* opponent,
                                   uint64_t seed, uint64_t update, size_t horizon, float reward_scale, void* stream) {
    using namespace t8b;
    return guarded([&] {
        if (!sim || !policy || !rollout || horizon == 0) raise(T8B_EINVAL, "rollout arguments");
        const size_t n = t8b_sim_environment_count(sim);
        cudaStream_t main = static_cast<cudaStream_t>(stream);
        auto ok = [](int status) {
            if (status != T8B_OK) raise(status, t8b_last_error());
        };
        ok(t8b_sim_set_stream(sim, stream));
        if (rollout_groups(n, opponent != nullptr) > 1) {
            collect_grouped(sim, policy, rollout, seed, update, horizon, reward_scale, main);
            return;
        }
        internal::sim_set_groups(sim, 1);
        cudaStream_t side = nullptr, mask_stream = nullptr;
        cudaEvent_t sim_ready = nullptr, opponent_done = nullptr, stepped = nullptr, masks_ready = nullptr;
        struct Cleanup {
            cudaStream_t* streams[2];
            cudaEvent_t* events[4];
            ~Cleanup() {
                for (cudaEvent_t* e : events) {
                    if (*e) cudaEventDestroy(*e);
                }
                for (cudaStream_t* s : streams) {
                    if (*s) cudaStreamDestroy(*s);
                }
            }
        } cleanup{{&side, &mask_stream}, {&sim_ready, &opponent_done, &stepped, &masks_ready}};
        if (opponent) {
            check(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking), "opponent stream");
            check(cudaEventCreateWithFlags(&sim_ready, cudaEventDisableTiming), "event");
            check(cudaEventCreateWithFlags(&opponent_done, cudaEventDisableTiming), "event");
        }
        // the learner's masks of a step run on their own stream beside the next forward's input
        // preparation and GEMMs (only its sampler reads them)
        check(cudaStreamCreateWithFlags(&mask_stream, cudaStreamNonBlocking), "mask stream");
        check(cudaEventCreateWithFlags(&stepped, cudaEventDisableTiming), "event");
        check(cudaEventCreateWithFlags(&masks_ready, cudaEventDisableTiming), "event");
        bool masks_pending = false;
        const int32_t* tables = t8b_sim_learner_feature_tables(sim);
        t8b_policy_output_t out{}, last{}, theirs{};
        for (size_t step = 0; step < horizon; ++step) {
            const uint64_t counter = update * horizon + step;
            const float* obs = t8b_sim_learner_observations(sim);
            const uint32_t* bits = t8b_sim_learner_mask_bits(sim);
            const int64_t* opponent_actions = nullptr;
            if (opponent) {
                const float* their_obs = t8b_sim_opponent_observations(sim);
                const uint32_t* their_bits = t8b_sim_opponent_mask_bits(sim);  // computed on the main stream
                const int32_t* their_tables = t8b_sim_opponent_feature_tables(sim);
                if (!their_bits) raise(T8B_ECUDA, t8b_last_error());
                check(cudaEventRecord(sim_ready, main), "event");
                check(cudaStreamWaitEvent(side, sim_ready, 0), "wait");
                ok(t8b_policy_forward(opponent, their_obs, nullptr, their_bits, n, seed + 2, counter, 0, side,
                                      their_tables, 0, &theirs));
                check(cudaEventRecord(opponent_done, side), "event");
                opponent_actions = theirs.actions;
            }
            internal::policy_forward_rows(policy, 0, n, obs, bits, tables, seed + 1, counter, 0, main, &out,
                                          masks_pending ? masks_ready : nullptr);
            masks_pending = false;
            if (step > 0) {
                ok(t8b_rollout_record_outcome_device(rollout, step - 1, t8b_sim_rewards(sim), t8b_sim_terminated(sim),
                                                     t8b_sim_truncated(sim), out.values, reward_scale, stream));
            }
            ok(t8b_rollout_record_policy_device(rollout, step, obs, nullptr, bits, out.actions, out.log_probabilities,
                                                out.values, stream, tables, out.entropies));
            if (opponent) check(cudaStreamWaitEvent(main, opponent_done, 0), "wait");
            if (step + 1 < horizon) {
                internal::sim_step_without_masks(sim, out.actions, opponent_actions, seed, counter + 1, true, main);
                check(cudaEventRecord(stepped, main), "event");
                check(cudaStreamWaitEvent(mask_stream, stepped, 0), "wait");
                internal::sim_learner_masks(sim, mask_stream);
                check(cudaEventRecord(masks_ready, mask_stream), "event");
                masks_pending = true;
                continue;
            }
            ok(t8b_sim_step(sim, out.actions, opponent_actions, seed, counter + 1));
            ok(t8b_policy_forward(policy, t8b_sim_learner_observations(sim), nullptr, t8b_sim_learner_mask_bits(sim), n,
                                  seed + 3, counter, 1, stream, tables, 0, &last));
            ok(t8b_rollout_record_outcome_device(rollout, step, t8b_sim_rewards(sim), t8b_sim_terminated(sim),
                                                 t8b_sim_truncated(sim), last.values, reward_scale, stream));
            ok(t8b_sim_reset_done(sim, seed, counter + 1));
        }
        if (opponent) check(cudaStreamSynchronize(side), "opponent stream");
        check(cudaStreamSynchronize(mask_stream), "mask stream");
    });
}
