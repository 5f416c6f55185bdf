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
// Every decision but the last steps and resets in one call (t8b_sim_step_and_reset): nothing
// reads the terminal observations there, while the last decision's bootstrap forward does.
#include "common.cuh"

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
        cudaStream_t side = nullptr;
        cudaEvent_t sim_ready = nullptr, opponent_done = nullptr;
        struct Cleanup {
            cudaStream_t* side;
            cudaEvent_t* a;
            cudaEvent_t* b;
            ~Cleanup() {
                if (*a) cudaEventDestroy(*a);
                if (*b) cudaEventDestroy(*b);
                if (*side) cudaStreamDestroy(*side);
            }
        } cleanup{&side, &sim_ready, &opponent_done};
        if (opponent) {
            check(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking), "opponent stream");
            check(cudaEventCreateWithFlags(&sim_ready, cudaEventDisableTiming), "event");
            check(cudaEventCreateWithFlags(&opponent_done, cudaEventDisableTiming), "event");
        }
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
            ok(t8b_policy_forward(policy, obs, nullptr, bits, n, seed + 1, counter, 0, stream, tables, 0, &out));
            if (step > 0) {
                ok(t8b_rollout_record_outcome_device(rollout, step - 1, t8b_sim_rewards(sim), t8b_sim_terminated(sim),
                                                     t8b_sim_truncated(sim), out.values, reward_scale, stream));
            }
            ok(t8b_rollout_record_policy_device(rollout, step, obs, nullptr, bits, out.actions, out.log_probabilities,
                                                out.values, stream, tables, out.entropies));
            if (opponent) check(cudaStreamWaitEvent(main, opponent_done, 0), "wait");
            if (step + 1 < horizon) {
                ok(t8b_sim_step_and_reset(sim, out.actions, opponent_actions, seed, counter + 1));
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
    });
}
