// Test infrastructure (not product code): C entry points over the reference's own
// GpuActorCritic and GpuRolloutBuffer (src/ppo.cu, compiled from the source where it lies by
// oracle/Makefile into _ref/libt8ppo_ref.so), so GPU tests can run the reference beside the
// library on the same inputs. Every entry point returns 0 on success or -1 with the exception
// text in t8pr_last_error().
#include "t8_v2/ppo.hpp"

#include <cstring>
#include <exception>
#include <string>
#include <vector>

using t8::v2::ActorCriticConfig;
using t8::v2::GpuActorCritic;
using t8::v2::GpuRolloutBuffer;
using t8::v2::GpuRolloutView;
using t8::v2::PpoUpdateConfig;
using t8::v2::PpoUpdateMetrics;

namespace {

thread_local std::string g_error;

template <typename Body>
int guard(Body&& body) {
    try {
        body();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
    } catch (...) {
        g_error = "unknown exception";
    }
    return -1;
}

}  // namespace

extern "C" {

// The ActorCriticConfig fields the harness sets (the rest keep the reference's defaults).
struct t8pr_config {
    int observation_size, action_count, hidden_size, action_feature_size, universal_action_count;
    int shared_layers, head_layers;
    int observation_normalization, orthogonal_initialization;
    float observation_clip, observation_epsilon;
    char matmul_precision[8];  // "fp32", "tf32" or "bf16"
};

// PpoUpdateConfig (include/t8_v2/ppo.hpp:60-73).
struct t8pr_ppo {
    int epochs;
    size_t minibatch_size;
    float learning_rate, clip_range, value_clip_range, target_kl, value_coefficient, entropy_coefficient;
    float max_gradient_norm, adam_beta1, adam_beta2, adam_epsilon;
};

const char* t8pr_last_error(void) { return g_error.c_str(); }

static ActorCriticConfig config_of(const t8pr_config* c) {
    ActorCriticConfig a;
    a.observation_size = c->observation_size;
    a.action_count = c->action_count;
    a.hidden_size = c->hidden_size;
    a.action_feature_size = c->action_feature_size;
    a.universal_action_count = c->universal_action_count;
    a.shared_layers = c->shared_layers;
    a.head_layers = c->head_layers;
    a.observation_normalization = c->observation_normalization != 0;
    a.orthogonal_initialization = c->orthogonal_initialization != 0;
    a.observation_clip = c->observation_clip;
    a.observation_epsilon = c->observation_epsilon;
    a.matmul_precision = std::string(c->matmul_precision, strnlen(c->matmul_precision, sizeof c->matmul_precision));
    return a;
}

int t8pr_policy_create(const t8pr_config* config, size_t capacity, uint64_t seed, void** out) {
    return guard([&] { *out = new GpuActorCritic(capacity, config_of(config), seed); });
}

void t8pr_policy_destroy(void* policy) { delete static_cast<GpuActorCritic*>(policy); }

size_t t8pr_policy_parameter_count(void* policy) { return static_cast<GpuActorCritic*>(policy)->parameter_count(); }

int t8pr_policy_set_features(void* policy, const float* host, size_t count, int tables) {
    return guard([&] { static_cast<GpuActorCritic*>(policy)->set_action_feature_tables({host, count}, tables); });
}

// forward: device inputs; out[0..4] = logits, actions, log-probabilities, values, entropies.
int t8pr_policy_forward(void* policy, const float* obs, const uint8_t* masks, size_t n, uint64_t seed, uint64_t step,
                        int deterministic, const int32_t* tables, const void** out) {
    return guard([&] {
        const auto view = static_cast<GpuActorCritic*>(policy)->forward(obs, masks, n, seed, step, deterministic != 0,
                                                                        nullptr, tables);
        static_cast<GpuActorCritic*>(policy)->synchronize();
        out[0] = view.logits;
        out[1] = view.actions;
        out[2] = view.log_probabilities;
        out[3] = view.values;
        out[4] = view.entropies;
    });
}

// update_ppo over a rollout given as device pointers in GpuRolloutView order; metrics[0..11]
// = the PpoUpdateMetrics fields in order (minibatches, epochs_completed, early_stopped last).
int t8pr_policy_update(void* policy, const void* const* ptrs, size_t environments, size_t horizon, size_t samples,
                       const t8pr_ppo* ppo, uint64_t shuffle_seed, double* metrics) {
    return guard([&] {
        GpuRolloutView v;
        v.observations = static_cast<const float*>(ptrs[0]);
        v.action_masks = static_cast<const uint8_t*>(ptrs[1]);
        v.actions = static_cast<const int64_t*>(ptrs[2]);
        v.old_log_probabilities = static_cast<const float*>(ptrs[3]);
        v.old_values = static_cast<const float*>(ptrs[4]);
        v.rewards = static_cast<const float*>(ptrs[5]);
        v.terminated = static_cast<const uint8_t*>(ptrs[6]);
        v.truncated = static_cast<const uint8_t*>(ptrs[7]);
        v.next_values = static_cast<const float*>(ptrs[8]);
        v.advantages = static_cast<const float*>(ptrs[9]);
        v.returns = static_cast<const float*>(ptrs[10]);
        v.feature_tables = static_cast<const int32_t*>(ptrs[11]);
        v.entropies = static_cast<const float*>(ptrs[12]);
        v.environment_count = environments;
        v.horizon = horizon;
        v.sample_count = samples;
        PpoUpdateConfig c;
        c.epochs = ppo->epochs;
        c.minibatch_size = ppo->minibatch_size;
        c.learning_rate = ppo->learning_rate;
        c.clip_range = ppo->clip_range;
        c.value_clip_range = ppo->value_clip_range;
        c.target_kl = ppo->target_kl;
        c.value_coefficient = ppo->value_coefficient;
        c.entropy_coefficient = ppo->entropy_coefficient;
        c.max_gradient_norm = ppo->max_gradient_norm;
        c.adam_beta1 = ppo->adam_beta1;
        c.adam_beta2 = ppo->adam_beta2;
        c.adam_epsilon = ppo->adam_epsilon;
        const PpoUpdateMetrics m = static_cast<GpuActorCritic*>(policy)->update_ppo(v, c, shuffle_seed);
        const double values[12] = {m.policy_loss, m.value_loss, m.entropy, m.approximate_kl, m.clip_fraction,
                                   m.gradient_norm, m.decision_fraction, m.decision_entropy,
                                   m.rollout_decision_entropy, static_cast<double>(m.minibatches),
                                   static_cast<double>(m.epochs_completed), m.early_stopped ? 1.0 : 0.0};
        std::memcpy(metrics, values, sizeof values);
    });
}

int t8pr_policy_save(void* policy, const char* path) {
    return guard([&] { static_cast<GpuActorCritic*>(policy)->save_checkpoint(path); });
}

int t8pr_policy_load(void* policy, const char* path, int load_optimizer_state) {
    return guard([&] { static_cast<GpuActorCritic*>(policy)->load_checkpoint(path, load_optimizer_state != 0); });
}

int t8pr_policy_observation_statistics(void* policy, float* mean_then_variance, uint64_t* count) {
    return guard([&] {
        const auto* p = static_cast<GpuActorCritic*>(policy);
        const auto stats = p->download_observation_statistics();
        std::memcpy(mean_then_variance, stats.data(), stats.size() * sizeof(float));
        *count = p->observation_count();
    });
}

int t8pr_rollout_create(size_t environments, size_t horizon, const t8pr_config* config, void** out) {
    return guard([&] { *out = new GpuRolloutBuffer(environments, horizon, config_of(config)); });
}

void t8pr_rollout_destroy(void* rollout) { delete static_cast<GpuRolloutBuffer*>(rollout); }

int t8pr_rollout_record_policy(void* rollout, size_t step, const float* obs, const uint8_t* masks,
                               const int64_t* actions, const float* log_probs, const float* values,
                               const int32_t* tables, const float* entropies) {
    return guard([&] {
        static_cast<GpuRolloutBuffer*>(rollout)->record_policy_device(step, obs, masks, actions, log_probs, values,
                                                                      nullptr, tables, entropies);
    });
}

int t8pr_rollout_record_outcome(void* rollout, size_t step, const float* rewards, const uint8_t* terminated,
                                const uint8_t* truncated, const float* next_values, float reward_scale) {
    return guard([&] {
        static_cast<GpuRolloutBuffer*>(rollout)->record_outcome_device(step, rewards, terminated, truncated,
                                                                       next_values, reward_scale);
    });
}

int t8pr_rollout_compute_gae(void* rollout, float gamma, float gae_lambda, int normalize) {
    return guard([&] { static_cast<GpuRolloutBuffer*>(rollout)->compute_gae(gamma, gae_lambda, normalize != 0); });
}

int t8pr_rollout_normalize_rewards(void* rollout, float gamma, float clip, float* std_out) {
    return guard([&] { *std_out = static_cast<GpuRolloutBuffer*>(rollout)->normalize_rewards(gamma, clip); });
}

// Host copies of advantages, returns and rewards ([horizon][environments] each).
int t8pr_rollout_download(void* rollout, float* advantages, float* returns, float* rewards) {
    return guard([&] {
        auto* r = static_cast<GpuRolloutBuffer*>(rollout);
        const auto a = r->download_advantages();
        const auto g = r->download_returns();
        const auto w = r->download_rewards();
        std::memcpy(advantages, a.data(), a.size() * sizeof(float));
        std::memcpy(returns, g.data(), g.size() * sizeof(float));
        std::memcpy(rewards, w.data(), w.size() * sizeof(float));
    });
}

// The rollout's device view in GpuRolloutView order (13 pointers, as t8pr_policy_update takes).
int t8pr_rollout_view(void* rollout, const void** ptrs) {
    return guard([&] {
        const GpuRolloutView v = static_cast<GpuRolloutBuffer*>(rollout)->device_view();
        const void* values[13] = {v.observations, v.action_masks, v.actions, v.old_log_probabilities, v.old_values,
                                  v.rewards, v.terminated, v.truncated, v.next_values, v.advantages, v.returns,
                                  v.feature_tables, v.entropies};
        std::memcpy(ptrs, values, sizeof values);
    });
}

}  // extern "C"
