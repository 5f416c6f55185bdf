// class GpuActorCritic (include/t8_v2/ppo.hpp:112-193), class GpuRolloutBuffer (ppo.hpp:223-291)
// and debug_ppo_objective_gradient (ppo.hpp:100-108) over the C ABI: the drop-in for the parts
// of src/ppo.cu these declarations cover. Each member calls the t8b_policy_* / t8b_rollout_*
// entry point include/t8b.h names beside it.
//
// Differences a caller can see, all documented in include/t8b.h: every matrix product runs
// bf16 x bf16 with fp32 accumulation whatever matmul_precision asks; separate policy/value
// heads (head_layers > 0), non-parametric heads and hidden sizes that are not a multiple of 128
// are refused with std::invalid_argument.
#include "t8_v2/ppo.hpp"

#include "shim.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <stdexcept>
#include <vector>

namespace t8::v2 {

using shim::copy_text;
using shim::ok;

namespace {

void check_cuda(cudaError_t error, const char* what) {
    if (error != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(error));
}

template <typename T>
std::vector<T> download(const T* device, std::size_t count, void* stream, const char* what) {
    std::vector<T> host(count);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (count != 0) {
        check_cuda(cudaMemcpyAsync(host.data(), device, sizeof(T) * count, cudaMemcpyDeviceToHost, st), what);
    }
    check_cuda(cudaStreamSynchronize(st), what);
    return host;
}

// A device buffer for the host-driven helpers below (released on scope exit).
template <typename T>
struct DeviceBuffer {
    T* pointer = nullptr;
    explicit DeviceBuffer(std::size_t count) {
        check_cuda(cudaMalloc(reinterpret_cast<void**>(&pointer), sizeof(T) * std::max<std::size_t>(count, 1)),
                   "allocate shim buffer");
    }
    ~DeviceBuffer() { cudaFree(pointer); }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    void upload(const T* host, std::size_t count) {
        check_cuda(cudaMemcpy(pointer, host, sizeof(T) * count, cudaMemcpyHostToDevice), "upload shim buffer");
    }
};

int precision_code(const std::string& precision) {
    if (precision == "fp32") return 0;
    if (precision == "tf32") return 1;
    if (precision == "bf16") return 2;
    throw std::invalid_argument("matmul precision must be fp32, tf32, or bf16");
}

t8b_actor_config_t actor_of(const ActorCriticConfig& c) {
    t8b_actor_config_t o{};
    o.observation_size = c.observation_size;
    o.action_count = c.action_count;
    o.hidden_size = c.hidden_size;
    o.action_feature_size = c.action_feature_size;
    o.universal_action_count = c.universal_action_count;
    o.shared_layers = c.shared_layers;
    o.head_layers = c.head_layers;
    o.observation_normalization = c.observation_normalization ? 1 : 0;
    o.orthogonal_initialization = c.orthogonal_initialization ? 1 : 0;
    o.observation_clip = c.observation_clip;
    o.observation_epsilon = c.observation_epsilon;
    o.matmul_precision = precision_code(c.matmul_precision);
    return o;
}

t8b_ppo_config_t ppo_of(const PpoUpdateConfig& c) {
    t8b_ppo_config_t o{};
    o.epochs = c.epochs;
    o.minibatch_size = c.minibatch_size;
    o.learning_rate = c.learning_rate;
    o.clip_range = c.clip_range;
    o.value_clip_range = c.value_clip_range;
    o.target_kl = c.target_kl;
    o.value_coefficient = c.value_coefficient;
    o.entropy_coefficient = c.entropy_coefficient;
    o.max_gradient_norm = c.max_gradient_norm;
    o.adam_beta1 = c.adam_beta1;
    o.adam_beta2 = c.adam_beta2;
    o.adam_epsilon = c.adam_epsilon;
    return o;
}

t8b_checkpoint_contract_t contract_of(const ActorCriticConfig& c) {
    t8b_checkpoint_contract_t o{};
    copy_text(o.catalog_sha256, c.catalog_sha256);
    copy_text(o.roster_version, c.roster_version);
    copy_text(o.observation_contract, c.observation_contract);
    copy_text(o.action_contract, c.action_contract);
    return o;
}

t8b_rollout_view_t rollout_of(const GpuRolloutView& v) {
    t8b_rollout_view_t o{};
    o.observations = v.observations;
    o.action_masks = v.action_masks;
    o.actions = v.actions;
    o.old_log_probabilities = v.old_log_probabilities;
    o.old_values = v.old_values;
    o.rewards = v.rewards;
    o.terminated = v.terminated;
    o.truncated = v.truncated;
    o.next_values = v.next_values;
    o.advantages = v.advantages;
    o.returns = v.returns;
    o.environment_count = v.environment_count;
    o.horizon = v.horizon;
    o.sample_count = v.sample_count;
    o.feature_tables = v.feature_tables;
    o.entropies = v.entropies;
    o.action_mask_bits = nullptr;  // the reference view carries uint8 masks
    return o;
}

}  // namespace

// debug_ppo_objective_gradient  ppo.hpp:100-108 -> t8b_ppo_output_gradient on one sample
std::vector<float> debug_ppo_objective_gradient(std::span<const float> logits_and_value,
                                                std::span<const std::uint8_t> action_mask, std::int64_t action,
                                                float old_log_probability, float old_value, float advantage,
                                                float return_value, const PpoUpdateConfig& config) {
    const bool any_legal = std::any_of(action_mask.begin(), action_mask.end(), [](std::uint8_t v) { return v != 0; });
    const bool valid_action = action >= 0 && static_cast<std::size_t>(action) < action_mask.size() &&
        ((any_legal && action_mask[static_cast<std::size_t>(action)] != 0) || (!any_legal && action == 0));
    if (logits_and_value.size() < 3 || action_mask.size() + 1 != logits_and_value.size() || !valid_action ||
        !std::all_of(logits_and_value.begin(), logits_and_value.end(), [](float v) { return std::isfinite(v); }) ||
        !std::isfinite(old_log_probability) || !std::isfinite(old_value) || !std::isfinite(advantage) ||
        !std::isfinite(return_value)) {
        throw std::invalid_argument("invalid PPO diagnostic objective input");
    }
    DeviceBuffer<float> outputs(logits_and_value.size()), gradients(logits_and_value.size());
    DeviceBuffer<std::uint8_t> mask(action_mask.size());
    DeviceBuffer<std::int64_t> selected(1);
    DeviceBuffer<float> scalars(4);
    outputs.upload(logits_and_value.data(), logits_and_value.size());
    mask.upload(action_mask.data(), action_mask.size());
    selected.upload(&action, 1);
    const float values[4] = {old_log_probability, old_value, advantage, return_value};
    scalars.upload(values, 4);
    const t8b_ppo_config_t c = ppo_of(config);
    ok(t8b_ppo_output_gradient(outputs.pointer, mask.pointer, selected.pointer, scalars.pointer, scalars.pointer + 1,
                               scalars.pointer + 2, scalars.pointer + 3, 1, static_cast<int>(action_mask.size()), &c,
                               gradients.pointer, nullptr, nullptr));
    return download(gradients.pointer, logits_and_value.size(), nullptr, "download PPO diagnostic gradient");
}

// ------------------------------------------------------------------ GpuActorCritic

struct GpuActorCritic::Impl {
    t8b_policy* policy = nullptr;
    ActorCriticConfig config;
    std::size_t capacity = 0;
    int tables = 0;
    t8b_policy_output_t last{};  // the last forward's outputs, for the download_* members

    ~Impl() {
        if (policy != nullptr) t8b_policy_destroy(policy);
    }
    // load_checkpoint adopts the file's normaliser setting; config() reports it
    void refresh_config() {
        t8b_actor_config_t c{};
        ok(t8b_policy_get_config(policy, &c));
        config.observation_normalization = c.observation_normalization != 0;
    }
};

// GpuActorCritic(capacity, config, initialization_seed)  ppo.hpp:114-117 -> t8b_policy_create
GpuActorCritic::GpuActorCritic(std::size_t capacity, ActorCriticConfig config, std::uint64_t initialization_seed)
    : impl_(std::make_unique<Impl>()) {
    const t8b_actor_config_t c = actor_of(config);
    ok(t8b_policy_create(capacity, &c, initialization_seed, &impl_->policy));
    impl_->config = std::move(config);
    impl_->capacity = capacity;
}

GpuActorCritic::~GpuActorCritic() = default;
GpuActorCritic::GpuActorCritic(GpuActorCritic&&) noexcept = default;
GpuActorCritic& GpuActorCritic::operator=(GpuActorCritic&&) noexcept = default;

std::size_t GpuActorCritic::capacity() const noexcept { return impl_->capacity; }  // ppo.hpp:125
std::size_t GpuActorCritic::parameter_count() const noexcept {                   // ppo.hpp:126
    return t8b_policy_parameter_count(impl_->policy);
}
const ActorCriticConfig& GpuActorCritic::config() const noexcept { return impl_->config; }  // ppo.hpp:127
int GpuActorCritic::action_feature_tables() const noexcept { return impl_->tables; }         // ppo.hpp:143

// set_action_features / set_action_feature_tables  ppo.hpp:132-137
void GpuActorCritic::set_action_features(std::span<const float> action_features, void* stream) {
    set_action_feature_tables(action_features, 1, stream);
}

void GpuActorCritic::set_action_feature_tables(std::span<const float> action_features, int tables, void* stream) {
    if (impl_->config.action_feature_size <= 0) {
        throw std::logic_error("action features require a parametric actor-critic config");
    }
    if (tables <= 0) throw std::invalid_argument("at least one action feature table is required");
    const std::size_t expected = static_cast<std::size_t>(tables) * impl_->config.action_count *
        static_cast<std::size_t>(impl_->config.action_feature_size);
    if (action_features.size() != expected) {
        throw std::invalid_argument("parametric action feature tensor has the wrong shape or non-finite values");
    }
    ok(t8b_policy_set_action_feature_tables(impl_->policy, action_features.data(), tables, stream));
    impl_->tables = tables;
}

// debug_backprop_relative_error  ppo.hpp:139-142: a random output gradient G backpropagated
// through the network for random inputs, three entries of every parameter tensor compared with
// central differences (step 1e-2) of sum(G * output); the largest relative error.
double GpuActorCritic::debug_backprop_relative_error(std::size_t batch, std::uint64_t seed) {
    auto& impl = *impl_;
    if (batch == 0 || batch > impl.capacity) throw std::invalid_argument("debug batch must fit the capacity");
    const std::size_t outputs = static_cast<std::size_t>(impl.config.action_feature_size) + 1;
    std::mt19937_64 random(seed);
    std::uniform_real_distribution<float> uniform(-1.0F, 1.0F);
    std::vector<float> inputs(batch * static_cast<std::size_t>(impl.config.observation_size));
    for (float& v : inputs) v = uniform(random);
    std::vector<float> weights(batch * outputs);
    for (float& v : weights) v = uniform(random);
    DeviceBuffer<float> d_inputs(inputs.size()), d_weights(weights.size()), d_outputs(weights.size());
    d_inputs.upload(inputs.data(), inputs.size());
    d_weights.upload(weights.data(), weights.size());
    ok(t8b_policy_debug_network(impl.policy, d_inputs.pointer, batch, d_weights.pointer, nullptr, nullptr));
    const std::size_t count = t8b_policy_parameter_count(impl.policy);
    std::vector<float> params(count), grads(count);
    ok(t8b_policy_get_parameters(impl.policy, params.data(), count));
    ok(t8b_policy_get_gradients(impl.policy, grads.data(), count));
    std::vector<float> out(weights.size());
    const auto objective = [&](std::vector<float>& p) {
        ok(t8b_policy_set_parameters(impl.policy, p.data(), count));
        ok(t8b_policy_debug_network(impl.policy, d_inputs.pointer, batch, nullptr, d_outputs.pointer, nullptr));
        check_cuda(cudaMemcpy(out.data(), d_outputs.pointer, sizeof(float) * out.size(), cudaMemcpyDeviceToHost),
                   "download debug output");
        double total = 0.0;
        for (std::size_t i = 0; i < out.size(); ++i) total += static_cast<double>(weights[i]) * out[i];
        return total;
    };
    // tensors in the canonical order w1, b1, ..., w_out, b_out
    std::vector<std::size_t> sizes;
    const std::size_t hidden = static_cast<std::size_t>(impl.config.hidden_size);
    for (int l = 0; l < impl.config.shared_layers; ++l) {
        sizes.push_back(hidden * (l == 0 ? static_cast<std::size_t>(impl.config.observation_size) : hidden));
        sizes.push_back(hidden);
    }
    sizes.push_back(outputs * hidden);
    sizes.push_back(outputs);
    double worst = 0.0;
    std::size_t offset = 0;
    for (const std::size_t size : sizes) {
        for (int sample = 0; sample < 3; ++sample) {
            const std::size_t index = offset + std::uniform_int_distribution<std::size_t>(0, size - 1)(random);
            constexpr float step = 1e-2F;
            const float original = params[index];
            params[index] = original + step;
            const double up = objective(params);
            params[index] = original - step;
            const double down = objective(params);
            params[index] = original;
            const double numeric = (up - down) / (2.0 * step);
            const double analytic = grads[index];
            worst = std::max(worst, std::abs(numeric - analytic) / std::max(1e-2, std::abs(numeric) + std::abs(analytic)));
        }
        offset += size;
    }
    ok(t8b_policy_set_parameters(impl.policy, params.data(), count));
    return worst;
}

// forward  ppo.hpp:146-154 -> t8b_policy_forward (the candidate scores are written too, as the
// reference's view carries them)
GpuPolicyOutputView GpuActorCritic::forward(const float* device_observations, const std::uint8_t* device_action_masks,
                                            std::size_t environment_count, std::uint64_t sampling_seed,
                                            std::uint64_t sampling_step, bool deterministic, void* stream,
                                            const std::int32_t* device_feature_tables) {
    t8b_policy_output_t out{};
    ok(t8b_policy_forward(impl_->policy, device_observations, device_action_masks, nullptr, environment_count,
                          sampling_seed, sampling_step, deterministic ? 1 : 0, stream, device_feature_tables, 1, &out));
    impl_->last = out;
    return {out.logits, out.actions, out.log_probabilities, out.values, out.entropies, out.environment_count};
}

// update_ppo  ppo.hpp:156-160 -> t8b_policy_update_ppo
PpoUpdateMetrics GpuActorCritic::update_ppo(const GpuRolloutView& rollout, const PpoUpdateConfig& update_config,
                                            std::uint64_t shuffle_seed, void* stream) {
    const t8b_rollout_view_t view = rollout_of(rollout);
    const t8b_ppo_config_t c = ppo_of(update_config);
    t8b_ppo_metrics_t m{};
    ok(t8b_policy_update_ppo(impl_->policy, &view, &c, shuffle_seed, stream, &m));
    PpoUpdateMetrics out;
    out.policy_loss = m.policy_loss;
    out.value_loss = m.value_loss;
    out.entropy = m.entropy;
    out.approximate_kl = m.approximate_kl;
    out.clip_fraction = m.clip_fraction;
    out.gradient_norm = m.gradient_norm;
    out.decision_fraction = m.decision_fraction;
    out.decision_entropy = m.decision_entropy;
    out.rollout_decision_entropy = m.rollout_decision_entropy;
    out.minibatches = m.minibatches;
    out.epochs_completed = m.epochs_completed;
    out.early_stopped = m.early_stopped != 0;
    return out;
}

// save_checkpoint / load_checkpoint  ppo.hpp:162-166 -> the .t8ppo format, byte for byte
void GpuActorCritic::save_checkpoint(const std::filesystem::path& path, void* stream) const {
    const t8b_checkpoint_contract_t c = contract_of(impl_->config);
    ok(t8b_policy_save_checkpoint(impl_->policy, path.string().c_str(), &c, stream));
}

void GpuActorCritic::load_checkpoint(const std::filesystem::path& path, bool load_optimizer_state, void* stream) {
    const t8b_checkpoint_contract_t c = contract_of(impl_->config);
    ok(t8b_policy_load_checkpoint(impl_->policy, path.string().c_str(), load_optimizer_state ? 1 : 0, &c, stream));
    impl_->refresh_config();
}

void GpuActorCritic::synchronize(void* stream) const { ok(t8b_policy_synchronize(impl_->policy, stream)); }

// observation_count / download_observation_statistics  ppo.hpp:174-177
std::uint64_t GpuActorCritic::observation_count() const noexcept {
    std::vector<float> mean(static_cast<std::size_t>(impl_->config.observation_size));
    std::vector<float> variance(mean.size());
    uint64_t count = 0;
    if (t8b_policy_get_observation_statistics(impl_->policy, mean.data(), variance.data(), &count) != T8B_OK) return 0;
    return count;
}

std::vector<float> GpuActorCritic::download_observation_statistics(void* stream) const {
    const std::size_t size = static_cast<std::size_t>(impl_->config.observation_size);
    std::vector<float> result(2 * size);
    uint64_t count = 0;
    ok(t8b_policy_synchronize(impl_->policy, stream));
    ok(t8b_policy_get_observation_statistics(impl_->policy, result.data(), result.data() + size, &count));
    return result;
}

// download_actions / values / log_probabilities / entropies  ppo.hpp:179-193 (the last forward's)
std::vector<std::int64_t> GpuActorCritic::download_actions(std::size_t count, void* stream) const {
    if (count > impl_->capacity) throw std::invalid_argument("download count exceeds capacity");
    if (impl_->last.actions == nullptr) return std::vector<std::int64_t>(count, 0);
    return download(impl_->last.actions, count, stream, "download actions");
}
std::vector<float> GpuActorCritic::download_values(std::size_t count, void* stream) const {
    if (count > impl_->capacity) throw std::invalid_argument("download count exceeds capacity");
    if (impl_->last.values == nullptr) return std::vector<float>(count, 0.0F);
    return download(impl_->last.values, count, stream, "download values");
}
std::vector<float> GpuActorCritic::download_log_probabilities(std::size_t count, void* stream) const {
    if (count > impl_->capacity) throw std::invalid_argument("download count exceeds capacity");
    if (impl_->last.log_probabilities == nullptr) return std::vector<float>(count, 0.0F);
    return download(impl_->last.log_probabilities, count, stream, "download log probabilities");
}
std::vector<float> GpuActorCritic::download_entropies(std::size_t count, void* stream) const {
    if (count > impl_->capacity) throw std::invalid_argument("download count exceeds capacity");
    if (impl_->last.entropies == nullptr) return std::vector<float>(count, 0.0F);
    return download(impl_->last.entropies, count, stream, "download entropies");
}

// ------------------------------------------------------------------ GpuRolloutBuffer

struct GpuRolloutBuffer::Impl {
    t8b_rollout* rollout = nullptr;
    std::size_t environments = 0, horizon = 0;
    ~Impl() {
        if (rollout != nullptr) t8b_rollout_destroy(rollout);
    }
    t8b_rollout_view_t view() const {
        t8b_rollout_view_t v{};
        ok(t8b_rollout_packed_view(rollout, &v));
        return v;
    }
};

// GpuRolloutBuffer(environment_count, horizon, config)  ppo.hpp:225-228 -> t8b_rollout_create
GpuRolloutBuffer::GpuRolloutBuffer(std::size_t environment_count, std::size_t horizon, ActorCriticConfig config)
    : impl_(std::make_unique<Impl>()) {
    const t8b_actor_config_t c = actor_of(config);
    ok(t8b_rollout_create(environment_count, horizon, &c, &impl_->rollout));
    impl_->environments = environment_count;
    impl_->horizon = horizon;
}

GpuRolloutBuffer::~GpuRolloutBuffer() = default;
GpuRolloutBuffer::GpuRolloutBuffer(GpuRolloutBuffer&&) noexcept = default;
GpuRolloutBuffer& GpuRolloutBuffer::operator=(GpuRolloutBuffer&&) noexcept = default;

std::size_t GpuRolloutBuffer::environment_count() const noexcept { return impl_->environments; }  // ppo.hpp:236
std::size_t GpuRolloutBuffer::horizon() const noexcept { return impl_->horizon; }                   // ppo.hpp:237
std::size_t GpuRolloutBuffer::sample_count() const noexcept {                                       // ppo.hpp:238
    return impl_->environments * impl_->horizon;
}

// device_view  ppo.hpp:239 -> t8b_rollout_device_view (uint8 masks expanded from the packed ones)
GpuRolloutView GpuRolloutBuffer::device_view() const noexcept {
    t8b_rollout_view_t v{};
    if (t8b_rollout_device_view(impl_->rollout, &v) != T8B_OK) return {};
    GpuRolloutView o;
    o.observations = v.observations;
    o.action_masks = v.action_masks;
    o.actions = v.actions;
    o.old_log_probabilities = v.old_log_probabilities;
    o.old_values = v.old_values;
    o.rewards = v.rewards;
    o.terminated = v.terminated;
    o.truncated = v.truncated;
    o.next_values = v.next_values;
    o.advantages = v.advantages;
    o.returns = v.returns;
    o.environment_count = v.environment_count;
    o.horizon = v.horizon;
    o.sample_count = v.sample_count;
    o.feature_tables = v.feature_tables;
    o.entropies = v.entropies;
    return o;
}

// record_policy_device  ppo.hpp:241-250
void GpuRolloutBuffer::record_policy_device(std::size_t step, const float* observations, const std::uint8_t* action_masks,
                                            const std::int64_t* actions, const float* log_probabilities,
                                            const float* values, void* stream, const std::int32_t* feature_tables,
                                            const float* entropies) {
    if (action_masks == nullptr) throw std::invalid_argument("rollout device pointers cannot be null");
    ok(t8b_rollout_record_policy_device(impl_->rollout, step, observations, action_masks, nullptr, actions,
                                        log_probabilities, values, stream, feature_tables, entropies));
}

// record_outcome_device  ppo.hpp:252-259
void GpuRolloutBuffer::record_outcome_device(std::size_t step, const float* rewards, const std::uint8_t* terminated,
                                             const std::uint8_t* truncated, const float* next_values, float reward_scale,
                                             void* stream) {
    ok(t8b_rollout_record_outcome_device(impl_->rollout, step, rewards, terminated, truncated, next_values, reward_scale,
                                         stream));
}

// compute_gae  ppo.hpp:261-265
void GpuRolloutBuffer::compute_gae(float gamma, float gae_lambda, bool normalize_advantages, void* stream) {
    ok(t8b_rollout_compute_gae(impl_->rollout, gamma, gae_lambda, normalize_advantages ? 1 : 0, stream));
}

// normalize_rewards  ppo.hpp:271
float GpuRolloutBuffer::normalize_rewards(float gamma, float clip, void* stream) {
    float used = 0.0F;
    ok(t8b_rollout_normalize_rewards(impl_->rollout, gamma, clip, stream, &used));
    return used;
}

// mean_reward  ppo.hpp:274
double GpuRolloutBuffer::mean_reward(void* stream) {
    double mean = 0.0;
    ok(t8b_rollout_mean_reward(impl_->rollout, stream, &mean));
    return mean;
}

// return_normalizer_state / restore_return_normalizer_state  ppo.hpp:275-276
ReturnNormalizerState GpuRolloutBuffer::return_normalizer_state(void* stream) const {
    ReturnNormalizerState state;
    state.discounted_returns.resize(impl_->environments);
    ok(t8b_rollout_synchronize(impl_->rollout, stream));
    ok(t8b_rollout_return_normalizer_state(impl_->rollout, &state.count, &state.mean, &state.variance,
                                           state.discounted_returns.data()));
    return state;
}

void GpuRolloutBuffer::restore_return_normalizer_state(const ReturnNormalizerState& state, void* stream) {
    if (state.discounted_returns.size() != impl_->environments) {
        throw std::invalid_argument("return normalizer state is invalid for this rollout buffer");
    }
    ok(t8b_rollout_synchronize(impl_->rollout, stream));
    ok(t8b_rollout_restore_return_normalizer_state(impl_->rollout, state.count, state.mean, state.variance,
                                                   state.discounted_returns.data()));
}

void GpuRolloutBuffer::synchronize(void* stream) const { ok(t8b_rollout_synchronize(impl_->rollout, stream)); }

// download_*  ppo.hpp:279-285: [step][environment] host copies
std::vector<float> GpuRolloutBuffer::download_advantages(void* stream) const {
    return download(impl_->view().advantages, sample_count(), stream, "download advantages");
}
std::vector<float> GpuRolloutBuffer::download_returns(void* stream) const {
    return download(impl_->view().returns, sample_count(), stream, "download returns");
}
std::vector<float> GpuRolloutBuffer::download_rewards(void* stream) const {
    return download(impl_->view().rewards, sample_count(), stream, "download rewards");
}
std::vector<float> GpuRolloutBuffer::download_values(void* stream) const {
    return download(impl_->view().old_values, sample_count(), stream, "download values");
}
std::vector<std::uint8_t> GpuRolloutBuffer::download_terminated(void* stream) const {
    return download(impl_->view().terminated, sample_count(), stream, "download terminated");
}
std::vector<std::uint8_t> GpuRolloutBuffer::download_truncated(void* stream) const {
    return download(impl_->view().truncated, sample_count(), stream, "download truncated");
}
std::vector<float> GpuRolloutBuffer::download_next_values(void* stream) const {
    return download(impl_->view().next_values, sample_count(), stream, "download next values");
}

}  // namespace t8::v2
