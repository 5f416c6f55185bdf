// class GpuFullMoveSimulator (include/t8_v2/full_move_gpu.hpp:42-141) over the C ABI: the
// drop-in for src/full_move_gpu.cu. Every member maps to the t8b_sim_* entry point include/t8b.h
// names beside it; the roster's tables and states cross as the t8b.h structs, field for field.
// Argument checks that the reference makes on the host (sizes and index ranges) are made here
// with the same exception types before the library is called.
#include "t8_v2/full_move_gpu.hpp"

#include "shim.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <iterator>
#include <stdexcept>
#include <vector>

namespace t8::v2 {

using shim::ok;
namespace fc = full_core;

namespace {

void check_cuda(cudaError_t error, const char* what) {
    if (error != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(error));
}

template <typename T>
std::vector<T> download(const T* device, std::size_t count, const char* what) {
    std::vector<T> host(count);
    if (count != 0) check_cuda(cudaMemcpy(host.data(), device, sizeof(T) * count, cudaMemcpyDeviceToHost), what);
    return host;
}

t8b_window_t window_of(const fc::Window& w) {
    t8b_window_t out{};
    out.count = w.count;
    for (int i = 0; i < fc::kMaxWindowSpans; ++i) {
        out.first[i] = w.first[i];
        out.last[i] = w.last[i];
    }
    return out;
}

t8b_move_t move_of(const fc::Move& m) {
    t8b_move_t o{};
    o.flags = m.flags;
    o.hit_offset = m.hit_offset;
    o.hit_count = m.hit_count;
    o.total_frames = m.total_frames;
    o.recovery = m.recovery;
    o.block_advantage = m.block_advantage;
    o.hit_advantage = m.hit_advantage;
    o.counter_hit_advantage = m.counter_hit_advantage;
    o.launch_air_frames = m.launch_air_frames;
    o.back_turned_hit_advantage = m.back_turned_hit_advantage;
    o.heat_dash_block_advantage = m.heat_dash_block_advantage;
    o.heat_dash_hit_advantage = m.heat_dash_hit_advantage;
    o.heat_cost_frames = m.heat_cost_frames;
    o.required_stance = m.required_stance;
    o.result_stance = m.result_stance;
    o.result_stance_on_hit = m.result_stance_on_hit;
    o.result_stance_on_block = m.result_stance_on_block;
    std::copy(m.parry_outcomes, m.parry_outcomes + 4, o.parry_outcomes);
    o.heat_parry_outcome = m.heat_parry_outcome;
    o.hit_effect = static_cast<uint8_t>(m.hit_effect);
    o.counter_hit_effect = static_cast<uint8_t>(m.counter_hit_effect);
    o.back_turned_hit_effect = static_cast<uint8_t>(m.back_turned_hit_effect);
    o.heat_dash_hit_effect = static_cast<uint8_t>(m.heat_dash_hit_effect);
    o.required_posture = static_cast<uint8_t>(m.required_posture);
    o.attack_throw = static_cast<uint8_t>(m.attack_throw);
    o.parry_levels = m.parry_levels;
    o.heat_parry_levels = m.heat_parry_levels;
    o.travel = m.travel;
    o.pushback_hit = m.pushback_hit;
    o.pushback_block = m.pushback_block;
    o.reversal_damage = m.reversal_damage;
    o.attack_throw_damage = m.attack_throw_damage;
    o.recoverable_damage = m.recoverable_damage;
    o.rage_art_max_damage = m.rage_art_max_damage;
    o.self_damage = m.self_damage;
    o.self_recoverable = m.self_recoverable;
    o.restore_health_hit = m.restore_health_hit;
    o.restore_recoverable_hit = m.restore_recoverable_hit;
    o.restore_recoverable_block = m.restore_recoverable_block;
    o.resource_gain_start = m.resource_gain_start;
    o.resource_gain_hit = m.resource_gain_hit;
    o.resource_gain_airborne_hit = m.resource_gain_airborne_hit;
    o.resource_gain_block = m.resource_gain_block;
    o.resource_gain_heat_activation = m.resource_gain_heat_activation;
    o.install_damage_bonus = m.install_damage_bonus;
    o.install_chip_damage = m.install_chip_damage;
    o.install_reach = m.install_reach;
    const fc::Window* windows[9] = {&m.high_crush, &m.low_crush, &m.power_crush, &m.armor,     &m.parry,
                                    &m.reversal,   &m.invincible, &m.airborne,   &m.heat_parry};
    for (int i = 0; i < 9; ++i) o.windows[i] = window_of(*windows[i]);
    return o;
}

t8b_hit_t hit_of(const fc::Hit& h) {
    t8b_hit_t o{};
    o.level = static_cast<uint8_t>(h.level);
    o.throw_break = static_cast<uint8_t>(h.throw_break);
    o.flags = h.flags;
    o.first_active_frame = h.first_active_frame;
    o.active_frames = h.active_frames;
    o.damage = h.damage;
    o.reach = h.reach;
    o.tracking_left = h.tracking_left;
    o.tracking_right = h.tracking_right;
    o.chip_damage = h.chip_damage;
    o.heat_chip_damage = h.heat_chip_damage;
    return o;
}

t8b_stance_t stance_of(const fc::Stance& s) {
    t8b_stance_t o{};
    o.can_guard = s.can_guard ? 1 : 0;
    o.has_max_frames = s.has_max_frames ? 1 : 0;
    o.auto_parry = s.auto_parry;
    o.max_frames = s.max_frames;
    std::copy(s.parry_outcomes, s.parry_outcomes + 4, o.parry_outcomes);
    o.pulse_interval_frames = s.pulse_interval_frames;
    o.pulse_recoverable = s.pulse_recoverable;
    o.pulse_resource = s.pulse_resource;
    return o;
}

t8b_rules_t rules_of(const fc::Rules& r) {
    t8b_rules_t o{};
    o.resource_max = r.resource_max;
    o.install_threshold = r.install_threshold;
    o.has_install_threshold = r.has_install_threshold ? 1 : 0;
    o.resource_persists = r.resource_persists ? 1 : 0;
    o.install_consumes = r.install_consumes ? 1 : 0;
    return o;
}

t8b_engine_config_t engine_of(const FullEngineConfig& c) {
    t8b_engine_config_t o{};
    o.half_width = c.half_width;
    o.body_radius = c.body_radius;
    o.walk_speed = c.walk_speed;
    o.dash_distance = c.dash_distance;
    o.dash_frames = c.dash_frames;
    o.backdash_frames = c.backdash_frames;
    o.backdash_distance = c.backdash_distance;
    o.sidestep_distance = c.sidestep_distance;
    o.sidestep_frames = c.sidestep_frames;
    o.launch_air_frames = c.launch_air_frames;
    o.axis_realign_per_frame = c.axis_realign_per_frame;
    o.juggle_window_frames = c.juggle_window_frames;
    o.juggle_window_decay = c.juggle_window_decay;
    o.tornado_extra_frames = c.tornado_extra_frames;
    o.knockdown_frames = c.knockdown_frames;
    o.wakeup_stand_frames = c.wakeup_stand_frames;
    o.wakeup_roll_frames = c.wakeup_roll_frames;
    o.wakeup_roll_distance = c.wakeup_roll_distance;
    o.tech_window_frames = c.tech_window_frames;
    o.tech_roll_frames = c.tech_roll_frames;
    o.wall_splat_frames = c.wall_splat_frames;
    o.crumple_frames = c.crumple_frames;
    o.stage_break_air_frames = c.stage_break_air_frames;
    o.wall_break_extension = c.wall_break_extension;
    o.combo_scale_step = c.combo_scale_step;
    o.combo_scale_floor = c.combo_scale_floor;
    o.counter_hit_damage_scale = c.counter_hit_damage_scale;
    o.throw_break_window = c.throw_break_window;
    o.throw_break_recovery = c.throw_break_recovery;
    o.parry_outcome_frames = c.parry_outcome_frames;
    o.side_exposure_ratio = c.side_exposure_ratio;
    o.back_to_wall_distance = c.back_to_wall_distance;
    o.ki_charge_frames = c.ki_charge_frames;
    o.ki_charge_damage_scale = c.ki_charge_damage_scale;
    o.parry_stun_frames = c.parry_stun_frames;
    o.reversal_recovery = c.reversal_recovery;
    o.heat_duration_frames = c.heat_duration_frames;
    o.heat_dash_frames = c.heat_dash_frames;
    o.heat_dash_distance = c.heat_dash_distance;
    o.rage_health_fraction = c.rage_health_fraction;
    o.rage_damage_scale = c.rage_damage_scale;
    o.wall_combo_scale = c.wall_combo_scale;
    o.recoverable_regain_hit = c.recoverable_regain_hit;
    o.recoverable_regain_block = c.recoverable_regain_block;
    o.max_health = c.max_health;
    return o;
}

t8b_env_config_t env_of(const fc::EnvConfig& c) {
    t8b_env_config_t o{};
    o.max_round_frames = c.max_round_frames;
    o.hold_frames = c.hold_frames;
    o.max_frames_per_decision = c.max_frames_per_decision;
    o.damage_reward = c.damage_reward;
    o.win_reward = c.win_reward;
    o.draw_penalty = c.draw_penalty;
    o.throw_break_penalty = c.throw_break_penalty;
    o.time_penalty_per_second = c.time_penalty_per_second;
    o.damage_dealt_weight = c.damage_dealt_weight;
    o.damage_taken_weight = c.damage_taken_weight;
    o.distance_penalty_per_second = c.distance_penalty_per_second;
    o.perception_delay = c.perception_delay;
    o.memory = c.memory ? 1 : 0;
    o.live_noise = c.live_noise ? 1 : 0;
    o.screen_view = c.screen_view ? 1 : 0;
    o.noise_position_max = c.noise_position_max;
    o.noise_flip_max = c.noise_flip_max;
    o.latency_min = c.latency_min;
    o.latency_max = c.latency_max;
    o.start_center_range = c.start_center_range;
    o.start_distance_min = c.start_distance_min;
    o.start_distance_max = c.start_distance_max;
    return o;
}

// A fighter's bools, in the bit order of t8b_fighter_t::flags (T8B_F_HEAT ... T8B_F_CRUMPLED).
constexpr bool fc::Fighter::*kFighterBits[] = {
    &fc::Fighter::heat,            &fc::Fighter::heat_available,        &fc::Fighter::rage,
    &fc::Fighter::rage_available,  &fc::Fighter::throw_break_attempted, &fc::Fighter::installed,
    &fc::Fighter::move_hit,        &fc::Fighter::move_blocked,          &fc::Fighter::resource_gained,
    &fc::Fighter::back_turned,     &fc::Fighter::move_in_heat,          &fc::Fighter::ki_charge_boost,
    &fc::Fighter::move_boosted,    &fc::Fighter::in_blockstun,          &fc::Fighter::tornado_used,
    &fc::Fighter::wall_splat_used, &fc::Fighter::wall_scaled,           &fc::Fighter::techable,
    &fc::Fighter::crumpled,
};
// The stage's bools, in the bit order of t8b_state_t::stage_flags (T8B_S_*).
constexpr bool FullEngineStage::*kStageBits[] = {
    &FullEngineStage::left_wall_breakable, &FullEngineStage::right_wall_breakable, &FullEngineStage::left_balcony,
    &FullEngineStage::right_balcony,       &FullEngineStage::floor_breakable,
};

t8b_state_t state_of(const fc::State& s) {
    t8b_state_t o{};
    for (int p = 0; p < 2; ++p) {
        const fc::Fighter& f = s.fighters[p];
        t8b_fighter_t& g = o.fighters[p];
        g.health = f.health;
        g.recoverable_health = f.recoverable_health;
        g.x = f.x;
        g.axis = f.axis;
        g.resource = f.resource;
        g.posture = static_cast<uint8_t>(f.posture);
        g.universal = static_cast<uint8_t>(f.universal);
        g.heat_dash_from = f.heat_dash_from;
        for (std::size_t b = 0; b < std::size(kFighterBits); ++b) g.flags |= (f.*kFighterBits[b]) ? (1u << b) : 0u;
        g.stance = f.stance;
        g.heat_frames = f.heat_frames;
        g.throw_break_frames = f.throw_break_frames;
        g.pending_throw_hit = f.pending_throw_hit;
        g.pending_throw_elapsed = f.pending_throw_elapsed;
        g.move = f.move;
        g.action_frame = f.action_frame;
        g.hits_landed = f.hits_landed;
        g.stance_frames = f.stance_frames;
        g.ki_charge_frames = f.ki_charge_frames;
        g.stun = f.stun;
        g.posture_frames = f.posture_frames;
        g.grounded_elapsed = f.grounded_elapsed;
        g.combo_hits = f.combo_hits;
    }
    o.left_wall = s.stage.left_wall;
    o.right_wall = s.stage.right_wall;
    for (std::size_t b = 0; b < std::size(kStageBits); ++b) o.stage_flags |= (s.stage.*kStageBits[b]) ? (1u << b) : 0u;
    o.stage_level = s.stage.level;
    o.frame = s.frame;
    o.winner = s.winner;
    return o;
}

fc::State state_from(const t8b_state_t& o) {
    fc::State s{};
    for (int p = 0; p < 2; ++p) {
        fc::Fighter& f = s.fighters[p];
        const t8b_fighter_t& g = o.fighters[p];
        f.health = g.health;
        f.recoverable_health = g.recoverable_health;
        f.x = g.x;
        f.axis = g.axis;
        f.resource = g.resource;
        f.posture = static_cast<FullPosture>(g.posture);
        f.universal = static_cast<FullUniversal>(g.universal);
        f.heat_dash_from = g.heat_dash_from;
        for (std::size_t b = 0; b < std::size(kFighterBits); ++b) f.*kFighterBits[b] = ((g.flags >> b) & 1u) != 0;
        f.stance = g.stance;
        f.heat_frames = g.heat_frames;
        f.throw_break_frames = g.throw_break_frames;
        f.pending_throw_hit = g.pending_throw_hit;
        f.pending_throw_elapsed = g.pending_throw_elapsed;
        f.move = g.move;
        f.action_frame = g.action_frame;
        f.hits_landed = g.hits_landed;
        f.stance_frames = g.stance_frames;
        f.ki_charge_frames = g.ki_charge_frames;
        f.stun = g.stun;
        f.posture_frames = g.posture_frames;
        f.grounded_elapsed = g.grounded_elapsed;
        f.combo_hits = g.combo_hits;
    }
    s.stage.left_wall = o.left_wall;
    s.stage.right_wall = o.right_wall;
    for (std::size_t b = 0; b < std::size(kStageBits); ++b) s.stage.*kStageBits[b] = ((o.stage_flags >> b) & 1u) != 0;
    s.stage.level = o.stage_level;
    s.frame = o.frame;
    s.winner = o.winner;
    return s;
}

fc::Events events_from(const t8b_events_t& o) {
    fc::Events e{};
    e.contact_count = std::min(o.contact_count, fc::kMaxContacts);
    for (int i = 0; i < e.contact_count; ++i) {
        e.contacts[i] = {o.contacts[i].attacker, o.contacts[i].hit_index, static_cast<FullContact>(o.contacts[i].contact),
                         o.contacts[i].damage};
    }
    e.transition_count = std::min(o.transition_count, fc::kMaxTransitions);
    for (int i = 0; i < e.transition_count; ++i) e.transitions[i] = static_cast<FullTransition>(o.transitions[i]);
    for (int p = 0; p < 2; ++p) {
        e.heat_activated[p] = o.heat_activated[p] != 0;
        e.rage_activated[p] = o.rage_activated[p] != 0;
    }
    return e;
}

}  // namespace

struct GpuFullMoveSimulator::Impl {
    std::vector<FullMoveCharacter> roster;
    fc::EnvConfig config{};
    t8b_sim* sim = nullptr;
    std::size_t environments = 0;
    int observation_size = 0;
    // the tallies download_and_clear_tally reads with the main one (full_move_gpu.hpp:124-131)
    std::vector<std::uint32_t> scenario_tally, learner_tally, bot_tally;

    ~Impl() {
        if (sim != nullptr) t8b_sim_destroy(sim);
    }
    void sized(std::size_t got, std::size_t want, const char* what) const {
        if (got != want) throw std::invalid_argument(what);
    }
    void character_range(std::span<const int> characters, int lowest, const char* what) const {
        for (const int c : characters) {
            if (c < lowest || c >= static_cast<int>(roster.size())) throw std::out_of_range(what);
        }
    }
};

// GpuFullMoveSimulator(roster, environments, config)  full_move_gpu.hpp:44-45 -> t8b_sim_create
GpuFullMoveSimulator::GpuFullMoveSimulator(std::vector<FullMoveCharacter> roster, std::size_t environments,
                                           fc::EnvConfig config)
    : impl_(std::make_unique<Impl>()) {
    if (roster.empty() || environments == 0) throw std::invalid_argument("full-move simulator needs characters and environments");
    auto& impl = *impl_;
    impl.roster = std::move(roster);
    impl.config = config;
    impl.environments = environments;
    const FullEngineConfig& engine = impl.roster.front().tables.config;
    std::vector<std::vector<t8b_move_t>> moves(impl.roster.size());
    std::vector<std::vector<t8b_hit_t>> hits(impl.roster.size());
    std::vector<std::vector<t8b_stance_t>> stances(impl.roster.size());
    std::vector<t8b_character_t> characters(impl.roster.size());
    for (std::size_t c = 0; c < impl.roster.size(); ++c) {
        const FullMoveCharacter& ch = impl.roster[c];
        if (std::memcmp(&ch.tables.config, &engine, sizeof(FullEngineConfig)) != 0) {
            throw std::invalid_argument("every roster character must share one engine configuration");
        }
        for (const auto& m : ch.tables.moves[0]) moves[c].push_back(move_of(m));
        for (const auto& h : ch.tables.hits[0]) hits[c].push_back(hit_of(h));
        for (const auto& s : ch.tables.stances[0]) stances[c].push_back(stance_of(s));
        t8b_character_t& out = characters[c];
        out.moves = moves[c].data();
        out.hits = hits[c].data();
        out.stances = stances[c].data();
        out.candidate_moves = ch.candidate_moves.data();
        out.candidate_features = ch.candidate_features.data();
        out.move_count = static_cast<int32_t>(moves[c].size());
        out.hit_count = static_cast<int32_t>(hits[c].size());
        out.stance_count = static_cast<int32_t>(stances[c].size());
        out.candidate_count = ch.candidate_count();
        out.roster_id = ch.roster_id;
        out.rules = rules_of(ch.tables.rules[0]);
    }
    const t8b_engine_config_t engine_c = engine_of(engine);
    const t8b_env_config_t env_c = env_of(config);
    ok(t8b_sim_create(characters.data(), static_cast<int>(characters.size()), &engine_c, environments, &env_c, &impl.sim));
    impl.observation_size = t8b_sim_observation_size(impl.sim);
}

GpuFullMoveSimulator::~GpuFullMoveSimulator() = default;
GpuFullMoveSimulator::GpuFullMoveSimulator(GpuFullMoveSimulator&&) noexcept = default;
GpuFullMoveSimulator& GpuFullMoveSimulator::operator=(GpuFullMoveSimulator&&) noexcept = default;

std::size_t GpuFullMoveSimulator::environment_count() const noexcept { return impl_->environments; }
const std::vector<FullMoveCharacter>& GpuFullMoveSimulator::roster() const noexcept { return impl_->roster; }
const fc::EnvConfig& GpuFullMoveSimulator::config() const noexcept { return impl_->config; }
int GpuFullMoveSimulator::observation_size() const noexcept { return impl_->observation_size; }

// set_matchups  full_move_gpu.hpp:61 -> t8b_sim_set_matchups
void GpuFullMoveSimulator::set_matchups(std::span<const int> p1_characters, std::span<const int> p2_characters) {
    auto& impl = *impl_;
    if (p1_characters.size() != impl.environments || p2_characters.size() != impl.environments) {
        throw std::invalid_argument("one matchup per environment is required");
    }
    impl.character_range(p1_characters, 0, "P1 character");
    impl.character_range(p2_characters, 0, "P2 character");
    ok(t8b_sim_set_matchups(impl.sim, p1_characters.data(), p2_characters.data()));
}

// reset_engine / step_engine / download_states / download_events / upload_states /
// download_legal_mask  full_move_gpu.hpp:64-74
void GpuFullMoveSimulator::reset_engine(std::span<const double> p1_x, std::span<const double> p2_x) {
    impl_->sized(p1_x.size(), impl_->environments, "one P1 position per environment is required");
    impl_->sized(p2_x.size(), impl_->environments, "one P2 position per environment is required");
    ok(t8b_sim_reset_engine(impl_->sim, p1_x.data(), p2_x.data()));
}

void GpuFullMoveSimulator::step_engine(std::span<const fc::Input> inputs, std::span<const std::uint8_t> new_round,
                                       std::span<const double> p1_x, std::span<const double> p2_x) {
    auto& impl = *impl_;
    impl.sized(inputs.size(), 2 * impl.environments, "two inputs per environment are required");
    std::vector<t8b_input_t> converted(inputs.size());
    for (std::size_t i = 0; i < inputs.size(); ++i) {
        converted[i] = {inputs[i].move, static_cast<int32_t>(inputs[i].universal)};
    }
    const bool rounds = !new_round.empty();
    if (rounds) {
        impl.sized(new_round.size(), impl.environments, "one new-round flag per environment is required");
        impl.sized(p1_x.size(), impl.environments, "one P1 position per environment is required");
        impl.sized(p2_x.size(), impl.environments, "one P2 position per environment is required");
    }
    ok(t8b_sim_step_engine(impl.sim, converted.data(), rounds ? new_round.data() : nullptr,
                           rounds ? p1_x.data() : nullptr, rounds ? p2_x.data() : nullptr));
}

std::vector<fc::State> GpuFullMoveSimulator::download_states() const {
    std::vector<t8b_state_t> packed(impl_->environments);
    ok(t8b_sim_download_states(impl_->sim, packed.data()));
    std::vector<fc::State> states(packed.size());
    std::transform(packed.begin(), packed.end(), states.begin(), state_from);
    return states;
}

std::vector<fc::Events> GpuFullMoveSimulator::download_events() const {
    std::vector<t8b_events_t> packed(impl_->environments);
    ok(t8b_sim_download_events(impl_->sim, packed.data()));
    std::vector<fc::Events> events(packed.size());
    std::transform(packed.begin(), packed.end(), events.begin(), events_from);
    return events;
}

void GpuFullMoveSimulator::upload_states(std::span<const fc::State> states) {
    impl_->sized(states.size(), impl_->environments, "one state per environment is required");
    std::vector<t8b_state_t> packed(states.size());
    std::transform(states.begin(), states.end(), packed.begin(), state_of);
    ok(t8b_sim_upload_states(impl_->sim, packed.data()));
}

std::vector<std::uint8_t> GpuFullMoveSimulator::download_legal_mask(int player) const {
    if (player != 0 && player != 1) throw std::out_of_range("player must be 0 or 1");
    std::vector<std::uint8_t> mask(impl_->environments * static_cast<std::size_t>(kFullMoveMaxCandidates));
    ok(t8b_sim_download_legal_mask(impl_->sim, player, mask.data()));
    return mask;
}

// set_learner_sides / set_pending_opponents / set_pending_learners  full_move_gpu.hpp:79-86
void GpuFullMoveSimulator::set_learner_sides(std::span<const std::uint8_t> learner_is_p1) {
    impl_->sized(learner_is_p1.size(), impl_->environments, "one learner side per environment is required");
    ok(t8b_sim_set_learner_sides(impl_->sim, learner_is_p1.data()));
}

void GpuFullMoveSimulator::set_pending_opponents(std::span<const int> characters, std::span<const float> aggression,
                                                 std::span<const int> scenarios) {
    auto& impl = *impl_;
    impl.sized(characters.size(), impl.environments, "one opponent per environment is required");
    impl.character_range(characters, 0, "opponent");
    if (!aggression.empty()) impl.sized(aggression.size(), impl.environments, "one aggression per environment is required");
    if (!scenarios.empty()) {
        impl.sized(scenarios.size(), impl.environments, "one scenario per environment is required");
        for (const int scenario : scenarios) {
            if (scenario < 0 || scenario >= T8B_SCENARIOS) throw std::out_of_range("scenario");
        }
    }
    ok(t8b_sim_set_pending_opponents(impl.sim, characters.data(), aggression.empty() ? nullptr : aggression.data(),
                                     scenarios.empty() ? nullptr : scenarios.data()));
}

void GpuFullMoveSimulator::set_pending_learners(std::span<const int> characters) {
    auto& impl = *impl_;
    impl.sized(characters.size(), impl.environments, "one learner per environment is required");
    impl.character_range(characters, -1, "learner");
    ok(t8b_sim_set_pending_learners(impl.sim, characters.data()));
}

// reset_all / reset_done / step  full_move_gpu.hpp:87-93
void GpuFullMoveSimulator::reset_all(std::uint64_t seed, std::uint64_t counter) {
    ok(t8b_sim_reset_all(impl_->sim, seed, counter));
}
void GpuFullMoveSimulator::reset_done(std::uint64_t seed, std::uint64_t counter) {
    ok(t8b_sim_reset_done(impl_->sim, seed, counter));
}
void GpuFullMoveSimulator::step(const std::int64_t* learner_candidates, const std::int64_t* opponent_candidates,
                                std::uint64_t seed, std::uint64_t counter) {
    ok(t8b_sim_step(impl_->sim, learner_candidates, opponent_candidates, seed, counter));
}

// device views  full_move_gpu.hpp:96-112
const float* GpuFullMoveSimulator::learner_observations() const noexcept { return t8b_sim_learner_observations(impl_->sim); }
const std::uint8_t* GpuFullMoveSimulator::learner_masks() const noexcept { return t8b_sim_learner_masks(impl_->sim); }
const float* GpuFullMoveSimulator::opponent_observations() const noexcept { return t8b_sim_opponent_observations(impl_->sim); }
const std::uint8_t* GpuFullMoveSimulator::opponent_masks() const noexcept { return t8b_sim_opponent_masks(impl_->sim); }
const float* GpuFullMoveSimulator::rewards() const noexcept { return t8b_sim_rewards(impl_->sim); }
const float* GpuFullMoveSimulator::sparse_rewards() const noexcept { return t8b_sim_sparse_rewards(impl_->sim); }
const std::uint8_t* GpuFullMoveSimulator::terminated() const noexcept { return t8b_sim_terminated(impl_->sim); }
const std::uint8_t* GpuFullMoveSimulator::truncated() const noexcept { return t8b_sim_truncated(impl_->sim); }
const std::int8_t* GpuFullMoveSimulator::outcomes() const noexcept { return t8b_sim_outcomes(impl_->sim); }
const std::int32_t* GpuFullMoveSimulator::learner_feature_tables() const noexcept {
    return t8b_sim_learner_feature_tables(impl_->sim);
}
const std::int32_t* GpuFullMoveSimulator::opponent_feature_tables() const noexcept {
    return t8b_sim_opponent_feature_tables(impl_->sim);
}

// download_noise_levels  full_move_gpu.hpp:110 (empty without live noise, as the reference)
std::vector<fc::NoiseLevels> GpuFullMoveSimulator::download_noise_levels() const {
    if (!impl_->config.live_noise) return {};
    std::vector<t8b_noise_levels_t> packed(impl_->environments);
    ok(t8b_sim_download_noise_levels(impl_->sim, packed.data()));
    std::vector<fc::NoiseLevels> levels(packed.size());
    for (std::size_t i = 0; i < packed.size(); ++i) {
        levels[i] = {packed[i].position_sigma, packed[i].flip_rate, packed[i].latency, packed[i].key};
    }
    return levels;
}

std::vector<std::int32_t> GpuFullMoveSimulator::download_learner_feature_tables() const {
    ok(t8b_sim_synchronize(impl_->sim));
    return download(learner_feature_tables(), impl_->environments, "download learner feature tables");
}
std::vector<std::uint8_t> GpuFullMoveSimulator::download_terminated() const {
    ok(t8b_sim_synchronize(impl_->sim));
    return download(terminated(), impl_->environments, "download terminated");
}
std::vector<std::int8_t> GpuFullMoveSimulator::download_outcomes() const {
    ok(t8b_sim_synchronize(impl_->sim));
    return download(outcomes(), impl_->environments, "download outcomes");
}
std::vector<float> GpuFullMoveSimulator::download_rewards() const {
    ok(t8b_sim_synchronize(impl_->sim));
    return download(rewards(), impl_->environments, "download rewards");
}
std::vector<float> GpuFullMoveSimulator::download_learner_observations() const {
    ok(t8b_sim_synchronize(impl_->sim));
    return download(learner_observations(), impl_->environments * static_cast<std::size_t>(impl_->observation_size),
                    "download learner observations");
}
std::vector<std::uint8_t> GpuFullMoveSimulator::download_learner_masks() const {
    const std::uint8_t* masks = learner_masks();
    ok(t8b_sim_synchronize(impl_->sim));
    return download(masks, impl_->environments * static_cast<std::size_t>(kFullMoveMaxCandidates),
                    "download learner masks");
}

std::vector<int> GpuFullMoveSimulator::download_opponent_characters() const {
    const FullMoveEnvSnapshot s = snapshot();
    std::vector<int> result(s.p1_characters.size());
    for (std::size_t env = 0; env < result.size(); ++env) {
        result[env] = s.learner_is_p1[env] ? s.p2_characters[env] : s.p1_characters[env];
    }
    return result;
}

// frames_simulated  full_move_gpu.hpp:120
std::uint64_t GpuFullMoveSimulator::frames_simulated() const {
    uint64_t frames = 0;
    ok(t8b_sim_frames_simulated(impl_->sim, &frames));
    return frames;
}

// download_and_clear_tally and the three tallies cleared with it  full_move_gpu.hpp:124-131
std::vector<std::uint32_t> GpuFullMoveSimulator::download_and_clear_tally() {
    auto& impl = *impl_;
    std::vector<std::uint32_t> tally(impl.roster.size() * kAggressionBuckets * 2 * 3);
    impl.scenario_tally.assign(static_cast<std::size_t>(T8B_SCENARIOS) * 3, 0);
    impl.learner_tally.assign(impl.roster.size() * 3, 0);
    impl.bot_tally.assign(static_cast<std::size_t>(T8B_SCRIPTED_PROFILES) * 3, 0);
    ok(t8b_sim_download_and_clear_tally(impl.sim, tally.data(), impl.scenario_tally.data(), impl.learner_tally.data(),
                                        impl.bot_tally.data()));
    return tally;
}
std::vector<std::uint32_t> GpuFullMoveSimulator::download_scenario_tally() const { return impl_->scenario_tally; }
std::vector<std::uint32_t> GpuFullMoveSimulator::download_learner_tally() const { return impl_->learner_tally; }
std::vector<std::uint32_t> GpuFullMoveSimulator::download_bot_tally() const { return impl_->bot_tally; }

// snapshot / restore  full_move_gpu.hpp:134-136
FullMoveEnvSnapshot GpuFullMoveSimulator::snapshot() const {
    const std::size_t n = impl_->environments;
    std::vector<t8b_state_t> packed(n);
    FullMoveEnvSnapshot s;
    s.p1_characters.resize(n);
    s.p2_characters.resize(n);
    s.learner_is_p1.resize(n);
    s.aggression.resize(n);
    s.pending_opponents.resize(n);
    s.pending_aggression.resize(n);
    s.terminated.resize(n);
    s.scenarios.resize(n);
    s.pending_scenarios.resize(n);
    s.pending_learners.resize(n);
    ok(t8b_sim_snapshot(impl_->sim, packed.data(), s.p1_characters.data(), s.p2_characters.data(),
                        s.learner_is_p1.data(), s.aggression.data(), s.pending_opponents.data(),
                        s.pending_aggression.data(), s.terminated.data(), s.scenarios.data(), s.pending_scenarios.data(),
                        s.pending_learners.data()));
    s.states.resize(n);
    std::transform(packed.begin(), packed.end(), s.states.begin(), state_from);
    return s;
}

void GpuFullMoveSimulator::restore(const FullMoveEnvSnapshot& s) {
    const std::size_t n = impl_->environments;
    if (s.states.size() != n || s.p1_characters.size() != n || s.p2_characters.size() != n ||
        s.learner_is_p1.size() != n || s.aggression.size() != n || s.pending_opponents.size() != n ||
        s.pending_aggression.size() != n || s.terminated.size() != n || s.scenarios.size() != n ||
        s.pending_scenarios.size() != n || s.pending_learners.size() != n) {
        throw std::invalid_argument("full-move snapshot does not match the environment count");
    }
    impl_->character_range(s.p1_characters, 0, "P1 character");
    impl_->character_range(s.p2_characters, 0, "P2 character");
    impl_->character_range(s.pending_opponents, 0, "opponent");
    std::vector<t8b_state_t> packed(n);
    std::transform(s.states.begin(), s.states.end(), packed.begin(), state_of);
    ok(t8b_sim_restore(impl_->sim, packed.data(), s.p1_characters.data(), s.p2_characters.data(), s.learner_is_p1.data(),
                       s.aggression.data(), s.pending_opponents.data(), s.pending_aggression.data(), s.terminated.data(),
                       s.scenarios.data(), s.pending_scenarios.data(), s.pending_learners.data()));
}

void GpuFullMoveSimulator::synchronize() const {
    check_cuda(cudaDeviceSynchronize(), "synchronize full-move simulator");
}

}  // namespace t8::v2
