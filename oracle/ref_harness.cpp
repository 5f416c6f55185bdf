// Test infrastructure, not product code: a C API over the reference's own CPU engine and
// environment contract, compiled from the reference sources where they lie (see
// oracle/Makefile). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs
// load the library this file builds (oracle/_ref/libt8ref.so).
//
// What it exposes:
//   * t8ref_export_roster: loads characters from the reference's data/generated CSVs with
//     the reference loader (src/full_move_roster.cpp:51 load_full_move_character, stand-in
//     geometry as the trainer's allow_provisional) and writes them into a roster file in
//     the boundary format of include/t8b.h, so the GPU box needs no CSV and no reference;
//   * t8ref_roster_*: reads such a file back into the reference's own full_core tables;
//   * t8ref_random_play: the engine-parity workload of include/t8b.h (PCG32 picks among
//     candidate_legal candidates at every has_decision), run on full_core::step;
//   * t8ref_env_*: the GpuFullMoveSimulator contract on the CPU, built only from the
//     reference's contract functions (include/t8_v2/full_move_contract.hpp: env_reset :980,
//     env_step :1071, encode_observation :535, apply_observation_noise :827,
//     apply_screen_view :905, encode_noise_levels :920, draw_noise_levels :805,
//     candidate_legal :42), in the order src/full_move_gpu.cu:188-255 launches them.
#include "t8_v2/full_move_contract.hpp"
#include "t8_v2/full_move_roster.hpp"

#include "t8b.h"

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <exception>
#include <filesystem>
#include <fstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

using namespace t8::v2;
namespace fc = t8::v2::full_core;

namespace {

thread_local std::string g_error;

int fail(const std::exception& error) {
    g_error = error.what();
    return 1;
}

// ------------------------------------------------------------ boundary conversions

t8b_window_t to_window(const fc::Window& w) {
    t8b_window_t out;
    std::memset(&out, 0, sizeof out);
    out.count = w.count;
    for (int i = 0; i < fc::kMaxWindowSpans; ++i) {
        out.first[i] = w.first[i];
        out.last[i] = w.last[i];
    }
    return out;
}

fc::Window from_window(const t8b_window_t& w) {
    fc::Window out{};
    out.count = w.count;
    for (int i = 0; i < fc::kMaxWindowSpans; ++i) {
        out.first[i] = w.first[i];
        out.last[i] = w.last[i];
    }
    return out;
}

t8b_move_t to_move(const fc::Move& m) {
    t8b_move_t o;
    std::memset(&o, 0, sizeof o);
    o.flags = m.flags;
    o.hit_offset = m.hit_offset; o.hit_count = m.hit_count; o.total_frames = m.total_frames;
    o.recovery = m.recovery; o.block_advantage = m.block_advantage; o.hit_advantage = m.hit_advantage;
    o.counter_hit_advantage = m.counter_hit_advantage; o.launch_air_frames = m.launch_air_frames;
    o.back_turned_hit_advantage = m.back_turned_hit_advantage;
    o.heat_dash_block_advantage = m.heat_dash_block_advantage; o.heat_dash_hit_advantage = m.heat_dash_hit_advantage;
    o.heat_cost_frames = m.heat_cost_frames; o.required_stance = m.required_stance; o.result_stance = m.result_stance;
    o.result_stance_on_hit = m.result_stance_on_hit; o.result_stance_on_block = m.result_stance_on_block;
    for (int i = 0; i < 4; ++i) o.parry_outcomes[i] = m.parry_outcomes[i];
    o.heat_parry_outcome = m.heat_parry_outcome;
    o.hit_effect = static_cast<uint8_t>(m.hit_effect); o.counter_hit_effect = static_cast<uint8_t>(m.counter_hit_effect);
    o.back_turned_hit_effect = static_cast<uint8_t>(m.back_turned_hit_effect);
    o.heat_dash_hit_effect = static_cast<uint8_t>(m.heat_dash_hit_effect);
    o.required_posture = static_cast<uint8_t>(m.required_posture); o.attack_throw = static_cast<uint8_t>(m.attack_throw);
    o.parry_levels = m.parry_levels; o.heat_parry_levels = m.heat_parry_levels;
    o.travel = m.travel; o.pushback_hit = m.pushback_hit; o.pushback_block = m.pushback_block;
    o.reversal_damage = m.reversal_damage; o.attack_throw_damage = m.attack_throw_damage;
    o.recoverable_damage = m.recoverable_damage; o.rage_art_max_damage = m.rage_art_max_damage;
    o.self_damage = m.self_damage; o.self_recoverable = m.self_recoverable; o.restore_health_hit = m.restore_health_hit;
    o.restore_recoverable_hit = m.restore_recoverable_hit; o.restore_recoverable_block = m.restore_recoverable_block;
    o.resource_gain_start = m.resource_gain_start; o.resource_gain_hit = m.resource_gain_hit;
    o.resource_gain_airborne_hit = m.resource_gain_airborne_hit; o.resource_gain_block = m.resource_gain_block;
    o.resource_gain_heat_activation = m.resource_gain_heat_activation;
    o.install_damage_bonus = m.install_damage_bonus; o.install_chip_damage = m.install_chip_damage;
    o.install_reach = m.install_reach;
    const fc::Window* ws[9] = {&m.high_crush, &m.low_crush, &m.power_crush, &m.armor, &m.parry,
                               &m.reversal, &m.invincible, &m.airborne, &m.heat_parry};
    for (int i = 0; i < 9; ++i) o.windows[i] = to_window(*ws[i]);
    return o;
}

fc::Move from_move(const t8b_move_t& o) {
    fc::Move m{};
    m.flags = o.flags;
    m.hit_offset = o.hit_offset; m.hit_count = o.hit_count; m.total_frames = o.total_frames; m.recovery = o.recovery;
    m.block_advantage = o.block_advantage; m.hit_advantage = o.hit_advantage;
    m.counter_hit_advantage = o.counter_hit_advantage; m.launch_air_frames = o.launch_air_frames;
    m.back_turned_hit_advantage = o.back_turned_hit_advantage;
    m.heat_dash_block_advantage = o.heat_dash_block_advantage; m.heat_dash_hit_advantage = o.heat_dash_hit_advantage;
    m.heat_cost_frames = o.heat_cost_frames; m.required_stance = o.required_stance; m.result_stance = o.result_stance;
    m.result_stance_on_hit = o.result_stance_on_hit; m.result_stance_on_block = o.result_stance_on_block;
    for (int i = 0; i < 4; ++i) m.parry_outcomes[i] = o.parry_outcomes[i];
    m.heat_parry_outcome = o.heat_parry_outcome;
    m.hit_effect = static_cast<FullHitEffect>(o.hit_effect);
    m.counter_hit_effect = static_cast<FullHitEffect>(o.counter_hit_effect);
    m.back_turned_hit_effect = static_cast<FullHitEffect>(o.back_turned_hit_effect);
    m.heat_dash_hit_effect = static_cast<FullHitEffect>(o.heat_dash_hit_effect);
    m.required_posture = static_cast<FullPosture>(o.required_posture);
    m.attack_throw = static_cast<FullMoveSpec::AttackThrow>(o.attack_throw);
    m.parry_levels = o.parry_levels; m.heat_parry_levels = o.heat_parry_levels;
    m.travel = o.travel; m.pushback_hit = o.pushback_hit; m.pushback_block = o.pushback_block;
    m.reversal_damage = o.reversal_damage; m.attack_throw_damage = o.attack_throw_damage;
    m.recoverable_damage = o.recoverable_damage; m.rage_art_max_damage = o.rage_art_max_damage;
    m.self_damage = o.self_damage; m.self_recoverable = o.self_recoverable; m.restore_health_hit = o.restore_health_hit;
    m.restore_recoverable_hit = o.restore_recoverable_hit; m.restore_recoverable_block = o.restore_recoverable_block;
    m.resource_gain_start = o.resource_gain_start; m.resource_gain_hit = o.resource_gain_hit;
    m.resource_gain_airborne_hit = o.resource_gain_airborne_hit; m.resource_gain_block = o.resource_gain_block;
    m.resource_gain_heat_activation = o.resource_gain_heat_activation;
    m.install_damage_bonus = o.install_damage_bonus; m.install_chip_damage = o.install_chip_damage;
    m.install_reach = o.install_reach;
    fc::Window* ws[9] = {&m.high_crush, &m.low_crush, &m.power_crush, &m.armor, &m.parry,
                         &m.reversal, &m.invincible, &m.airborne, &m.heat_parry};
    for (int i = 0; i < 9; ++i) *ws[i] = from_window(o.windows[i]);
    return m;
}

t8b_hit_t to_hit(const fc::Hit& h) {
    t8b_hit_t o;
    std::memset(&o, 0, sizeof o);
    o.level = static_cast<uint8_t>(h.level); o.throw_break = static_cast<uint8_t>(h.throw_break); o.flags = h.flags;
    o.first_active_frame = h.first_active_frame; o.active_frames = h.active_frames;
    o.damage = h.damage; o.reach = h.reach; o.tracking_left = h.tracking_left; o.tracking_right = h.tracking_right;
    o.chip_damage = h.chip_damage; o.heat_chip_damage = h.heat_chip_damage;
    return o;
}

fc::Hit from_hit(const t8b_hit_t& o) {
    fc::Hit h{};
    h.level = static_cast<FullHitLevel>(o.level); h.throw_break = static_cast<FullThrowBreak>(o.throw_break);
    h.flags = o.flags; h.first_active_frame = o.first_active_frame; h.active_frames = o.active_frames;
    h.damage = o.damage; h.reach = o.reach; h.tracking_left = o.tracking_left; h.tracking_right = o.tracking_right;
    h.chip_damage = o.chip_damage; h.heat_chip_damage = o.heat_chip_damage;
    return h;
}

t8b_stance_t to_stance(const fc::Stance& s) {
    t8b_stance_t o;
    std::memset(&o, 0, sizeof o);
    o.can_guard = s.can_guard; o.has_max_frames = s.has_max_frames; o.max_frames = s.max_frames;
    o.auto_parry = s.auto_parry;
    for (int i = 0; i < 4; ++i) o.parry_outcomes[i] = s.parry_outcomes[i];
    o.pulse_interval_frames = s.pulse_interval_frames; o.pulse_recoverable = s.pulse_recoverable;
    o.pulse_resource = s.pulse_resource;
    return o;
}

fc::Stance from_stance(const t8b_stance_t& o) {
    fc::Stance s{};
    s.can_guard = o.can_guard != 0; s.has_max_frames = o.has_max_frames != 0; s.max_frames = o.max_frames;
    s.auto_parry = o.auto_parry;
    for (int i = 0; i < 4; ++i) s.parry_outcomes[i] = o.parry_outcomes[i];
    s.pulse_interval_frames = o.pulse_interval_frames; s.pulse_recoverable = o.pulse_recoverable;
    s.pulse_resource = o.pulse_resource;
    return s;
}

t8b_rules_t to_rules(const fc::Rules& r) {
    t8b_rules_t o;
    std::memset(&o, 0, sizeof o);
    o.resource_max = r.resource_max; o.has_install_threshold = r.has_install_threshold;
    o.install_threshold = r.install_threshold; o.resource_persists = r.resource_persists;
    o.install_consumes = r.install_consumes;
    return o;
}

fc::Rules from_rules(const t8b_rules_t& o) {
    return {o.resource_max, o.has_install_threshold != 0, o.install_threshold, o.resource_persists != 0,
            o.install_consumes != 0};
}

t8b_engine_config_t to_config(const FullEngineConfig& c) {
    t8b_engine_config_t o;
    std::memset(&o, 0, sizeof o);
#define T8_COPY(field) o.field = c.field;
    T8_COPY(half_width) T8_COPY(body_radius) T8_COPY(walk_speed) T8_COPY(dash_distance) T8_COPY(dash_frames)
    T8_COPY(backdash_distance) T8_COPY(backdash_frames) T8_COPY(sidestep_distance) T8_COPY(sidestep_frames)
    T8_COPY(axis_realign_per_frame) T8_COPY(launch_air_frames) T8_COPY(juggle_window_frames)
    T8_COPY(juggle_window_decay) T8_COPY(tornado_extra_frames) T8_COPY(knockdown_frames)
    T8_COPY(wakeup_stand_frames) T8_COPY(wakeup_roll_frames) T8_COPY(wakeup_roll_distance)
    T8_COPY(tech_window_frames) T8_COPY(tech_roll_frames) T8_COPY(wall_splat_frames) T8_COPY(crumple_frames)
    T8_COPY(stage_break_air_frames) T8_COPY(wall_break_extension) T8_COPY(combo_scale_step)
    T8_COPY(combo_scale_floor) T8_COPY(counter_hit_damage_scale) T8_COPY(throw_break_window)
    T8_COPY(throw_break_recovery) T8_COPY(parry_outcome_frames) T8_COPY(side_exposure_ratio)
    T8_COPY(back_to_wall_distance) T8_COPY(ki_charge_frames) T8_COPY(ki_charge_damage_scale)
    T8_COPY(parry_stun_frames) T8_COPY(reversal_recovery) T8_COPY(heat_duration_frames) T8_COPY(heat_dash_frames)
    T8_COPY(heat_dash_distance) T8_COPY(rage_health_fraction) T8_COPY(rage_damage_scale) T8_COPY(wall_combo_scale)
    T8_COPY(recoverable_regain_hit) T8_COPY(recoverable_regain_block) T8_COPY(max_health)
#undef T8_COPY
    return o;
}

FullEngineConfig from_config(const t8b_engine_config_t& o) {
    FullEngineConfig c{};
#define T8_COPY(field) c.field = o.field;
    T8_COPY(half_width) T8_COPY(body_radius) T8_COPY(walk_speed) T8_COPY(dash_distance) T8_COPY(dash_frames)
    T8_COPY(backdash_distance) T8_COPY(backdash_frames) T8_COPY(sidestep_distance) T8_COPY(sidestep_frames)
    T8_COPY(axis_realign_per_frame) T8_COPY(launch_air_frames) T8_COPY(juggle_window_frames)
    T8_COPY(juggle_window_decay) T8_COPY(tornado_extra_frames) T8_COPY(knockdown_frames)
    T8_COPY(wakeup_stand_frames) T8_COPY(wakeup_roll_frames) T8_COPY(wakeup_roll_distance)
    T8_COPY(tech_window_frames) T8_COPY(tech_roll_frames) T8_COPY(wall_splat_frames) T8_COPY(crumple_frames)
    T8_COPY(stage_break_air_frames) T8_COPY(wall_break_extension) T8_COPY(combo_scale_step)
    T8_COPY(combo_scale_floor) T8_COPY(counter_hit_damage_scale) T8_COPY(throw_break_window)
    T8_COPY(throw_break_recovery) T8_COPY(parry_outcome_frames) T8_COPY(side_exposure_ratio)
    T8_COPY(back_to_wall_distance) T8_COPY(ki_charge_frames) T8_COPY(ki_charge_damage_scale)
    T8_COPY(parry_stun_frames) T8_COPY(reversal_recovery) T8_COPY(heat_duration_frames) T8_COPY(heat_dash_frames)
    T8_COPY(heat_dash_distance) T8_COPY(rage_health_fraction) T8_COPY(rage_damage_scale) T8_COPY(wall_combo_scale)
    T8_COPY(recoverable_regain_hit) T8_COPY(recoverable_regain_block) T8_COPY(max_health)
#undef T8_COPY
    return c;
}

fc::EnvConfig from_env_config(const t8b_env_config_t& o) {
    fc::EnvConfig c{};
    c.max_round_frames = o.max_round_frames; c.hold_frames = o.hold_frames;
    c.max_frames_per_decision = o.max_frames_per_decision; c.damage_reward = o.damage_reward;
    c.win_reward = o.win_reward; c.draw_penalty = o.draw_penalty; c.throw_break_penalty = o.throw_break_penalty;
    c.time_penalty_per_second = o.time_penalty_per_second; c.damage_dealt_weight = o.damage_dealt_weight;
    c.damage_taken_weight = o.damage_taken_weight; c.distance_penalty_per_second = o.distance_penalty_per_second;
    c.perception_delay = o.perception_delay; c.memory = o.memory != 0; c.live_noise = o.live_noise != 0;
    c.noise_position_max = o.noise_position_max; c.noise_flip_max = o.noise_flip_max;
    c.latency_min = o.latency_min; c.latency_max = o.latency_max; c.screen_view = o.screen_view != 0;
    c.start_center_range = o.start_center_range; c.start_distance_min = o.start_distance_min;
    c.start_distance_max = o.start_distance_max;
    return c;
}

t8b_env_config_t to_env_config(const fc::EnvConfig& c) {
    t8b_env_config_t o;
    std::memset(&o, 0, sizeof o);
    o.max_round_frames = c.max_round_frames; o.hold_frames = c.hold_frames;
    o.max_frames_per_decision = c.max_frames_per_decision; o.damage_reward = c.damage_reward;
    o.win_reward = c.win_reward; o.draw_penalty = c.draw_penalty; o.throw_break_penalty = c.throw_break_penalty;
    o.time_penalty_per_second = c.time_penalty_per_second; o.damage_dealt_weight = c.damage_dealt_weight;
    o.damage_taken_weight = c.damage_taken_weight; o.distance_penalty_per_second = c.distance_penalty_per_second;
    o.perception_delay = c.perception_delay; o.memory = c.memory ? 1 : 0; o.live_noise = c.live_noise ? 1 : 0;
    o.noise_position_max = c.noise_position_max; o.noise_flip_max = c.noise_flip_max;
    o.latency_min = c.latency_min; o.latency_max = c.latency_max; o.screen_view = c.screen_view ? 1 : 0;
    o.start_center_range = c.start_center_range; o.start_distance_min = c.start_distance_min;
    o.start_distance_max = c.start_distance_max;
    return o;
}

t8b_state_t to_state(const fc::State& s) {
    t8b_state_t o;
    std::memset(&o, 0, sizeof o);
    for (int p = 0; p < 2; ++p) {
        const fc::Fighter& f = s.fighters[p];
        t8b_fighter_t& g = o.fighters[p];
        g.health = f.health; g.recoverable_health = f.recoverable_health; g.x = f.x; g.axis = f.axis;
        g.resource = f.resource;
        g.posture = static_cast<uint8_t>(f.posture); g.universal = static_cast<uint8_t>(f.universal);
        g.heat_dash_from = f.heat_dash_from;
        const bool bits[19] = {f.heat, f.heat_available, f.rage, f.rage_available, f.throw_break_attempted,
                               f.installed, f.move_hit, f.move_blocked, f.resource_gained, f.back_turned,
                               f.move_in_heat, f.ki_charge_boost, f.move_boosted, f.in_blockstun, f.tornado_used,
                               f.wall_splat_used, f.wall_scaled, f.techable, f.crumpled};
        for (int b = 0; b < 19; ++b) g.flags |= bits[b] ? (1u << b) : 0u;
        g.stance = f.stance; g.heat_frames = f.heat_frames; g.throw_break_frames = f.throw_break_frames;
        g.pending_throw_hit = f.pending_throw_hit; g.pending_throw_elapsed = f.pending_throw_elapsed;
        g.move = f.move; g.action_frame = f.action_frame; g.hits_landed = f.hits_landed;
        g.stance_frames = f.stance_frames; g.ki_charge_frames = f.ki_charge_frames; g.stun = f.stun;
        g.posture_frames = f.posture_frames; g.grounded_elapsed = f.grounded_elapsed; g.combo_hits = f.combo_hits;
    }
    o.left_wall = s.stage.left_wall; o.right_wall = s.stage.right_wall;
    o.stage_flags = (s.stage.left_wall_breakable ? 1u : 0u) | (s.stage.right_wall_breakable ? 2u : 0u) |
                    (s.stage.left_balcony ? 4u : 0u) | (s.stage.right_balcony ? 8u : 0u) |
                    (s.stage.floor_breakable ? 16u : 0u);
    o.stage_level = s.stage.level;
    o.frame = s.frame;
    o.winner = s.winner;
    return o;
}

fc::State from_state(const t8b_state_t& o) {
    fc::State s{};
    for (int p = 0; p < 2; ++p) {
        const t8b_fighter_t& g = o.fighters[p];
        fc::Fighter& f = s.fighters[p];
        f.health = g.health; f.recoverable_health = g.recoverable_health; f.x = g.x; f.axis = g.axis;
        f.resource = g.resource;
        f.posture = static_cast<FullPosture>(g.posture); f.universal = static_cast<FullUniversal>(g.universal);
        f.heat_dash_from = g.heat_dash_from;
        bool* bits[19] = {&f.heat, &f.heat_available, &f.rage, &f.rage_available, &f.throw_break_attempted,
                          &f.installed, &f.move_hit, &f.move_blocked, &f.resource_gained, &f.back_turned,
                          &f.move_in_heat, &f.ki_charge_boost, &f.move_boosted, &f.in_blockstun, &f.tornado_used,
                          &f.wall_splat_used, &f.wall_scaled, &f.techable, &f.crumpled};
        for (int b = 0; b < 19; ++b) *bits[b] = (g.flags >> b) & 1u;
        f.stance = g.stance; f.heat_frames = g.heat_frames; f.throw_break_frames = g.throw_break_frames;
        f.pending_throw_hit = g.pending_throw_hit; f.pending_throw_elapsed = g.pending_throw_elapsed;
        f.move = g.move; f.action_frame = g.action_frame; f.hits_landed = g.hits_landed;
        f.stance_frames = g.stance_frames; f.ki_charge_frames = g.ki_charge_frames; f.stun = g.stun;
        f.posture_frames = g.posture_frames; f.grounded_elapsed = g.grounded_elapsed; f.combo_hits = g.combo_hits;
    }
    s.stage.left_wall = o.left_wall; s.stage.right_wall = o.right_wall;
    s.stage.left_wall_breakable = o.stage_flags & 1u; s.stage.right_wall_breakable = (o.stage_flags >> 1) & 1u;
    s.stage.left_balcony = (o.stage_flags >> 2) & 1u; s.stage.right_balcony = (o.stage_flags >> 3) & 1u;
    s.stage.floor_breakable = (o.stage_flags >> 4) & 1u;
    s.stage.level = o.stage_level;
    s.frame = o.frame;
    s.winner = o.winner;
    return s;
}

t8b_events_t to_events(const fc::Events& e) {
    t8b_events_t o;
    std::memset(&o, 0, sizeof o);
    o.contact_count = e.contact_count;
    for (int i = 0; i < e.contact_count; ++i) {
        o.contacts[i].attacker = e.contacts[i].attacker;
        o.contacts[i].hit_index = e.contacts[i].hit_index;
        o.contacts[i].contact = static_cast<int>(e.contacts[i].contact);
        o.contacts[i].damage = e.contacts[i].damage;
    }
    o.transition_count = e.transition_count;
    for (int i = 0; i < e.transition_count; ++i) o.transitions[i] = static_cast<uint8_t>(e.transitions[i]);
    o.heat_activated[0] = e.heat_activated[0]; o.heat_activated[1] = e.heat_activated[1];
    o.rage_activated[0] = e.rage_activated[0]; o.rage_activated[1] = e.rage_activated[1];
    return o;
}

// FNV-1a over the 60 32-bit words of the packed state (the hash include/t8b.h defines).
uint64_t state_hash(const t8b_state_t& s) {
    static_assert(sizeof(t8b_state_t) == 240, "packed state layout");
    uint32_t words[60];
    std::memcpy(words, &s, sizeof words);
    uint64_t h = 0xcbf29ce484222325ULL;
    for (uint32_t w : words) h = (h ^ w) * 0x100000001b3ULL;
    return h;
}

// ------------------------------------------------------------ roster file
// Layout: "T8BRST01", u32 count, u32 0, t8b_engine_config_t, then per character
// i32 roster_id, move_count, hit_count, stance_count, candidate_count, 0; char slug[32];
// t8b_rules_t; moves; hits; stances; i32 candidate_moves[]; f32 features[count*32].

struct Character {
    std::string slug;
    int roster_id = -1;
    std::vector<fc::Move> moves;
    std::vector<fc::Hit> hits;
    std::vector<fc::Stance> stances;
    fc::Rules rules{};
    std::vector<int> candidate_moves;
    std::vector<float> features;
    fc::Side side() const {
        fc::Side s{};
        s.moves = moves.data();
        s.move_count = static_cast<int>(moves.size());
        s.hits = hits.data();
        s.stances = stances.data();
        s.stance_count = static_cast<int>(stances.size());
        s.rules = rules;
        return s;
    }
    fc::CandidateMap map() const { return {candidate_moves.data(), static_cast<int>(candidate_moves.size())}; }
};

struct Roster {
    FullEngineConfig config{};
    std::vector<Character> characters;
    fc::Tables tables(int p1, int p2) const {
        fc::Tables t{};
        t.side[0] = characters[static_cast<std::size_t>(p1)].side();
        t.side[1] = characters[static_cast<std::size_t>(p2)].side();
        t.config = config;
        return t;
    }
};

template <typename T>
void put(std::string& out, const T& value) {
    out.append(reinterpret_cast<const char*>(&value), sizeof(T));
}

template <typename T>
T take(const char*& cursor, const char* end) {
    if (static_cast<std::size_t>(end - cursor) < sizeof(T)) throw std::runtime_error("roster file is truncated");
    T value;
    std::memcpy(&value, cursor, sizeof(T));
    cursor += sizeof(T);
    return value;
}

Roster parse_roster(const char* data, std::size_t size) {
    const char* cursor = data;
    const char* end = data + size;
    if (size < 8 || std::memcmp(data, "T8BRST01", 8) != 0) throw std::runtime_error("not a roster file");
    cursor += 8;
    const auto count = take<uint32_t>(cursor, end);
    take<uint32_t>(cursor, end);
    Roster roster;
    roster.config = from_config(take<t8b_engine_config_t>(cursor, end));
    for (uint32_t c = 0; c < count; ++c) {
        Character ch;
        ch.roster_id = take<int32_t>(cursor, end);
        const int moves = take<int32_t>(cursor, end), hits = take<int32_t>(cursor, end);
        const int stances = take<int32_t>(cursor, end), candidates = take<int32_t>(cursor, end);
        take<int32_t>(cursor, end);
        char slug[32];
        for (char& ch_ : slug) ch_ = take<char>(cursor, end);
        slug[31] = 0;
        ch.slug = slug;
        ch.rules = from_rules(take<t8b_rules_t>(cursor, end));
        for (int i = 0; i < moves; ++i) ch.moves.push_back(from_move(take<t8b_move_t>(cursor, end)));
        for (int i = 0; i < hits; ++i) ch.hits.push_back(from_hit(take<t8b_hit_t>(cursor, end)));
        for (int i = 0; i < stances; ++i) ch.stances.push_back(from_stance(take<t8b_stance_t>(cursor, end)));
        for (int i = 0; i < candidates; ++i) ch.candidate_moves.push_back(take<int32_t>(cursor, end));
        for (int i = 0; i < candidates * 32; ++i) ch.features.push_back(take<float>(cursor, end));
        roster.characters.push_back(std::move(ch));
    }
    return roster;
}

// ------------------------------------------------------------ PCG32 (the parity workload's RNG)
// O'Neill's PCG-XSH-RR 64/32 with the reference seeding procedure; bounded draws by
// Lemire's multiply-shift (no rejection loop, so the GPU has no data-dependent loop).
struct Pcg32 {
    uint64_t state = 0, inc = 1;
    Pcg32(uint64_t seed, uint64_t stream) {
        inc = (stream << 1u) | 1u;
        next();
        state += seed;
        next();
    }
    uint32_t next() {
        const uint64_t old = state;
        state = old * 6364136223846793005ULL + inc;
        const uint32_t shifted = static_cast<uint32_t>(((old >> 18u) ^ old) >> 27u);
        const uint32_t rot = static_cast<uint32_t>(old >> 59u);
        return (shifted >> rot) | (shifted << ((32u - rot) & 31u));
    }
    uint32_t below(uint32_t bound) { return static_cast<uint32_t>((static_cast<uint64_t>(next()) * bound) >> 32u); }
};

fc::Input pick_random(const fc::Tables& tables, const fc::State& state, int player, const fc::CandidateMap& map,
                      Pcg32& rng) {
    int legal[kFullMoveMaxCandidates];
    int count = 0;
    for (int c = 0; c < map.count; ++c) {
        if (fc::candidate_legal(tables, state, player, map, c)) legal[count++] = c;
    }
    fc::Input input{};
    if (count == 0) return input;
    const int chosen = legal[rng.below(static_cast<uint32_t>(count))];
    if (!fc::candidate_input(map, chosen, input)) input = fc::Input{};
    return input;
}

template <typename Body>
void parallel_for(std::size_t count, int threads, Body body) {
    if (threads <= 1 || count < 2) {
        for (std::size_t i = 0; i < count; ++i) body(i);
        return;
    }
    std::atomic<std::size_t> next{0};
    std::vector<std::thread> pool;
    std::exception_ptr error;
    std::atomic<bool> failed{false};
    for (int t = 0; t < threads; ++t) {
        pool.emplace_back([&] {
            try {
                for (;;) {
                    const std::size_t i = next.fetch_add(1);
                    if (i >= count) break;
                    body(i);
                }
            } catch (...) {
                if (!failed.exchange(true)) error = std::current_exception();
            }
        });
    }
    for (auto& thread : pool) thread.join();
    if (error) std::rethrow_exception(error);
}

// ------------------------------------------------------------ CPU environment (GpuFullMoveSimulator contract)

struct Env {
    const Roster* roster = nullptr;
    fc::EnvConfig config{};
    std::size_t n = 0;
    int width = 0;
    std::vector<fc::State> states;
    std::vector<fc::Memory> memories;
    std::vector<fc::NoiseLevels> noise;
    std::vector<int> p1, p2, pending_opponents, pending_learners, scenarios, pending_scenarios;
    std::vector<uint8_t> learner_is_p1, terminated;
    std::vector<float> aggression, pending_aggression;
    std::vector<float> learner_obs, opponent_obs, rewards, sparse;
    std::vector<uint8_t> learner_masks, opponent_masks;
    std::vector<int8_t> outcomes;
    uint64_t frames = 0;
    int threads = 1;

    fc::Tables tables(std::size_t env) const { return roster->tables(p1[env], p2[env]); }

    void reset_one(std::size_t env, uint64_t seed, uint64_t counter) {
        // src/full_move_gpu.cu:231-255 env_reset_kernel
        if (config.memory) memories[env] = fc::Memory{};
        if (config.live_noise) noise[env] = fc::draw_noise_levels(config, seed, env, counter);
        if (learner_is_p1[env]) {
            p2[env] = pending_opponents[env];
            if (pending_learners[env] >= 0) p1[env] = pending_learners[env];
        } else {
            p1[env] = pending_opponents[env];
            if (pending_learners[env] >= 0) p2[env] = pending_learners[env];
        }
        aggression[env] = pending_aggression[env];
        scenarios[env] = pending_scenarios[env];
        const int learner = learner_is_p1[env] ? 0 : 1;
        const auto opponent_map = roster->characters[static_cast<std::size_t>(learner == 0 ? p2[env] : p1[env])].map();
        fc::env_reset(tables(env), states[env], config, seed, env, counter, scenarios[env], learner, &opponent_map);
    }

    void observe_one(std::size_t env) {
        // src/full_move_gpu.cu:131-186 observe_kernel + candidate_mask_kernel
        const auto t = tables(env);
        const int learner = learner_is_p1[env] ? 0 : 1;
        const int own = learner == 0 ? p1[env] : p2[env];
        const int other = learner == 0 ? p2[env] : p1[env];
        const auto& chars = roster->characters;
        float* lo = learner_obs.data() + env * static_cast<std::size_t>(width);
        float* oo = opponent_obs.data() + env * static_cast<std::size_t>(width);
        std::fill(lo, lo + width, 0.0F);
        std::fill(oo, oo + width, 0.0F);
        fc::encode_observation(t, states[env], learner, config.max_round_frames, chars[own].roster_id,
                               chars[other].roster_id, lo, config.perception_delay);
        fc::encode_observation(t, states[env], 1 - learner, config.max_round_frames, chars[other].roster_id,
                               chars[own].roster_id, oo, config.perception_delay);
        if (config.memory) {
            fc::encode_memory(memories[env], learner, config.perception_delay, lo + fc::kFullMoveObservationSize);
            fc::encode_memory(memories[env], 1 - learner, config.perception_delay, oo + fc::kFullMoveObservationSize);
        }
        if (config.live_noise) {
            const int offset = fc::full_move_observation_size(config.memory, false);
            fc::apply_observation_noise(noise[env], states[env], learner, lo);
            fc::apply_observation_noise(noise[env], states[env], 1 - learner, oo);
            fc::encode_noise_levels(noise[env], lo + offset);
            fc::encode_noise_levels(noise[env], oo + offset);
        }
        if (config.screen_view) {
            fc::apply_screen_view(lo);
            fc::apply_screen_view(oo);
        }
        for (int side = 0; side < 2; ++side) {
            const int player = side == 0 ? learner : 1 - learner;
            const int character = player == 0 ? p1[env] : p2[env];
            const auto map = chars[static_cast<std::size_t>(character)].map();
            uint8_t* mask = (side == 0 ? learner_masks : opponent_masks).data() + env * kFullMoveMaxCandidates;
            for (int c = 0; c < kFullMoveMaxCandidates; ++c) {
                mask[c] = c < map.count && fc::candidate_legal(t, states[env], player, map, c);
            }
        }
    }

    void observe() {
        parallel_for(n, threads, [&](std::size_t env) { observe_one(env); });
    }
};

}  // namespace

extern "C" {

const char* t8ref_last_error(void) { return g_error.c_str(); }

// Loads characters (comma-separated slugs, or NULL for the 41 roster characters with moves)
// with the reference loader and writes the roster file.
int t8ref_export_roster(const char* generated_dir, const char* slugs, const char* out_path) {
    try {
        std::vector<std::string> names;
        if (slugs == nullptr || *slugs == 0) {
            for (const auto slug : kRosterCharacterSlugs) {
                if (slug != "bob") names.emplace_back(slug);
            }
        } else {
            std::string list = slugs;
            std::size_t start = 0;
            while (start <= list.size()) {
                const auto comma = list.find(',', start);
                names.push_back(list.substr(start, comma == std::string::npos ? std::string::npos : comma - start));
                if (comma == std::string::npos) break;
                start = comma + 1;
            }
        }
        FullMoveRosterOptions options{};
        options.allow_provisional = true;
        std::string out("T8BRST01", 8);
        put(out, static_cast<uint32_t>(names.size()));
        put(out, static_cast<uint32_t>(0));
        put(out, to_config(options.engine));
        for (const auto& name : names) {
            const FullMoveCharacter ch = load_full_move_character(generated_dir, name, options);
            put(out, static_cast<int32_t>(ch.roster_id));
            put(out, static_cast<int32_t>(ch.tables.moves[0].size()));
            put(out, static_cast<int32_t>(ch.tables.hits[0].size()));
            put(out, static_cast<int32_t>(ch.tables.stances[0].size()));
            put(out, static_cast<int32_t>(ch.candidate_count()));
            put(out, static_cast<int32_t>(0));
            char slug[32] = {};
            std::snprintf(slug, sizeof slug, "%s", ch.slug.c_str());
            out.append(slug, sizeof slug);
            put(out, to_rules(ch.tables.rules[0]));
            for (const auto& m : ch.tables.moves[0]) put(out, to_move(m));
            for (const auto& h : ch.tables.hits[0]) put(out, to_hit(h));
            for (const auto& s : ch.tables.stances[0]) put(out, to_stance(s));
            for (int m : ch.candidate_moves) put(out, static_cast<int32_t>(m));
            for (float f : ch.candidate_features) put(out, f);
        }
        std::ofstream file(out_path, std::ios::binary);
        file.write(out.data(), static_cast<std::streamsize>(out.size()));
        if (!file) throw std::runtime_error(std::string("cannot write ") + out_path);
        return 0;
    } catch (const std::exception& error) {
        return fail(error);
    }
}

void* t8ref_roster_parse(const void* data, size_t size) {
    try {
        return new Roster(parse_roster(static_cast<const char*>(data), size));
    } catch (const std::exception& error) {
        fail(error);
        return nullptr;
    }
}

void t8ref_roster_free(void* roster) { delete static_cast<Roster*>(roster); }
// full_core::EnvConfig's default member initialisers (include/t8_v2/full_move_contract.hpp:737-773).
void t8ref_env_config_default(t8b_env_config_t* out) { *out = to_env_config(fc::EnvConfig{}); }

// Candidate feature tables of a parsed roster: out[character][stride][32], zero past each
// character's candidates (the trainer's table layout, src/full_move_train.cpp:1176-1184).
int t8ref_roster_features(void* roster_handle, float* out, int stride) {
    const Roster& roster = *static_cast<Roster*>(roster_handle);
    for (std::size_t c = 0; c < roster.characters.size(); ++c) {
        float* table = out + c * static_cast<std::size_t>(stride) * 32;
        std::fill(table, table + static_cast<std::size_t>(stride) * 32, 0.0F);
        const auto& f = roster.characters[c].features;
        std::copy(f.begin(), f.begin() + std::min<std::size_t>(f.size(), static_cast<std::size_t>(stride) * 32), table);
    }
    return 0;
}

int t8ref_roster_count(void* roster) { return static_cast<int>(static_cast<Roster*>(roster)->characters.size()); }

// The engine-parity workload (include/t8b.h t8b_sim_random_play) on full_core::step.
// hashes: [fights][frames]; states (optional): [fights][frames] packed states;
// inputs (optional): [fights][frames][2].
int t8ref_random_play(void* roster_handle, int fights, const int32_t* p1, const int32_t* p2, const double* x1,
                      const double* x2, int frames, uint64_t seed, uint64_t* hashes, t8b_state_t* states,
                      t8b_input_t* inputs, t8b_events_t* events, int threads) {
    try {
        const Roster& roster = *static_cast<Roster*>(roster_handle);
        parallel_for(static_cast<std::size_t>(fights), threads, [&](std::size_t f) {
            const auto tables = roster.tables(p1[f], p2[f]);
            const fc::CandidateMap maps[2] = {roster.characters[static_cast<std::size_t>(p1[f])].map(),
                                              roster.characters[static_cast<std::size_t>(p2[f])].map()};
            Pcg32 rng(seed, f);
            fc::State state{};
            fc::reset(tables, state, x1[f], x2[f]);
            for (int frame = 0; frame < frames; ++frame) {
                if (state.winner >= 0) fc::next_round(tables, state, x1[f], x2[f]);
                fc::Input chosen[2] = {};
                for (int player = 0; player < 2; ++player) {
                    if (fc::has_decision(tables, state, player)) chosen[player] = pick_random(tables, state, player, maps[player], rng);
                }
                fc::Events ev{};
                fc::step(tables, state, chosen[0], chosen[1], ev);
                const std::size_t at = f * static_cast<std::size_t>(frames) + static_cast<std::size_t>(frame);
                const t8b_state_t packed = to_state(state);
                hashes[at] = state_hash(packed);
                if (states) states[at] = packed;
                if (inputs) {
                    for (int p = 0; p < 2; ++p) inputs[2 * at + static_cast<std::size_t>(p)] = {chosen[p].move, static_cast<int32_t>(chosen[p].universal)};
                }
                if (events) events[at] = to_events(ev);
            }
        });
        return 0;
    } catch (const std::exception& error) {
        return fail(error);
    }
}

// One engine frame from explicit states and inputs (engine-level API parity).
int t8ref_engine_step(void* roster_handle, int count, const int32_t* p1, const int32_t* p2, t8b_state_t* states,
                      const t8b_input_t* inputs, t8b_events_t* events) {
    try {
        const Roster& roster = *static_cast<Roster*>(roster_handle);
        for (int i = 0; i < count; ++i) {
            const auto tables = roster.tables(p1[i], p2[i]);
            fc::State s = from_state(states[i]);
            fc::Events e{};
            fc::Input a{inputs[2 * i].move, static_cast<FullUniversal>(inputs[2 * i].universal)};
            fc::Input b{inputs[2 * i + 1].move, static_cast<FullUniversal>(inputs[2 * i + 1].universal)};
            fc::step(tables, s, a, b, e);
            states[i] = to_state(s);
            if (events) events[i] = to_events(e);
        }
        return 0;
    } catch (const std::exception& error) {
        return fail(error);
    }
}

int t8ref_reset_state(void* roster_handle, int p1, int p2, double x1, double x2, t8b_state_t* out) {
    const Roster& roster = *static_cast<Roster*>(roster_handle);
    fc::State s{};
    fc::reset(roster.tables(p1, p2), s, x1, x2);
    *out = to_state(s);
    return 0;
}

uint64_t t8ref_state_hash(const t8b_state_t* state) { return state_hash(*state); }

// ---- CPU environment
void* t8ref_env_create(void* roster_handle, size_t n, const t8b_env_config_t* config, int threads) {
    try {
        auto* env = new Env();
        env->roster = static_cast<Roster*>(roster_handle);
        env->config = from_env_config(*config);
        env->n = n;
        env->threads = threads;
        env->width = fc::full_move_observation_size(env->config.memory, env->config.live_noise);
        env->states.assign(n, fc::State{});
        env->memories.assign(n, fc::Memory{});
        env->noise.assign(n, fc::NoiseLevels{});
        env->p1.assign(n, 0); env->p2.assign(n, 0); env->pending_opponents.assign(n, 0);
        env->pending_learners.assign(n, -1); env->scenarios.assign(n, 0); env->pending_scenarios.assign(n, 0);
        env->learner_is_p1.assign(n, 1); env->terminated.assign(n, 0);
        env->aggression.assign(n, 0.0F); env->pending_aggression.assign(n, 0.0F);
        env->learner_obs.assign(n * static_cast<std::size_t>(env->width), 0.0F);
        env->opponent_obs.assign(n * static_cast<std::size_t>(env->width), 0.0F);
        env->rewards.assign(n, 0.0F); env->sparse.assign(n, 0.0F); env->outcomes.assign(n, 0);
        env->learner_masks.assign(n * kFullMoveMaxCandidates, 0);
        env->opponent_masks.assign(n * kFullMoveMaxCandidates, 0);
        for (auto& s : env->states) fc::reset(env->roster->tables(0, 0), s, -0.8, 0.8);
        return env;
    } catch (const std::exception& error) {
        fail(error);
        return nullptr;
    }
}

void t8ref_env_free(void* env) { delete static_cast<Env*>(env); }
int t8ref_env_observation_size(void* env) { return static_cast<Env*>(env)->width; }

int t8ref_env_setup(void* handle, const int32_t* p1, const int32_t* p2, const uint8_t* learner_is_p1,
                    const int32_t* pending_opponents, const float* pending_aggression, const int32_t* pending_scenarios,
                    const int32_t* pending_learners) {
    auto& env = *static_cast<Env*>(handle);
    for (std::size_t i = 0; i < env.n; ++i) {
        if (p1) env.p1[i] = p1[i];
        if (p2) env.p2[i] = p2[i];
        if (learner_is_p1) env.learner_is_p1[i] = learner_is_p1[i];
        if (pending_opponents) env.pending_opponents[i] = pending_opponents[i];
        if (pending_aggression) env.pending_aggression[i] = pending_aggression[i];
        if (pending_scenarios) env.pending_scenarios[i] = pending_scenarios[i];
        if (pending_learners) env.pending_learners[i] = pending_learners[i];
    }
    return 0;
}

// src/full_move_gpu.cu:531-543 reset_all
int t8ref_env_reset_all(void* handle, uint64_t seed, uint64_t counter) {
    try {
        auto& env = *static_cast<Env*>(handle);
        parallel_for(env.n, env.threads, [&](std::size_t i) { env.reset_one(i, seed, counter); });
        std::fill(env.terminated.begin(), env.terminated.end(), 0);
        env.observe();
        return 0;
    } catch (const std::exception& error) {
        return fail(error);
    }
}

// src/full_move_gpu.cu:545-556 reset_done
int t8ref_env_reset_done(void* handle, uint64_t seed, uint64_t counter) {
    try {
        auto& env = *static_cast<Env*>(handle);
        parallel_for(env.n, env.threads, [&](std::size_t i) {
            if (env.terminated[i]) env.reset_one(i, seed, counter);
        });
        env.observe();
        return 0;
    } catch (const std::exception& error) {
        return fail(error);
    }
}

// src/full_move_gpu.cu:188-229 env_step_kernel + observe. opponent may be NULL (scripted).
int t8ref_env_step(void* handle, const int64_t* learner, const int64_t* opponent, uint64_t seed, uint64_t counter,
                   int observe) {
    try {
        auto& env = *static_cast<Env*>(handle);
        std::vector<uint64_t> frames(env.n, 0);
        parallel_for(env.n, env.threads, [&](std::size_t i) {
            const int learner_side = env.learner_is_p1[i] ? 0 : 1;
            const auto& chars = env.roster->characters;
            const auto lmap = chars[static_cast<std::size_t>(learner_side == 0 ? env.p1[i] : env.p2[i])].map();
            const auto omap = chars[static_cast<std::size_t>(learner_side == 0 ? env.p2[i] : env.p1[i])].map();
            const auto result = fc::env_step(env.tables(i), env.states[i], learner_side, lmap, omap,
                                             static_cast<int>(learner[i]),
                                             opponent != nullptr ? static_cast<int>(opponent[i]) : -1,
                                             env.aggression[i], env.config, seed, i, counter,
                                             env.config.memory ? &env.memories[i] : nullptr,
                                             env.config.live_noise ? &env.noise[i] : nullptr);
            env.rewards[i] = result.reward;
            env.sparse[i] = result.sparse_reward;
            env.terminated[i] = result.terminated ? 1 : 0;
            env.outcomes[i] = result.outcome;
            frames[i] = static_cast<uint64_t>(result.frames);
        });
        for (uint64_t f : frames) env.frames += f;
        if (observe) env.observe();
        return 0;
    } catch (const std::exception& error) {
        return fail(error);
    }
}

int t8ref_env_read(void* handle, float* learner_obs, float* opponent_obs, uint8_t* learner_masks,
                   uint8_t* opponent_masks, float* rewards, float* sparse, uint8_t* terminated, int8_t* outcomes,
                   t8b_state_t* states, t8b_noise_levels_t* noise, int32_t* p1, int32_t* p2, uint64_t* frames) {
    auto& env = *static_cast<Env*>(handle);
    const std::size_t n = env.n;
    if (learner_obs) std::copy(env.learner_obs.begin(), env.learner_obs.end(), learner_obs);
    if (opponent_obs) std::copy(env.opponent_obs.begin(), env.opponent_obs.end(), opponent_obs);
    if (learner_masks) std::copy(env.learner_masks.begin(), env.learner_masks.end(), learner_masks);
    if (opponent_masks) std::copy(env.opponent_masks.begin(), env.opponent_masks.end(), opponent_masks);
    if (rewards) std::copy(env.rewards.begin(), env.rewards.end(), rewards);
    if (sparse) std::copy(env.sparse.begin(), env.sparse.end(), sparse);
    if (terminated) std::copy(env.terminated.begin(), env.terminated.end(), terminated);
    if (outcomes) std::copy(env.outcomes.begin(), env.outcomes.end(), outcomes);
    for (std::size_t i = 0; i < n; ++i) {
        if (states) states[i] = to_state(env.states[i]);
        if (noise) noise[i] = {env.noise[i].position_sigma, env.noise[i].flip_rate, env.noise[i].latency, env.noise[i].key};
        if (p1) p1[i] = env.p1[i];
        if (p2) p2[i] = env.p2[i];
    }
    if (frames) *frames = env.frames;
    return 0;
}

int t8ref_env_upload_states(void* handle, const t8b_state_t* states) {
    auto& env = *static_cast<Env*>(handle);
    for (std::size_t i = 0; i < env.n; ++i) env.states[i] = from_state(states[i]);
    return 0;
}

}  // extern "C"
