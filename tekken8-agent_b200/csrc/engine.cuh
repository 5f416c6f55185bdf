// Frame-stepped fight engine for the GPU: one fight per thread, fp64 state, the exact
// arithmetic of the reference CPU engine (include/t8_v2/full_combat_core.hpp) so that a
// fight stepped here is bit-identical to one stepped by full_core::step. Built with
// --fmad=false: a fused multiply-add rounds once where the reference rounds twice.
//
// Layout differs from the reference. A fight lives in registers as `Fight` (fighter flags
// packed in one word), loaded from and stored to HBM once per decision. Moves use the
// compact `DMove` record (304 B instead of 880 B): scalars plus nine packed window
// descriptors into a per-roster span pool, since no window has more than a few spans.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define T8B_HD __host__ __device__ __forceinline__
#else
#define T8B_HD inline
#endif

namespace t8b {

// ------------------------------------------------------------------ enumerations
// Values of the reference enums (include/t8_v2/full_combat_engine.hpp:44-77,215-230,347-353).
enum Level : uint8_t { kHigh = 0, kMid = 1, kLow = 2, kSpecialMid = 3, kSpecialLow = 4, kThrow = 5 };
enum Effect : uint8_t { kStun = 0, kLaunch = 1, kKnockdown = 2, kCrumple = 3 };
enum BreakRule : uint8_t { kBreakNone = 0, kBreakOne = 1, kBreakTwo = 2, kBreakOneTwo = 3, kBreakOneOrTwo = 4 };
enum Posture : uint8_t { kStanding = 0, kCrouching = 1, kAirborne = 2, kGrounded = 3, kWakeup = 4, kWallSplat = 5 };
enum Universal : uint8_t {
    kIdle = 0, kWalkForward = 1, kWalkBack = 2, kDashForward = 3, kBackdash = 4, kCrouch = 5,
    kSidestepLeft = 6, kSidestepRight = 7, kThrowBreak = 8, kThrowBreak1 = 9, kThrowBreak2 = 10,
    kHeatDash = 11, kWakeupStand = 12, kWakeupRoll = 13, kTechRoll = 14,
};
enum Contact : uint8_t {
    kHit = 0, kCounterHit = 1, kBlocked = 2, kCrushed = 3, kParried = 4, kArmored = 5, kEvaded = 6,
    kThrowBroken = 7, kReversed = 8, kThrowHeld = 9,
};
enum Transition : uint8_t { kWallBreak = 0, kFloorBreak = 1, kBalconyBreak = 2 };
enum AttackThrow : uint8_t { kAttackThrowNone = 0, kAttackThrowOnHit = 1, kAttackThrowOnCounterHit = 2 };

// Hit flag bits (full_combat_core.hpp:49-53).
constexpr uint16_t kHoming = 1u << 0, kGroundHit = 1u << 1, kWallSplatHit = 1u << 2, kWallBreakHit = 1u << 3,
                   kFloorBreakHit = 1u << 4, kBalconyBreakHit = 1u << 5, kTornado = 1u << 6, kSpike = 1u << 7,
                   kUnparryable = 1u << 8, kReversalBreak = 1u << 9, kHasHeatChip = 1u << 10;
// Move flag bits (full_combat_core.hpp:69-82).
constexpr uint64_t kReactive = 1ull << 0, kRequiresSidestep = 1ull << 1, kRequiresBackToWall = 1ull << 2,
    kRequiresBackTurned = 1ull << 3, kRequiresOpponentBackTurned = 1ull << 4, kRequiresOpponentLeft = 1ull << 5,
    kRequiresOpponentRight = 1ull << 6, kResultBackTurned = 1ull << 7, kResultCrouching = 1ull << 8,
    kAttackThrowFrontOnly = 1ull << 9, kAttackThrowStandingOnly = 1ull << 10, kAttackThrowAirborne = 1ull << 11,
    kCannotKo = 1ull << 12, kKiCharge = 1ull << 13, kRequiresHeat = 1ull << 14, kRequiresRage = 1ull << 15,
    kEngagesHeat = 1ull << 16, kHeatEngager = 1ull << 17, kConsumesHeat = 1ull << 18, kConsumesRage = 1ull << 19,
    kRecoverableOnly = 1ull << 20, kRemovesRecoverable = 1ull << 21, kArmorDamageRecoverable = 1ull << 22,
    kSelfDamageWithoutHeatOnly = 1ull << 23, kSideSwitchOnHit = 1ull << 24, kSideSwitchOnBreak = 1ull << 25,
    kHasCounterHitAdvantage = 1ull << 26, kHasCounterHitEffect = 1ull << 27, kHasLaunchAirFrames = 1ull << 28,
    kHasBackTurnedHitAdvantage = 1ull << 29, kHasRageArtMax = 1ull << 30, kHasHeatDashBlock = 1ull << 31,
    kHasHeatDashHit = 1ull << 32, kHasInstallChip = 1ull << 33, kHasInstallReach = 1ull << 34;

// Fighter flag bits (the packed order of include/t8b.h).
constexpr uint32_t fHeat = 1u << 0, fHeatAvailable = 1u << 1, fRage = 1u << 2, fRageAvailable = 1u << 3,
    fBreakAttempted = 1u << 4, fInstalled = 1u << 5, fMoveHit = 1u << 6, fMoveBlocked = 1u << 7,
    fResourceGained = 1u << 8, fBackTurned = 1u << 9, fMoveInHeat = 1u << 10, fKiBoost = 1u << 11,
    fMoveBoosted = 1u << 12, fInBlockstun = 1u << 13, fTornadoUsed = 1u << 14, fWallSplatUsed = 1u << 15,
    fWallScaled = 1u << 16, fTechable = 1u << 17, fCrumpled = 1u << 18;
// Stage flag bits.
constexpr uint32_t sLeftBreakable = 1u << 0, sRightBreakable = 1u << 1, sLeftBalcony = 1u << 2,
                   sRightBalcony = 1u << 3, sFloorBreakable = 1u << 4;

constexpr int kNoContactFrom = -1;
constexpr int kNoOutcome = -1;
constexpr int kUniversalCount = 22;
constexpr int kMaxCandidates = 368;
constexpr int kStateFeatures = 64;
constexpr int kRosterSlots = 42;
constexpr int kObservationBase = kStateFeatures + 2 * kRosterSlots;  // 148
constexpr int kMaxContacts = 8;
constexpr int kMaxTransitions = 4;

// Windows, in DMove::windows order.
enum WindowKind { wHighCrush = 0, wLowCrush, wPowerCrush, wArmor, wParry, wReversal, wInvincible, wAirborne, wHeatParry };

// ------------------------------------------------------------------ tables (device layout)
struct DHit {
    uint8_t level, throw_break;
    uint16_t flags;
    int32_t first_active_frame, active_frames, pad;
    double damage, reach, tracking_left, tracking_right, chip_damage, heat_chip_damage;
};

struct alignas(16) DMove {
    uint64_t flags;
    int32_t hit_offset, hit_count, total_frames, recovery;
    int32_t block_advantage, hit_advantage, counter_hit_advantage, launch_air_frames;
    int32_t back_turned_hit_advantage, heat_dash_block_advantage, heat_dash_hit_advantage, heat_cost_frames;
    int32_t required_stance, result_stance, result_stance_on_hit, result_stance_on_block;
    int32_t parry_outcomes[4];
    int32_t heat_parry_outcome;
    int32_t approach_frames;  // frames of travel before the first hit (first_active_frame - 1), 0 without hits
    uint8_t hit_effect, counter_hit_effect, back_turned_hit_effect, heat_dash_hit_effect;
    uint8_t required_posture, attack_throw, parry_levels, heat_parry_levels;
    double travel, pushback_hit, pushback_block, reversal_damage, attack_throw_damage;
    double recoverable_damage, rage_art_max_damage, self_damage, self_recoverable;
    double restore_health_hit, restore_recoverable_hit, restore_recoverable_block;
    double resource_gain_start, resource_gain_hit, resource_gain_airborne_hit, resource_gain_block;
    double resource_gain_heat_activation, install_damage_bonus, install_chip_damage, install_reach;
    uint32_t windows[9];  // (first span index << 4) | span count, into the span pool
    uint32_t pad;
};

struct DStance {
    uint8_t can_guard, has_max_frames, auto_parry, pad;
    int32_t max_frames;
    int32_t parry_outcomes[4];
    int32_t pulse_interval_frames;
    double pulse_recoverable, pulse_resource;
};

struct DRules {
    double resource_max, install_threshold;
    uint32_t has_install_threshold, resource_persists;
};

// Precomputed per-candidate move facts for the tiered bots (full_move_contract.hpp:280-313).
struct DFacts {
    double damage, reach;
    uint64_t flags;
    int32_t startup;
    uint32_t bits;  // 1 valid, 2 safe, 4 launcher, 8 low, 16 throw
};

// What legal's move branch reads of a move candidate's move (flags, required posture, stance
// and heat cost), per candidate: one 16-byte record instead of three 32-byte sectors of the
// move record behind the candidate's move index. move is -1 for candidates without a move.
struct alignas(16) DGate {
    uint64_t flags;
    int32_t required_stance;
    uint8_t required_posture;
    uint8_t heat_cost;  // heat_cost_frames != 0
    int16_t move;
};

// One roster character on the device.
struct DCharacter {
    const DMove* moves;
    const DHit* hits;
    const DStance* stances;
    const int2* spans;
    const int32_t* candidate_moves;
    const DFacts* facts;
    const DGate* gates;  // [candidate_count]
    double move_candidate_inverse;  // 1 / (candidate_count - kUniversalCount), 0 without move candidates
    int32_t move_count, stance_count, candidate_count, roster_id;
    DRules rules;
};

// FullEngineConfig (full_combat_engine.hpp:236-289).
struct Cfg {
    double half_width, body_radius, walk_speed, dash_distance;
    int32_t dash_frames, backdash_frames;
    double backdash_distance, sidestep_distance;
    int32_t sidestep_frames, launch_air_frames;
    double axis_realign_per_frame;
    int32_t juggle_window_frames, juggle_window_decay, tornado_extra_frames, knockdown_frames;
    int32_t wakeup_stand_frames, wakeup_roll_frames;
    double wakeup_roll_distance;
    int32_t tech_window_frames, tech_roll_frames, wall_splat_frames, crumple_frames, stage_break_air_frames, pad0;
    double wall_break_extension, combo_scale_step, combo_scale_floor, counter_hit_damage_scale;
    int32_t throw_break_window, throw_break_recovery, parry_outcome_frames, pad1;
    double side_exposure_ratio, back_to_wall_distance;
    int32_t ki_charge_frames, pad2;
    double ki_charge_damage_scale;
    int32_t parry_stun_frames, reversal_recovery, heat_duration_frames, heat_dash_frames;
    double heat_dash_distance, rage_health_fraction, rage_damage_scale, wall_combo_scale;
    double recoverable_regain_hit, recoverable_regain_block, max_health;
};

// EnvConfig (full_move_contract.hpp:737-773).
struct EnvCfg {
    int32_t max_round_frames, hold_frames, max_frames_per_decision;
    float damage_reward, win_reward, draw_penalty, throw_break_penalty, time_penalty_per_second;
    float damage_dealt_weight, damage_taken_weight, distance_penalty_per_second;
    int32_t perception_delay;
    uint8_t memory, live_noise, screen_view, pad;
    float noise_position_max, noise_flip_max;
    int32_t latency_min, latency_max, pad2;
    double start_center_range, start_distance_min, start_distance_max;
};

// ------------------------------------------------------------------ fight state
struct Fighter {
    double health, recoverable, x, axis, resource;
    uint8_t posture, universal;
    int8_t dash_from;  // Heat Dash enabled by this contact, or -1
    uint8_t pad;
    uint32_t flags;
    int32_t stance, heat_frames, break_frames, pending_throw_hit, pending_throw_elapsed;
    int32_t move, action_frame;
    uint32_t hits_landed;
    int32_t stance_frames, ki_frames, stun, posture_frames, grounded_elapsed, combo_hits;
};

struct Fight {
    Fighter f[2];
    double left_wall, right_wall;
    uint32_t stage;
    int32_t level, frame, winner;
};

struct Input {
    int32_t move;       // -1: the universal action
    int32_t universal;  // Universal
};

struct ContactEvent {
    int32_t attacker, hit_index, contact, pad;
    double damage;
};

struct Events {
    int32_t contact_count, transition_count;
    ContactEvent contacts[kMaxContacts];
    uint8_t transitions[kMaxTransitions];
    uint8_t heat_activated[2], rage_activated[2];
};

// The fighters' tables during one step.
struct Match {
    const DCharacter* side[2];
    const Cfg* cfg;
};

// ------------------------------------------------------------------ small helpers
T8B_HD double lo(double a, double b) { return b < a ? b : a; }
T8B_HD double hi(double a, double b) { return a < b ? b : a; }
T8B_HD int ilo(int a, int b) { return b < a ? b : a; }
T8B_HD int ihi(int a, int b) { return a < b ? b : a; }
T8B_HD double mag(double v) { return v < 0.0 ? -v : v; }
T8B_HD double clampd(double v, double a, double b) { return v < a ? a : (b < v ? b : v); }
T8B_HD bool on(const Fighter& f, uint32_t bit) { return (f.flags & bit) != 0u; }
T8B_HD void put(Fighter& f, uint32_t bit, bool value) { f.flags = value ? (f.flags | bit) : (f.flags & ~bit); }
T8B_HD bool has(const DMove& m, uint64_t bit) { return (m.flags & bit) != 0ull; }
T8B_HD void swapd(double& a, double& b) { const double t = a; a = b; b = t; }

T8B_HD uint8_t level_bits(uint8_t level) {
    return level == kHigh ? 1 : (level == kLow || level == kSpecialLow) ? 4 : level == kThrow ? 8 : 2;
}
T8B_HD int level_slot(uint8_t level) {
    return level == kHigh ? 0 : (level == kLow || level == kSpecialLow) ? 2 : level == kThrow ? 3 : 1;
}
T8B_HD bool is_low(uint8_t level) { return level == kLow || level == kSpecialLow; }
T8B_HD bool is_break_input(int u) { return u == kThrowBreak || u == kThrowBreak1 || u == kThrowBreak2; }
T8B_HD bool escapes(uint8_t rule, int u) {
    switch (rule) {
        case kBreakOne: return u == kThrowBreak1;
        case kBreakTwo: return u == kThrowBreak2;
        case kBreakOneTwo: return u == kThrowBreak;
        case kBreakOneOrTwo: return u == kThrowBreak1 || u == kThrowBreak2;
        default: return false;
    }
}
T8B_HD int action_length(int u, const Cfg& c) {
    switch (u) {
        case kDashForward: return c.dash_frames;
        case kBackdash: return c.backdash_frames;
        case kSidestepLeft:
        case kSidestepRight: return c.sidestep_frames;
        case kHeatDash: return c.heat_dash_frames;
        default: return 1;
    }
}

T8B_HD const DMove& move_at(const Match& m, int p, int index) { return m.side[p]->moves[index]; }
T8B_HD const DHit& hit_at(const Match& m, int p, const DMove& mv, int k) { return m.side[p]->hits[mv.hit_offset + k]; }
T8B_HD const DStance* stance_of(const Match& m, const Fight& s, int p) {
    const int st = s.f[p].stance;
    if (st < 0 || st >= m.side[p]->stance_count) return nullptr;
    return &m.side[p]->stances[st];
}
T8B_HD bool in_window(const Match& m, int p, const DMove& mv, int kind, int frame) {
    const uint32_t packed = mv.windows[kind];
    const uint32_t count = packed & 15u;
    const int2* span = m.side[p]->spans + (packed >> 4);
    for (uint32_t i = 0; i < count; ++i) {
        if (frame >= span[i].x && frame <= span[i].y) return true;
    }
    return false;
}

T8B_HD void add_contact(Events& e, int attacker, int hit, int contact, double damage) {
    if (e.contact_count < kMaxContacts) {
        ContactEvent& c = e.contacts[e.contact_count++];
        c.attacker = attacker;
        c.hit_index = hit;
        c.contact = contact;
        c.pad = 0;
        c.damage = damage;
    }
}
T8B_HD void add_transition(Events& e, int t) {
    if (e.transition_count < kMaxTransitions) e.transitions[e.transition_count++] = static_cast<uint8_t>(t);
}

// ------------------------------------------------------------------ resources and damage
// gain_resource (full_combat_core.hpp:342-348)
T8B_HD void gain(const Match& m, Fight& s, int p, double amount) {
    const DRules& r = m.side[p]->rules;
    if (!(r.resource_max > 0.0) || !(amount > 0.0)) return;
    Fighter& f = s.f[p];
    f.resource = lo(r.resource_max, f.resource + amount);
    if (r.has_install_threshold && f.resource >= r.install_threshold) f.flags |= fInstalled;
}

// reset / next_round (full_combat_core.hpp:350-368)
T8B_HD void fresh_fight(const Match& m, Fight& s, double x1, double x2) {
    const Cfg& c = *m.cfg;
    for (int p = 0; p < 2; ++p) {
        Fighter& f = s.f[p];
        f.health = c.max_health;
        f.recoverable = 0.0;
        f.x = p == 0 ? x1 : x2;
        f.axis = 0.0;
        f.resource = 0.0;
        f.posture = kStanding;
        f.universal = kIdle;
        f.dash_from = kNoContactFrom;
        f.pad = 0;
        f.flags = fHeatAvailable | fRageAvailable;
        f.stance = -1;
        f.heat_frames = 0;
        f.break_frames = 0;
        f.pending_throw_hit = -1;
        f.pending_throw_elapsed = 0;
        f.move = -1;
        f.action_frame = action_length(kIdle, c);
        f.hits_landed = 0;
        f.stance_frames = 0;
        f.ki_frames = 0;
        f.stun = 0;
        f.posture_frames = 0;
        f.grounded_elapsed = 0;
        f.combo_hits = 0;
    }
    s.left_wall = -c.half_width;
    s.right_wall = c.half_width;
    s.stage = sLeftBreakable | sRightBreakable | sFloorBreakable;
    s.level = 0;
    s.frame = 0;
    s.winner = -1;
}

T8B_HD void next_round(const Match& m, Fight& s, double x1, double x2) {
    const double kept0 = s.f[0].resource, kept1 = s.f[1].resource;
    fresh_fight(m, s, x1, x2);
    if (m.side[0]->rules.resource_persists) gain(m, s, 0, kept0);
    if (m.side[1]->rules.resource_persists) gain(m, s, 1, kept1);
}

// actionable (full_combat_core.hpp:370-378)
T8B_HD bool can_act(const Match& m, const Fight& s, int p) {
    const Fighter& f = s.f[p];
    if (f.stun > 0 || on(f, fCrumpled) || f.break_frames > 0 || f.pending_throw_hit >= 0) return false;
    if (f.posture != kStanding && f.posture != kCrouching) return false;
    if (f.move >= 0) return f.action_frame >= move_at(m, p, f.move).total_frames;
    return f.action_frame >= action_length(f.universal, *m.cfg);
}

// The move branch of legal (full_combat_core.hpp:380-441) for a move with these flags,
// required posture and stance, and heat cost; the round is still running. `can()` gives
// can_act(m, s, p) when the move needs it (move_allowed computes it there; a caller checking
// many candidates of one state passes the value it took once).
template <class Can>
T8B_HD bool move_allowed_with(const Match& m, const Fight& s, int p, Can can, uint64_t flags, uint8_t required_posture,
                              int32_t required_stance, bool heat_cost) {
    const Fighter& f = s.f[p];
    const Cfg& c = *m.cfg;
    const auto need = [flags](uint64_t bit) { return (flags & bit) != 0ull; };
    if (need(kReactive)) return false;
    if (need(kRequiresSidestep)) {
        const bool stepping = f.move < 0 && f.action_frame >= 1 && f.stun == 0 && !on(f, fCrumpled) &&
            f.break_frames == 0 && f.pending_throw_hit < 0 &&
            (f.universal == kSidestepLeft || f.universal == kSidestepRight);
        if (!stepping) return false;
    } else if (!can()) {
        return false;
    }
    const Fighter& o = s.f[1 - p];
    if (need(kRequiresBackTurned) != on(f, fBackTurned)) return false;
    if (need(kRequiresOpponentBackTurned) && !on(o, fBackTurned)) return false;
    if (need(kRequiresBackToWall)) {
        const double wall = o.x >= f.x ? s.left_wall : s.right_wall;
        if (mag(f.x - wall) > c.back_to_wall_distance) return false;
    }
    if (need(kRequiresOpponentLeft) || need(kRequiresOpponentRight)) {
        const double toward = f.x >= o.x ? 1.0 : -1.0;
        const double gap = hi(mag(f.x - o.x), 1e-9);
        const double side = (f.axis - o.axis) * toward / gap;
        if (need(kRequiresOpponentLeft) && side > -c.side_exposure_ratio) return false;
        if (need(kRequiresOpponentRight) && side < c.side_exposure_ratio) return false;
    }
    const bool heat = on(f, fHeat);
    return required_posture == f.posture && (required_stance < 0 || required_stance == f.stance) &&
        (!need(kRequiresHeat) || heat) && (!need(kConsumesHeat) || heat) && (!heat_cost || heat) &&
        (!need(kEngagesHeat) || (on(f, fHeatAvailable) && !heat)) &&
        (!(need(kRequiresRage) || need(kConsumesRage)) || on(f, fRage));
}

T8B_HD bool move_allowed(const Match& m, const Fight& s, int p, uint64_t flags, uint8_t required_posture,
                         int32_t required_stance, bool heat_cost) {
    return move_allowed_with(m, s, p, [&] { return can_act(m, s, p); }, flags, required_posture, required_stance,
                             heat_cost);
}
T8B_HD bool move_allowed_given(const Match& m, const Fight& s, int p, bool can, uint64_t flags, uint8_t required_posture,
                               int32_t required_stance, bool heat_cost) {
    return move_allowed_with(m, s, p, [can] { return can; }, flags, required_posture, required_stance, heat_cost);
}

// What move_allowed derives from the fight rather than from the move, computed once for a
// fighter whose candidates are all checked against the same state (the legal-move masks).
struct MoveContext {
    bool can, stepping, back_turned, opponent_back_turned, near_wall, left_ok, right_ok, heat, heat_available, rage;
    uint8_t posture;
    int32_t stance;
};
T8B_HD MoveContext move_context(const Match& m, const Fight& s, int p) {
    const Fighter& f = s.f[p];
    const Fighter& o = s.f[1 - p];
    const Cfg& c = *m.cfg;
    MoveContext x;
    x.stepping = f.move < 0 && f.action_frame >= 1 && f.stun == 0 && !on(f, fCrumpled) && f.break_frames == 0 &&
        f.pending_throw_hit < 0 && (f.universal == kSidestepLeft || f.universal == kSidestepRight);
    x.can = can_act(m, s, p);
    x.back_turned = on(f, fBackTurned);
    x.opponent_back_turned = on(o, fBackTurned);
    const double wall = o.x >= f.x ? s.left_wall : s.right_wall;
    x.near_wall = !(mag(f.x - wall) > c.back_to_wall_distance);
    const double toward = f.x >= o.x ? 1.0 : -1.0;
    const double gap = hi(mag(f.x - o.x), 1e-9);
    const double side = (f.axis - o.axis) * toward / gap;
    x.left_ok = !(side > -c.side_exposure_ratio);
    x.right_ok = !(side < c.side_exposure_ratio);
    x.heat = on(f, fHeat);
    x.heat_available = on(f, fHeatAvailable);
    x.rage = on(f, fRage);
    x.posture = f.posture;
    x.stance = f.stance;
    return x;
}
// move_allowed with the fight's side taken from a MoveContext (the same decisions in the same
// order; the round is still running).
T8B_HD bool context_allows(const MoveContext& x, uint64_t flags, uint8_t required_posture, int32_t required_stance,
                           bool heat_cost) {
    const auto need = [flags](uint64_t bit) { return (flags & bit) != 0ull; };
    if (need(kReactive)) return false;
    if (need(kRequiresSidestep) ? !x.stepping : !x.can) return false;
    if (need(kRequiresBackTurned) != x.back_turned) return false;
    if (need(kRequiresOpponentBackTurned) && !x.opponent_back_turned) return false;
    if (need(kRequiresBackToWall) && !x.near_wall) return false;
    if (need(kRequiresOpponentLeft) && !x.left_ok) return false;
    if (need(kRequiresOpponentRight) && !x.right_ok) return false;
    return required_posture == x.posture && (required_stance < 0 || required_stance == x.stance) &&
        (!need(kRequiresHeat) || x.heat) && (!need(kConsumesHeat) || x.heat) && (!heat_cost || x.heat) &&
        (!need(kEngagesHeat) || (x.heat_available && !x.heat)) &&
        (!(need(kRequiresRage) || need(kConsumesRage)) || x.rage);
}

// legal (full_combat_core.hpp:380-441)
T8B_HD bool input_ok(const Match& m, const Fight& s, int p, const Input& in) {
    if (s.winner >= 0) return false;
    const Fighter& f = s.f[p];
    const Cfg& c = *m.cfg;
    if (in.move >= 0) {
        if (in.move >= m.side[p]->move_count) return false;
        const DMove& mv = move_at(m, p, in.move);
        return move_allowed(m, s, p, mv.flags, mv.required_posture, mv.required_stance, mv.heat_cost_frames != 0);
    }
    switch (in.universal) {
        case kWakeupStand:
        case kWakeupRoll: return f.posture == kGrounded && f.grounded_elapsed >= c.knockdown_frames;
        case kTechRoll:
            return f.posture == kGrounded && on(f, fTechable) && f.grounded_elapsed < c.tech_window_frames;
        case kThrowBreak:
        case kThrowBreak1:
        case kThrowBreak2: return f.break_frames > 0 && !on(f, fBreakAttempted);
        case kHeatDash: {
            if (f.move < 0 || !on(f, fHeat) || f.dash_from == kNoContactFrom) return false;
            const DMove& mv = move_at(m, p, f.move);
            return f.dash_from == kBlocked ? has(mv, kHasHeatDashBlock) : has(mv, kHasHeatDashHit);
        }
        default: return can_act(m, s, p);
    }
}

// deal_damage (full_combat_core.hpp:443-458)
T8B_HD void hurt(const Match& m, Fight& s, int target, double damage, bool recoverable, bool can_ko, Events& e) {
    Fighter& f = s.f[target];
    const Cfg& c = *m.cfg;
    if (!can_ko) damage = lo(damage, hi(0.0, f.health - 1.0));
    damage = hi(0.0, damage);
    f.health -= damage;
    if (recoverable) f.recoverable += damage;
    f.recoverable = clampd(f.recoverable, 0.0, c.max_health - f.health);
    if (f.health > 0.0 && on(f, fRageAvailable) && f.health <= c.rage_health_fraction * c.max_health) {
        f.flags = (f.flags | fRage) & ~fRageAvailable;
        e.rage_activated[target] = 1;
    }
}

// regain (full_combat_core.hpp:460-465)
T8B_HD void restore(Fighter& f, double recoverable, double health, double max_health) {
    const double back = lo(hi(0.0, recoverable), f.recoverable);
    f.recoverable -= back;
    f.health = lo(max_health, f.health + back + hi(0.0, health));
    f.recoverable = lo(f.recoverable, max_health - f.health);
}

// activate_heat (full_combat_core.hpp:467-474)
T8B_HD void heat_on(const Match& m, Fight& s, int p, Events& e) {
    Fighter& f = s.f[p];
    if (!on(f, fHeatAvailable) || on(f, fHeat)) return;
    f.flags = (f.flags | fHeat) & ~fHeatAvailable;
    f.heat_frames = m.cfg->heat_duration_frames;
    e.heat_activated[p] = 1;
}

// break_throw (full_combat_core.hpp:476-497)
T8B_HD void throw_escape(const Match& m, Fight& s, int thrower, Events& e) {
    Fighter& a = s.f[thrower];
    Fighter& d = s.f[1 - thrower];
    const Cfg& c = *m.cfg;
    const int hit = a.pending_throw_hit;
    const bool switch_sides = a.move >= 0 && has(move_at(m, thrower, a.move), kSideSwitchOnBreak);
    add_contact(e, thrower, hit, kThrowBroken, 0.0);
    for (int k = 0; k < 2; ++k) {
        Fighter& f = k == 0 ? a : d;
        f.move = -1;
        f.universal = kIdle;
        f.action_frame = action_length(kIdle, c);
        f.stun = c.throw_break_recovery;
        f.flags |= fInBlockstun;
        f.dash_from = kNoContactFrom;
    }
    a.pending_throw_hit = -1;
    d.break_frames = 0;
    if (switch_sides) swapd(a.x, d.x);
    const double dir = d.x >= a.x ? 1.0 : -1.0;
    a.x = hi(s.left_wall, lo(s.right_wall, a.x - dir * 0.2));
    d.x = hi(s.left_wall, lo(s.right_wall, d.x + dir * 0.2));
}

// release_throw (full_combat_core.hpp:499-506)
T8B_HD void let_go(Fight& s, int thrower) {
    Fighter& f = s.f[thrower];
    if (f.pending_throw_hit < 0) return;
    f.pending_throw_hit = -1;
    Fighter& held = s.f[1 - thrower];
    held.break_frames = 0;
    held.flags &= ~fBreakAttempted;
}

T8B_HD void heat_spend(Fighter& f, int frames) {
    f.heat_frames -= frames;
    if (f.heat_frames <= 0) {
        f.flags &= ~fHeat;
        f.heat_frames = 0;
    }
}

// apply_parry_outcome (full_combat_core.hpp:508-568)
T8B_HD void play_parry_outcome(const Match& m, Fight& s, int parrier_p, int outcome, int attacker_p, Events& e) {
    Fighter& parrier = s.f[parrier_p];
    Fighter& att = s.f[attacker_p];
    const Cfg& c = *m.cfg;
    const DMove& mv = move_at(m, parrier_p, outcome);
    double total = 0.0;
    for (int k = 0; k < mv.hit_count; ++k) total += hit_at(m, parrier_p, mv, k).damage;
    const bool recoverable_only = has(mv, kRecoverableOnly);
    hurt(m, s, attacker_p, total, recoverable_only, !recoverable_only, e);
    let_go(s, attacker_p);
    att.move = -1;
    att.universal = kIdle;
    att.stance = -1;
    att.dash_from = kNoContactFrom;
    att.flags &= ~fInBlockstun;
    const int frames = mv.recovery > 0 ? mv.recovery : c.parry_outcome_frames;
    if (mv.hit_effect == kLaunch) {
        att.stun = 0;
        att.posture = kAirborne;
        att.posture_frames = has(mv, kHasLaunchAirFrames) ? mv.launch_air_frames
            : (frames + mv.hit_advantage > 0 ? frames + mv.hit_advantage : c.launch_air_frames);
        att.combo_hits = 1;
    } else if (mv.hit_effect == kKnockdown || mv.hit_effect == kCrumple) {
        att.stun = 0;
        att.posture = kGrounded;
        att.grounded_elapsed = 0;
        att.flags &= ~fTechable;
    } else if (mv.hit_effect == kStun) {
        att.stun = ihi(0, frames + mv.hit_advantage);
    }
    let_go(s, parrier_p);
    parrier.move = outcome;
    parrier.universal = kIdle;
    parrier.stance = -1;
    parrier.stun = 0;
    parrier.flags &= ~fInBlockstun;
    parrier.dash_from = kNoContactFrom;
    parrier.action_frame = ihi(0, mv.total_frames - frames);
    parrier.hits_landed = mv.hit_count >= 32 ? ~0u : (1u << static_cast<unsigned>(mv.hit_count)) - 1u;
    parrier.flags = (parrier.flags | fMoveHit | fResourceGained) & ~fMoveBlocked;
    if (mv.heat_cost_frames > 0 && on(parrier, fHeat)) heat_spend(parrier, mv.heat_cost_frames);
    restore(parrier, mv.restore_recoverable_hit, mv.restore_health_hit, c.max_health);
    gain(m, s, parrier_p, mv.resource_gain_start + mv.resource_gain_hit);
    if (has(mv, kRemovesRecoverable)) att.recoverable = 0.0;
}

// push_defender (full_combat_core.hpp:570-580)
T8B_HD void push_away(const Fight& s, Fighter& a, Fighter& d, double distance) {
    const double dir = d.x >= a.x ? 1.0 : -1.0;
    d.x += dir * distance;
    const double wall = dir > 0.0 ? s.right_wall : s.left_wall;
    const double over = dir > 0.0 ? d.x - wall : wall - d.x;
    if (over > 0.0) {
        d.x = wall;
        a.x -= dir * over;
    }
}

// enable_heat_dash (full_combat_core.hpp:582-593)
T8B_HD void after_contact_heat(const Match& m, Fight& s, int ap, const DMove& mv, bool last, int from, Events& e) {
    Fighter& a = s.f[ap];
    if (!last) return;
    if (has(mv, kHeatEngager) && on(a, fHeatAvailable) && !on(a, fHeat)) {
        heat_on(m, s, ap, e);
        gain(m, s, ap, mv.resource_gain_heat_activation);
    }
    if (on(a, fHeat) && (has(mv, kHasHeatDashBlock) || has(mv, kHasHeatDashHit))) a.dash_from = static_cast<int8_t>(from);
}

// scaled_damage (full_combat_core.hpp:595-604)
T8B_HD double scale_damage(const Cfg& c, const Fighter& a, const Fighter& d, double damage, bool counter) {
    damage *= counter ? c.counter_hit_damage_scale : 1.0;
    if (on(a, fRage)) damage *= c.rage_damage_scale;
    if (d.combo_hits > 0) damage *= hi(c.combo_scale_floor, 1.0 - c.combo_scale_step * d.combo_hits);
    if (on(d, fWallScaled)) damage *= c.wall_combo_scale;
    return damage;
}

T8B_HD double facing(const Fight& s, int p) {
    const double own = s.f[p].x, other = s.f[1 - p].x;
    if (other == own) return p == 0 ? 1.0 : -1.0;
    return other > own ? 1.0 : -1.0;
}

// apply_contact, parry branch (full_combat_core.hpp:629-661)
T8B_HD void resolve_parry(const Match& m, Fight& s, int ap, const DHit& hit, int defense_move, Events& e, double& dealt) {
    const Cfg& c = *m.cfg;
    const int dp = 1 - ap;
    Fighter& a = s.f[ap];
    const Fighter& d = s.f[dp];
    const int slot = level_slot(hit.level);
    int outcome = -1;
    if (defense_move >= 0) {
        const DMove& def = move_at(m, dp, defense_move);
        const bool heat_parry = on(d, fMoveInHeat) && (def.heat_parry_levels & level_bits(hit.level)) &&
            in_window(m, dp, def, wHeatParry, d.action_frame);
        outcome = heat_parry ? def.heat_parry_outcome : def.parry_outcomes[slot];
        if (outcome == kNoOutcome && def.result_stance >= 0 && def.result_stance < m.side[dp]->stance_count) {
            outcome = m.side[dp]->stances[def.result_stance].parry_outcomes[slot];
        }
    } else if (const DStance* rule = stance_of(m, s, dp)) {
        outcome = rule->parry_outcomes[slot];
    }
    if (outcome >= 0) {
        const double before = a.health;
        play_parry_outcome(m, s, dp, outcome, ap, e);
        dealt = before - a.health;
        return;
    }
    let_go(s, ap);
    a.stance = -1;
    a.move = -1;
    a.universal = kIdle;
    a.action_frame = action_length(kIdle, c);
    a.stun = c.parry_stun_frames;
    a.flags &= ~fInBlockstun;
    a.dash_from = kNoContactFrom;
}

// apply_contact, clean-hit branch (full_combat_core.hpp:701-855)
T8B_HD void resolve_hit(const Match& m, Fight& s, int ap, const DMove& mv, const DHit& hit, int hit_index, int contact,
                        int defense_move, int remaining, bool last, Events& e, double& dealt) {
    const Cfg& c = *m.cfg;
    const int dp = 1 - ap;
    Fighter& a = s.f[ap];
    Fighter& d = s.f[dp];
    const bool counter = contact == kCounterHit;
    const bool juggle = d.posture == kAirborne || d.posture == kWallSplat;
    const bool was_back_turned = on(d, fBackTurned);
    const uint8_t was_posture = d.posture;
    double base = hit.damage + (on(a, fInstalled) && last ? mv.install_damage_bonus : 0.0);
    if (last && has(mv, kHasRageArtMax)) {
        double listed = 0.0;
        for (int k = 0; k < mv.hit_count; ++k) listed += hit_at(m, ap, mv, k).damage;
        const double missing = 1.0 - a.health / c.max_health;
        base += hi(0.0, mv.rage_art_max_damage - listed) * clampd(missing, 0.0, 1.0);
    }
    if (on(a, fMoveBoosted)) base *= c.ki_charge_damage_scale;
    const double damage = scale_damage(c, a, d, base, counter);
    if (contact == kArmored) {
        const bool recoverable = defense_move >= 0 && has(move_at(m, dp, defense_move), kArmorDamageRecoverable);
        hurt(m, s, dp, damage, recoverable, true, e);
        dealt = damage;
        return;
    }
    {
        const bool can_ko = !has(mv, kCannotKo) && !has(mv, kRecoverableOnly);
        const double part = has(mv, kRecoverableOnly) ? damage : last ? lo(damage, mv.recoverable_damage) : 0.0;
        hurt(m, s, dp, damage - part, false, can_ko, e);
        hurt(m, s, dp, part, true, false, e);
    }
    dealt = damage;
    if (has(mv, kRemovesRecoverable)) d.recoverable = 0.0;
    a.flags |= fMoveHit;
    if (last && !on(a, fResourceGained)) {
        a.flags |= fResourceGained;
        gain(m, s, ap, juggle ? mv.resource_gain_airborne_hit : mv.resource_gain_hit);
    }
    restore(a, c.recoverable_regain_hit * damage + (last ? mv.restore_recoverable_hit : 0.0),
            last ? mv.restore_health_hit : 0.0, c.max_health);

    let_go(s, dp);
    d.stance = -1;
    d.move = -1;
    d.universal = kIdle;
    d.action_frame = 0;
    d.flags &= ~(fInBlockstun | fBackTurned);
    d.dash_from = kNoContactFrom;
    const bool bt_hit = was_back_turned && has(mv, kHasBackTurnedHitAdvantage);
    const uint8_t effect = bt_hit ? mv.back_turned_hit_effect
        : counter && has(mv, kHasCounterHitEffect) ? mv.counter_hit_effect : mv.hit_effect;
    const int advantage = bt_hit ? mv.back_turned_hit_advantage
        : counter && has(mv, kHasCounterHitAdvantage) ? mv.counter_hit_advantage : mv.hit_advantage;
    const bool trigger = mv.attack_throw == kAttackThrowOnHit || (mv.attack_throw == kAttackThrowOnCounterHit && counter);
    const bool front = !has(mv, kAttackThrowFrontOnly) || !was_back_turned;
    const bool posture_ok = was_posture == kAirborne ? has(mv, kAttackThrowAirborne)
        : !has(mv, kAttackThrowStandingOnly) || was_posture == kStanding;
    if (last && trigger && front && posture_ok && !bt_hit) {
        const double extra = scale_damage(c, a, d, mv.attack_throw_damage, false);
        hurt(m, s, dp, extra, false, !has(mv, kCannotKo), e);
        dealt += extra;
    }
    const bool thrown = hit.level == kThrow;
    if (juggle && (hit.flags & kSpike)) {
        ++d.combo_hits;
        d.posture = kGrounded;
        d.grounded_elapsed = 0;
        d.flags &= ~fTechable;
    } else if (juggle) {
        ++d.combo_hits;
        if (d.posture == kAirborne) {
            const int window = ihi(0, c.juggle_window_frames - c.juggle_window_decay * (d.combo_hits - 1));
            d.posture_frames = ihi(d.posture_frames, remaining + window);
            if ((hit.flags & kTornado) && !on(d, fTornadoUsed)) {
                d.flags |= fTornadoUsed;
                d.posture_frames += c.tornado_extra_frames;
            }
        } else {
            d.posture_frames = ihi(d.posture_frames, remaining + c.wall_splat_frames);
        }
    } else if (d.posture == kGrounded) {
        ++d.combo_hits;
        d.grounded_elapsed = 0;
    } else if (last && effect == kLaunch) {
        d.posture = kAirborne;
        d.posture_frames = has(mv, kHasLaunchAirFrames) ? mv.launch_air_frames
            : (remaining + advantage > 0 ? remaining + advantage : c.launch_air_frames);
        d.combo_hits = 1;
        d.stun = 0;
    } else if (last && effect == kKnockdown) {
        d.posture = kGrounded;
        d.grounded_elapsed = 0;
        put(d, fTechable, !thrown);
        d.stun = 0;
    } else if (last && effect == kCrumple) {
        d.stun = c.crumple_frames;
        d.flags |= fCrumpled;
    } else {
        d.stun = ihi(0, remaining + advantage);
        if (d.posture == kCrouching) d.posture = kStanding;
    }
    after_contact_heat(m, s, ap, mv, last, contact, e);
    if (last && has(mv, kSideSwitchOnHit)) swapd(a.x, d.x);
    push_away(s, a, d, mv.pushback_hit);

    // Walls and stage transitions on the side the defender was driven toward.
    const bool right = d.x >= a.x;
    const double wall = right ? s.right_wall : s.left_wall;
    const bool at_wall = mag(d.x - wall) < 1e-9;
    const uint32_t breakable_bit = right ? sRightBreakable : sLeftBreakable;
    const uint32_t balcony_bit = right ? sRightBalcony : sLeftBalcony;
    const double extension = right ? c.wall_break_extension : -c.wall_break_extension;
    bool airborne_again = false;
    if (at_wall && (hit.flags & kBalconyBreakHit) && (s.stage & balcony_bit)) {
        s.stage &= ~balcony_bit;
        ++s.level;
        if (right) s.right_wall += extension; else s.left_wall += extension;
        d.x += (right ? 1.0 : -1.0) * 1.0;
        airborne_again = true;
        add_transition(e, kBalconyBreak);
    } else if (at_wall && (hit.flags & kWallBreakHit) && (s.stage & breakable_bit)) {
        s.stage &= ~breakable_bit;
        if (right) s.right_wall += extension; else s.left_wall += extension;
        airborne_again = true;
        add_transition(e, kWallBreak);
    } else if (at_wall && ((hit.flags & kWallSplatHit) || juggle) && !on(d, fWallSplatUsed)) {
        d.posture = kWallSplat;
        d.posture_frames = remaining + c.wall_splat_frames;
        d.flags |= fWallSplatUsed | fWallScaled;
        d.stun = 0;
        d.combo_hits = ihi(1, d.combo_hits);
    } else if ((hit.flags & kFloorBreakHit) && (s.stage & sFloorBreakable) && (juggle || d.posture == kGrounded)) {
        s.stage &= ~sFloorBreakable;
        ++s.level;
        airborne_again = true;
        add_transition(e, kFloorBreak);
    }
    if (airborne_again) {
        d.posture = kAirborne;
        d.posture_frames = c.stage_break_air_frames;
        d.stun = 0;
        d.combo_hits = ihi(1, d.combo_hits);
    }
    (void)hit_index;
}

// apply_contact (full_combat_core.hpp:606-858)
T8B_HD void resolve(const Match& m, Fight& s, int ap, int move_index, int defense_move, int hit_index, int contact,
                    int elapsed, Events& e) {
    const Cfg& c = *m.cfg;
    const int dp = 1 - ap;
    Fighter& a = s.f[ap];
    Fighter& d = s.f[dp];
    const DMove& mv = move_at(m, ap, move_index);
    const DHit& hit = hit_at(m, ap, mv, hit_index);
    const bool last = hit_index + 1 == mv.hit_count;
    double dealt = 0.0;
    const int remaining = ihi(0, mv.total_frames - hit.first_active_frame - elapsed);
    switch (contact) {
        case kParried: resolve_parry(m, s, ap, hit, defense_move, e, dealt); break;
        case kReversed: {
            const double damage = defense_move >= 0 ? move_at(m, dp, defense_move).reversal_damage : 0.0;
            hurt(m, s, ap, damage, false, true, e);
            dealt = damage;
            let_go(s, ap);
            a.move = -1;
            a.universal = kIdle;
            a.stance = -1;
            a.stun = 0;
            a.dash_from = kNoContactFrom;
            a.posture = kGrounded;
            a.grounded_elapsed = 0;
            a.flags &= ~fTechable;
            d.move = -1;
            d.universal = kIdle;
            d.action_frame = action_length(kIdle, c);
            d.stun = c.reversal_recovery;
            d.flags |= fInBlockstun;
            break;
        }
        case kBlocked: {
            d.stun = ihi(0, remaining + mv.block_advantage);
            put(d, fInBlockstun, d.stun > 0);
            a.flags |= fMoveBlocked;
            if (last && !on(a, fResourceGained)) {
                a.flags |= fResourceGained;
                gain(m, s, ap, mv.resource_gain_block);
            }
            const double chip = on(a, fInstalled) && last && has(mv, kHasInstallChip) ? mv.install_chip_damage
                : on(a, fHeat) && (hit.flags & kHasHeatChip) ? hit.heat_chip_damage : hit.chip_damage;
            if (chip > 0.0) hurt(m, s, dp, chip, true, false, e);
            dealt = chip;
            restore(a, c.recoverable_regain_block * hit.damage + (last ? mv.restore_recoverable_block : 0.0), 0.0,
                    c.max_health);
            after_contact_heat(m, s, ap, mv, last, kBlocked, e);
            push_away(s, a, d, mv.pushback_block);
            break;
        }
        case kArmored:
        case kHit:
        case kCounterHit:
            resolve_hit(m, s, ap, mv, hit, hit_index, contact, defense_move, remaining, last, e, dealt);
            break;
        default: break;  // evaded, crushed, broken, held: no effect here
    }
    add_contact(e, ap, hit_index, contact, dealt);
}

// ------------------------------------------------------------------ the frame step
struct Pending {
    int attacker, move_index, defense_move, hit_index, contact;
};

// Phase 1 for one fighter whose input was accepted (full_combat_core.hpp:898-1016).
T8B_HD void start_action(const Match& m, Fight& s, int p, const Input& in, Events& e) {
    const Cfg& c = *m.cfg;
    Fighter& f = s.f[p];
    Fighter& o = s.f[1 - p];
    if (in.move < 0 && is_break_input(in.universal)) {
        f.flags |= fBreakAttempted;
        if (f.break_frames > 0 && o.move >= 0 && o.pending_throw_hit >= 0) {
            const DMove& tm = move_at(m, 1 - p, o.move);
            if (escapes(hit_at(m, 1 - p, tm, o.pending_throw_hit).throw_break, in.universal)) {
                throw_escape(m, s, 1 - p, e);
            }
        }
        return;
    }
    if (in.move < 0 && in.universal == kHeatDash) {
        const DMove& mv = move_at(m, p, f.move);
        const int frames = c.heat_dash_frames;
        if (f.dash_from == kBlocked) {
            o.stun = ihi(0, frames + mv.heat_dash_block_advantage);
            put(o, fInBlockstun, o.stun > 0);
        } else {
            const int advantage = frames + mv.heat_dash_hit_advantage;
            o.flags &= ~(fInBlockstun | fCrumpled);
            o.posture = kStanding;
            o.posture_frames = 0;
            if (mv.heat_dash_hit_effect == kLaunch) {
                o.posture = kAirborne;
                o.posture_frames = ihi(1, advantage);
                o.combo_hits = ihi(1, o.combo_hits);
                o.stun = 0;
            } else if (mv.heat_dash_hit_effect == kKnockdown || mv.heat_dash_hit_effect == kCrumple) {
                o.stun = ihi(1, advantage);
                o.flags |= fCrumpled;
            } else if (mv.heat_dash_hit_effect == kStun) {
                o.stun = ihi(0, advantage);
            }
        }
        let_go(s, p);
        f.move = -1;
        f.universal = kHeatDash;
        f.flags &= ~fHeat;
        f.heat_frames = 0;
        f.dash_from = kNoContactFrom;
        f.action_frame = 0;
        f.hits_landed = 0;
        return;
    }
    f.dash_from = kNoContactFrom;
    if (in.move >= 0) {
        const DMove& mv = move_at(m, p, in.move);
        f.move = in.move;
        f.universal = kIdle;
        f.stance = -1;
        if (has(mv, kEngagesHeat) && on(f, fHeatAvailable) && !on(f, fHeat)) {
            heat_on(m, s, p, e);
            gain(m, s, p, mv.resource_gain_heat_activation);
        }
        if (mv.heat_cost_frames > 0) heat_spend(f, mv.heat_cost_frames);
        f.flags &= ~(fMoveHit | fMoveBlocked | fResourceGained | fBackTurned);
        put(f, fMoveInHeat, on(f, fHeat));
        const bool ki = has(mv, kKiCharge);
        put(f, fMoveBoosted, on(f, fKiBoost) && !ki);
        if (!ki) f.flags &= ~fKiBoost;
        if (ki) {
            f.ki_frames = c.ki_charge_frames;
            f.flags |= fKiBoost;
        }
        gain(m, s, p, mv.resource_gain_start);
        if (has(mv, kConsumesHeat)) {
            f.flags &= ~fHeat;
            f.heat_frames = 0;
        }
        if (has(mv, kConsumesRage)) f.flags &= ~fRage;
        if (mv.self_damage > 0.0 && !(has(mv, kSelfDamageWithoutHeatOnly) && on(f, fHeat))) {
            hurt(m, s, p, mv.self_damage - mv.self_recoverable, false, false, e);
            hurt(m, s, p, mv.self_recoverable, true, false, e);
        }
    } else if (in.universal == kWakeupStand) {
        f.posture = kWakeup;
        f.posture_frames = c.wakeup_stand_frames;
        f.move = -1;
        f.universal = kIdle;
    } else if (in.universal == kWakeupRoll || in.universal == kTechRoll) {
        const bool tech = in.universal == kTechRoll;
        f.posture = kWakeup;
        f.posture_frames = tech ? c.tech_roll_frames : c.wakeup_roll_frames;
        f.x -= facing(s, p) * (tech ? 0.5 : 1.0) * c.wakeup_roll_distance;
        f.move = -1;
        f.universal = kIdle;
    } else {
        f.move = -1;
        f.universal = static_cast<uint8_t>(in.universal);
        if (in.universal != kIdle) {
            f.stance = -1;
            f.flags &= ~fBackTurned;
        }
        f.posture = in.universal == kCrouch ? kCrouching : kStanding;
    }
    f.action_frame = 0;
    f.hits_landed = 0;
}

// Phase 2 for one fighter (full_combat_core.hpp:1024-1135).
T8B_HD void advance(const Match& m, Fight& s, int p) {
    const Cfg& c = *m.cfg;
    Fighter& f = s.f[p];
    const double forward = facing(s, p);
    if (f.move >= 0) {
        const DMove& mv = move_at(m, p, f.move);
        const bool holding = f.pending_throw_hit >= 0;
        if (!holding || f.action_frame < mv.total_frames) ++f.action_frame;
        const int approach = mv.approach_frames;
        if (approach > 0 && f.action_frame <= approach) f.x += forward * mv.travel / approach;
        if (f.action_frame >= mv.total_frames && !holding) {
            f.stance = on(f, fMoveHit) && mv.result_stance_on_hit >= 0 ? mv.result_stance_on_hit
                : on(f, fMoveBlocked) && mv.result_stance_on_block >= 0 ? mv.result_stance_on_block
                : mv.result_stance;
            f.stance_frames = 0;
            put(f, fBackTurned, has(mv, kResultBackTurned));
            f.move = -1;
            f.dash_from = kNoContactFrom;
            f.action_frame = action_length(kIdle, c);
            if (has(mv, kResultCrouching)) {
                f.posture = kCrouching;
                f.universal = kCrouch;
            } else if (f.posture == kCrouching && f.stance < 0) {
                f.posture = kStanding;
            }
        }
    } else if (f.posture == kStanding || f.posture == kCrouching) {
        ++f.action_frame;
        const DStance* rule = stance_of(m, s, p);
        if (rule && f.stun == 0) {
            ++f.stance_frames;
            if (rule->pulse_interval_frames > 0 && f.stance_frames % rule->pulse_interval_frames == 0) {
                restore(f, rule->pulse_recoverable, 0.0, c.max_health);
                gain(m, s, p, rule->pulse_resource);
            }
            if (rule->has_max_frames && f.stance_frames >= rule->max_frames) {
                f.stance = -1;
                f.stance_frames = 0;
            }
        }
        switch (f.universal) {
            case kWalkForward: f.x += forward * c.walk_speed; break;
            case kWalkBack: f.x -= forward * c.walk_speed; break;
            case kDashForward:
                if (f.action_frame <= c.dash_frames) f.x += forward * c.dash_distance / c.dash_frames;
                break;
            case kHeatDash:
                if (f.action_frame <= c.heat_dash_frames) f.x += forward * c.heat_dash_distance / c.heat_dash_frames;
                break;
            case kBackdash:
                if (f.action_frame <= c.backdash_frames) f.x -= forward * c.backdash_distance / c.backdash_frames;
                break;
            case kSidestepLeft:
            case kSidestepRight:
                if (f.action_frame <= c.sidestep_frames) {
                    const double side = f.universal == kSidestepLeft ? -1.0 : 1.0;
                    f.axis += side * forward * c.sidestep_distance / c.sidestep_frames;
                }
                break;
            default: break;
        }
    }
    if (f.stun > 0 && --f.stun == 0) f.flags &= ~fInBlockstun;
    if (f.stun == 0 && on(f, fCrumpled)) {
        f.flags &= ~(fCrumpled | fTechable);
        f.posture = kGrounded;
        f.grounded_elapsed = 0;
    }
    switch (f.posture) {
        case kAirborne:
            if (--f.posture_frames <= 0) {
                f.posture = kGrounded;
                f.grounded_elapsed = 0;
                put(f, fTechable, !on(f, fTornadoUsed));
            }
            break;
        case kWallSplat:
            if (--f.posture_frames <= 0) {
                f.posture = kGrounded;
                f.grounded_elapsed = 0;
                f.flags &= ~fTechable;
            }
            break;
        case kGrounded:
            ++f.grounded_elapsed;
            if (f.grounded_elapsed >= 4 * c.knockdown_frames) {
                f.posture = kWakeup;
                f.posture_frames = c.wakeup_stand_frames;
            }
            break;
        case kWakeup:
            if (--f.posture_frames <= 0) {
                f.posture = kStanding;
                f.combo_hits = 0;
                f.flags &= ~(fTornadoUsed | fWallSplatUsed | fWallScaled);
                f.action_frame = action_length(kIdle, c);
                f.universal = kIdle;
            }
            break;
        default: break;
    }
}

// Phase 4 for one attacker: the contact its move makes this frame, if any (full_combat_core.hpp:1172-1246).
T8B_HD bool find_contact(const Match& m, const Fight& s, int ap, Pending& out) {
    const Fighter& own = s.f[ap];
    const Fighter& tgt = s.f[1 - ap];
    if (own.move < 0 || own.pending_throw_hit >= 0 || tgt.break_frames > 0) return false;
    const DMove& mv = move_at(m, ap, own.move);
    const DMove* def = tgt.move >= 0 ? &move_at(m, 1 - ap, tgt.move) : nullptr;
    const int dframe = tgt.action_frame;
    const DStance* trule = tgt.move >= 0 ? nullptr : stance_of(m, s, 1 - ap);
    const int dp = 1 - ap;
    for (int k = 0; k < mv.hit_count; ++k) {
        const DHit& hit = hit_at(m, ap, mv, k);
        if ((own.hits_landed >> static_cast<unsigned>(k)) & 1u) continue;
        if (own.action_frame < hit.first_active_frame || own.action_frame >= hit.first_active_frame + hit.active_frames)
            continue;
        const double reach = on(own, fInstalled) && has(mv, kHasInstallReach) ? mv.install_reach : hit.reach;
        if (mag(tgt.x - own.x) > reach) continue;
        const double lateral = (tgt.axis - own.axis) * facing(s, ap);
        if (!(hit.flags & kHoming) && (lateral < -hit.tracking_left || lateral > hit.tracking_right)) continue;
        const bool airborne = tgt.posture == kAirborne || (def && in_window(m, dp, *def, wAirborne, dframe));
        if (tgt.posture == kGrounded && !((hit.flags & kGroundHit) || is_low(hit.level))) continue;
        if (tgt.posture == kCrouching && (hit.level == kHigh || hit.level == kThrow)) continue;
        if (airborne && hit.level == kThrow) continue;

        out.attacker = ap;
        out.move_index = own.move;
        out.defense_move = tgt.move;
        out.hit_index = k;
        const bool high_mid = hit.level != kThrow && !is_low(hit.level);
        const uint8_t bits = level_bits(hit.level);
        if (def && in_window(m, dp, *def, wInvincible, dframe)) {
            out.contact = kEvaded;
        } else if (def && (((hit.level == kHigh || hit.level == kThrow) && in_window(m, dp, *def, wHighCrush, dframe)) ||
                           (is_low(hit.level) && in_window(m, dp, *def, wLowCrush, dframe)))) {
            out.contact = kCrushed;
        } else if (def && high_mid && !(hit.flags & kReversalBreak) && in_window(m, dp, *def, wReversal, dframe)) {
            out.contact = kReversed;
        } else if (def && !(hit.flags & kUnparryable) &&
                   (((def->parry_levels & bits) && in_window(m, dp, *def, wParry, dframe)) ||
                    (on(tgt, fMoveInHeat) && (def->heat_parry_levels & bits) &&
                     in_window(m, dp, *def, wHeatParry, dframe)))) {
            out.contact = kParried;
        } else if (!def && !(hit.flags & kUnparryable) && trule && tgt.stun == 0 && tgt.posture == kStanding &&
                   (trule->auto_parry & bits)) {
            out.contact = kParried;
        } else if (def && hit.level != kThrow &&
                   (in_window(m, dp, *def, wArmor, dframe) || (high_mid && in_window(m, dp, *def, wPowerCrush, dframe)))) {
            out.contact = kArmored;
        } else {
            const bool guard_ok = (!trule || trule->can_guard) && !on(tgt, fBackTurned) && tgt.ki_frames == 0;
            const bool can_block = tgt.stun == 0 || on(tgt, fInBlockstun);
            const bool stand_guard = guard_ok && tgt.posture == kStanding && tgt.move < 0 &&
                (tgt.universal == kIdle || tgt.universal == kWalkBack) && can_block;
            const bool crouch_guard = guard_ok && tgt.posture == kCrouching && tgt.move < 0 &&
                tgt.universal == kCrouch && can_block;
            const bool blocked = hit.level != kThrow && !airborne &&
                ((stand_guard && !(hit.level == kLow)) || (crouch_guard && hit.level != kMid && hit.level != kHigh));
            const bool counter = !blocked && tgt.stun == 0 && !airborne && (def != nullptr || tgt.ki_frames > 0);
            out.contact = blocked ? kBlocked : counter ? kCounterHit : kHit;
            if (hit.level == kThrow && hit.throw_break != kBreakNone) out.contact = kThrowHeld;
        }
        return true;
    }
    return false;
}

// step (full_combat_core.hpp:877-1296)
// One contact found in phase 4 by attacker A (full_combat_core.hpp:1269-1290).
template <int A>
T8B_HD void apply_contact(const Match& m, Fight& s, const Pending& d, Events& e) {
    Fighter& a = s.f[A];
    Fighter& t = s.f[1 - A];
    a.hits_landed |= 1u << static_cast<unsigned>(d.hit_index);
    if (d.contact == kThrowHeld) {
        if (a.move < 0) return;
        a.pending_throw_hit = d.hit_index;
        t.break_frames = m.cfg->throw_break_window;
        t.flags &= ~(fBreakAttempted | fInBlockstun);
        t.stance = -1;
        t.move = -1;
        t.universal = kIdle;
        t.stun = 0;
        t.dash_from = kNoContactFrom;
        add_contact(e, A, d.hit_index, kThrowHeld, 0.0);
        return;
    }
    resolve(m, s, A, d.move_index, d.defense_move, d.hit_index, d.contact, 0, e);
}

T8B_HD void frame_step(const Match& m, Fight& s, const Input& in0, const Input& in1, Events& e) {
    e.contact_count = 0;
    e.transition_count = 0;
    e.heat_activated[0] = e.heat_activated[1] = 0;
    e.rage_activated[0] = e.rage_activated[1] = 0;
    if (s.winner >= 0) return;
    const Cfg& c = *m.cfg;

    // 0. timers
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        Fighter& f = s.f[p];
        if (f.ki_frames > 0 && --f.ki_frames == 0) f.flags &= ~fKiBoost;
        if (on(f, fHeat) && --f.heat_frames <= 0) {
            f.flags &= ~fHeat;
            f.heat_frames = 0;
            f.dash_from = kNoContactFrom;
        }
    }
    // 1. new actions, legality judged for both first
    const bool ok0 = input_ok(m, s, 0, in0);
    const bool ok1 = input_ok(m, s, 1, in1);
    if (ok0) start_action(m, s, 0, in0, e);
    if (ok1) start_action(m, s, 1, in1, e);

    // 2. advance
    bool stepping = false;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        const Fighter& f = s.f[p];
        stepping = stepping || (f.move < 0 && (f.universal == kSidestepLeft || f.universal == kSidestepRight));
    }
    advance(m, s, 0);
    advance(m, s, 1);
    if (!stepping) {
        Fighter& a = s.f[0];
        Fighter& b = s.f[1];
        const double gap = a.axis - b.axis;
        const double shift = lo(mag(gap) / 2.0, c.axis_realign_per_frame / 2.0);
        a.axis -= copysign(shift, gap);
        b.axis += copysign(shift, gap);
    }

    // 3. walls and body collision
#pragma unroll
    for (int p = 0; p < 2; ++p) s.f[p].x = clampd(s.f[p].x, s.left_wall, s.right_wall);
    {
        Fighter& a = s.f[0];
        Fighter& b = s.f[1];
        const double minimum = 2.0 * c.body_radius;
        const double dx = b.x - a.x;
        if (mag(a.axis - b.axis) < minimum && mag(dx) < minimum) {
            const double push = (minimum - mag(dx)) / 2.0;
            const double dir = dx >= 0.0 ? 1.0 : -1.0;
            a.x -= dir * push;
            b.x += dir * push;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                Fighter& f = s.f[k];
                Fighter& other = s.f[1 - k];
                const double over = f.x < s.left_wall ? s.left_wall - f.x
                    : f.x > s.right_wall ? s.right_wall - f.x : 0.0;
                if (over != 0.0) {
                    f.x += over;
                    other.x += over;
                }
            }
#pragma unroll
            for (int p = 0; p < 2; ++p) s.f[p].x = clampd(s.f[p].x, s.left_wall, s.right_wall);
        }
    }

    // 4. contacts from one snapshot
    Pending pend0, pend1;
    const bool found0 = find_contact(m, s, 0, pend0);
    const bool found1 = find_contact(m, s, 1, pend1);

    // 5. a held throw whose window closes lands first, then the new contacts (attacker 0's,
    // then attacker 1's). Every fighter index here is a constant, so a caller that keeps the
    // fight in registers is not forced into local memory.
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        Fighter& held = s.f[p];
        Fighter& thrower = s.f[1 - p];
        if (held.break_frames <= 0 || --held.break_frames > 0) continue;
        held.flags &= ~fBreakAttempted;
        if (thrower.move < 0 || thrower.pending_throw_hit < 0) continue;
        const int move_index = thrower.move;
        const int hit_index = thrower.pending_throw_hit;
        const DMove& mv = move_at(m, 1 - p, move_index);
        thrower.pending_throw_hit = -1;
        resolve(m, s, 1 - p, move_index, -1, hit_index, kHit,
                thrower.action_frame - hit_at(m, 1 - p, mv, hit_index).first_active_frame, e);
        if (thrower.move >= 0 && thrower.action_frame >= mv.total_frames) {
            thrower.stance = mv.result_stance;
            thrower.move = -1;
            thrower.action_frame = action_length(kIdle, c);
        }
    }
    if (found0) apply_contact<0>(m, s, pend0, e);
    if (found1) apply_contact<1>(m, s, pend1, e);

    const bool down0 = s.f[0].health <= 0.0;
    const bool down1 = s.f[1].health <= 0.0;
    if (down0 || down1) s.winner = down0 && down1 ? 2 : (down0 ? 1 : 0);
    ++s.frame;
}

}  // namespace t8b
