// Environment contract on the GPU: candidate inputs and legality, the counter-based RNG,
// the scripted opponents, observation encoding with live noise and the screen view,
// round resets and the per-decision frame loop. Same results as the reference contract
// (include/t8_v2/full_move_contract.hpp), bit for bit: every random draw uses the same
// (seed, stream, counter) triple and every float/double expression keeps its rounding.
#pragma once

#include "engine.cuh"

namespace t8b {

// ------------------------------------------------------------------ candidates
// universal_candidate_input (include/t8_v2/full_move_roster.hpp:27-50): candidate -> universal,
// -1 where the engine has no such mechanic.
T8B_HD int universal_of_candidate(int candidate) {
    switch (candidate) {
        case 0: return kIdle;
        case 1: return kWalkForward;
        case 2: return kWalkBack;
        case 3: return kDashForward;
        case 4: return kBackdash;
        case 5: return kCrouch;
        case 6: return kIdle;
        case 8: return kSidestepLeft;
        case 9: return kSidestepRight;
        case 15: return kThrowBreak1;
        case 16: return kThrowBreak2;
        case 17: return kThrowBreak;
        case 18: return kHeatDash;
        case 19: return kWakeupStand;
        case 20: return kWakeupRoll;
        case 21: return kTechRoll;
        default: return -1;
    }
}

// candidate_input (full_move_contract.hpp:30-38)
T8B_HD bool to_input(const DCharacter& ch, int candidate, Input& in) {
    if (candidate < 0 || candidate >= ch.candidate_count) return false;
    if (candidate < kUniversalCount) {
        in.move = -1;
        const int u = universal_of_candidate(candidate);
        if (u < 0) return false;
        in.universal = u;
        return true;
    }
    const int move = ch.candidate_moves[candidate];
    if (move < 0) return false;
    in.move = move;
    in.universal = kIdle;
    return true;
}

// candidate_legal (full_move_contract.hpp:42-49). A move candidate's legality reads its gate
// record (the same fields input_ok reads of the move; candidates name existing moves).
T8B_HD bool candidate_ok(const Match& m, const Fight& s, int p, int candidate) {
    if (candidate == 0) return true;
    const DCharacter& ch = *m.side[p];
    if (candidate >= kUniversalCount && candidate < ch.candidate_count) {
        const DGate g = ch.gates[candidate];
        if (g.move < 0 || s.winner >= 0) return false;
        return move_allowed(m, s, p, g.flags, g.required_posture, g.required_stance, g.heat_cost != 0);
    }
    Input in{-1, kIdle};
    if (!to_input(ch, candidate, in)) return false;
    if (candidate == 6 && s.f[p].posture != kCrouching) return false;
    return input_ok(m, s, p, in);
}

// candidate_ok for the universal candidates 0..21 of fighter p, as bit c of one word: the same
// decisions (to_input's mapping, candidate 6's crouch requirement, input_ok's cases) taken once
// for the fight instead of once per candidate, so the lanes of a warp that each check one
// candidate of the same fight follow one path. `can` is can_act(m, s, p). Bits at or past the
// fighter's candidate count are the caller's to clear.
T8B_HD uint32_t universal_mask(const Match& m, const Fight& s, int p, bool can) {
    uint32_t mask = 1u;  // candidate 0 is always legal
    if (s.winner >= 0) return mask;
    const Fighter& f = s.f[p];
    const Cfg& c = *m.cfg;
    const bool wake = f.posture == kGrounded && f.grounded_elapsed >= c.knockdown_frames;
    const bool tech = f.posture == kGrounded && on(f, fTechable) && f.grounded_elapsed < c.tech_window_frames;
    const bool escape = f.break_frames > 0 && !on(f, fBreakAttempted);
    bool heat_dash = false;
    if (f.move >= 0 && on(f, fHeat) && f.dash_from != kNoContactFrom) {
        const DMove& mv = move_at(m, p, f.move);
        heat_dash = f.dash_from == kBlocked ? has(mv, kHasHeatDashBlock) : has(mv, kHasHeatDashHit);
    }
#pragma unroll
    for (int candidate = 1; candidate < kUniversalCount; ++candidate) {
        const int u = universal_of_candidate(candidate);
        bool legal;
        if (u < 0) legal = false;
        else if (candidate == 6) legal = f.posture == kCrouching && can;
        else if (u == kWakeupStand || u == kWakeupRoll) legal = wake;
        else if (u == kTechRoll) legal = tech;
        else if (u == kThrowBreak || u == kThrowBreak1 || u == kThrowBreak2) legal = escape;
        else if (u == kHeatDash) legal = heat_dash;
        else legal = can;
        mask |= (legal ? 1u : 0u) << candidate;
    }
    return mask;
}

// candidate_ok for many candidates of one fighter in one state (a scripted opponent's choice):
// can_act and the universal candidates' word are taken once. `moves_possible` is false when no
// move candidate can pass (the fighter can neither act nor continue a sidestep, or the round is
// over), so a caller may skip probing them.
struct Legality {
    const Match& m;
    const Fight& s;
    int p;
    bool can;
    uint32_t universal;
    bool moves_possible;
    T8B_HD Legality(const Match& match, const Fight& state, int player)
        : m(match), s(state), p(player), can(can_act(match, state, player)),
          universal(universal_mask(match, state, player, can)), moves_possible(false) {
        const Fighter& f = state.f[player];
        const bool stepping = f.move < 0 && f.action_frame >= 1 && f.stun == 0 && !on(f, fCrumpled) &&
            f.break_frames == 0 && f.pending_throw_hit < 0 &&
            (f.universal == kSidestepLeft || f.universal == kSidestepRight);
        moves_possible = state.winner < 0 && (can || stepping);
    }
    T8B_HD bool operator()(int candidate) const {
        if (candidate == 0) return true;
        const DCharacter& ch = *m.side[p];
        if (candidate < 0 || candidate >= ch.candidate_count) return false;
        if (candidate < kUniversalCount) return ((universal >> candidate) & 1u) != 0u;
        return move_ok(candidate);
    }
    // The same for a candidate known to be universal (0 <= candidate < kUniversalCount) or a
    // move (kUniversalCount <= candidate < the candidate count): each call site then carries only
    // its branch of the check, which keeps the frame loop's code small.
    T8B_HD bool universal_ok(int candidate) const {
        return candidate == 0 || (candidate < m.side[p]->candidate_count && ((universal >> candidate) & 1u) != 0u);
    }
    T8B_HD bool move_ok(int candidate) const {
        const DGate g = m.side[p]->gates[candidate];
        if (g.move < 0 || s.winner >= 0) return false;
        return move_allowed_given(m, s, p, can, g.flags, g.required_posture, g.required_stance, g.heat_cost != 0);
    }
};

// has_decision (full_move_contract.hpp:52-67)
T8B_HD bool decides(const Match& m, const Fight& s, int p) {
    if (s.winner >= 0) return false;
    if (can_act(m, s, p)) return true;
    const Fighter& f = s.f[p];
    if (f.move < 0 && f.action_frame >= 1 && (f.universal == kSidestepLeft || f.universal == kSidestepRight) &&
        f.stun == 0 && f.posture == kStanding) {
        return true;
    }
    return input_ok(m, s, p, Input{-1, kThrowBreak}) || input_ok(m, s, p, Input{-1, kHeatDash}) ||
        input_ok(m, s, p, Input{-1, kWakeupStand}) || input_ok(m, s, p, Input{-1, kTechRoll});
}

// ------------------------------------------------------------------ counter-based RNG
// mix64 / random_bits / random_below / random_unit (full_move_contract.hpp:71-85): the
// SplitMix64 finaliser (Steele, Lea, Flood 2014) applied to a hashed (seed, stream, counter).
T8B_HD uint64_t mix64(uint64_t v) {
    v += 0x9E3779B97F4A7C15ull;
    v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ull;
    v = (v ^ (v >> 27)) * 0x94D049BB133111EBull;
    return v ^ (v >> 31);
}
// hash3(seed, stream, counter) = draw(prefix_of(seed, stream), counter): a caller making many
// draws from one (seed, stream) takes the prefix once.
T8B_HD uint64_t prefix_of(uint64_t seed, uint64_t stream) { return mix64(seed ^ mix64(stream)); }
T8B_HD uint64_t draw(uint64_t prefix, uint64_t counter) { return mix64(prefix ^ counter); }
T8B_HD uint64_t hash3(uint64_t seed, uint64_t stream, uint64_t counter) { return draw(prefix_of(seed, stream), counter); }
T8B_HD int below(uint64_t bits, int bound) { return static_cast<int>(bits % static_cast<uint64_t>(bound)); }
// x mod b for x < 2^53 and b < 2^20, given inverse = 1.0 / b: the double quotient estimate is off
// by at most one, so one correction gives the exact remainder.
T8B_HD uint32_t reduce_by(uint64_t x, uint32_t b, double inverse) {
    int64_t r = static_cast<int64_t>(x) -
        static_cast<int64_t>(static_cast<double>(x) * inverse) * static_cast<int64_t>(b);
    if (r < 0) r += b;
    else if (r >= static_cast<int64_t>(b)) r -= b;
    return static_cast<uint32_t>(r);
}
// below(bits, bound) for a bound below 2^20 with its reciprocal at hand: the high word reduced
// first, then the 52-bit rest.
T8B_HD int below_with(uint64_t bits, int bound, double inverse) {
    const uint32_t b = static_cast<uint32_t>(bound);
    const uint64_t r = reduce_by(bits >> 32, b, inverse);
    return static_cast<int>(reduce_by((r << 32) | (bits & 0xffffffffull), b, inverse));
}
T8B_HD double unit(uint64_t bits) { return static_cast<double>(bits >> 11) * (1.0 / 9007199254740992.0); }

// ------------------------------------------------------------------ scripted opponents
// scripted_candidate (full_move_contract.hpp:90-119): the legacy random opponent.
T8B_HD int random_opponent(const Match& m, const Fight& s, int p, double aggression, uint64_t prefix, uint64_t counter) {
    const DCharacter& ch = *m.side[p];
    const Legality legal(m, s, p);
    const bool close = mag(s.f[p].x - s.f[1 - p].x) < 1.6;
    uint64_t draw_index = 0;
    const int roll = below(draw(prefix, counter * 64u + draw_index++), 100);
    if (!close && roll < 55) {
        const int approach = roll < 30 ? 3 : 1;
        if (legal.universal_ok(approach)) return approach;
    }
    if (close && roll < 15) {
        const int guard = roll < 8 ? 0 : 5;
        if (legal.universal_ok(guard)) return guard;
    }
    const int share = static_cast<int>((close ? 55.0 : 15.0) + 30.0 * aggression);
    if (ch.candidate_count > kUniversalCount && below(draw(prefix, counter * 64u + draw_index++), 100) < share) {
        if (legal.moves_possible) {
            for (int k = 0; k < 24; ++k) {
                const int c = kUniversalCount + below_with(draw(prefix, counter * 64u + draw_index++), ch.candidate_count - kUniversalCount, ch.move_candidate_inverse);
                if (legal.move_ok(c)) return c;
            }
        } else {
            draw_index += 24;  // every probe would fail: their draws are skipped, not their indices
        }
    }
    for (int k = 0; k < 24; ++k) {
        const int c = below(draw(prefix, counter * 64u + draw_index++), kUniversalCount);
        if (legal.universal_ok(c)) return c;
    }
    return 0;
}

// ScriptedProfile (full_move_contract.hpp:131-148); the host computes the 331 profiles once.
struct Profile {
    int32_t tier, fixed;
    float aggression, block;
    int32_t reaction;
    float punish, throw_break, sidestep, smart, distance, keepaway, low_bias, throw_bias, heat_use, movement, pressure;
};

// decode_bot (full_move_contract.hpp:273)
T8B_HD int bot_id(double behaviour) { return behaviour < 0.0 ? static_cast<int>(-behaviour + 0.5) - 1 : -1; }

// scripted_bot_candidate (full_move_contract.hpp:319-502)
T8B_HD int bot_choice(const Match& m, const Fight& s, int p, const Profile& pr, uint64_t seed, uint64_t stream,
                      uint64_t prefix, uint64_t counter) {
    constexpr int cNeutral = 0, cWalkForward = 1, cWalkBack = 2, cDash = 3, cBackdash = 4, cCrouch = 5;
    constexpr int cStepLeft = 8, cStepRight = 9, cBreak1 = 15, cBreak2 = 16, cBreak12 = 17;
    constexpr int cWakeStand = 19, cWakeRoll = 20, cTechRoll = 21;
    const DCharacter& ch = *m.side[p];
    const Legality legal(m, s, p);
    if (pr.fixed >= 0) return legal(pr.fixed) ? pr.fixed : cNeutral;
    const Fighter& own = s.f[p];
    const Fighter& other = s.f[1 - p];
    const double distance = mag(own.x - other.x);
    uint64_t draw_index = 0;
    const uint64_t attack_key = static_cast<uint64_t>(s.frame - other.action_frame) * 4096u +
        static_cast<uint64_t>(other.move + 1);
#define T8B_ROLL() unit(draw(prefix, counter * 64u + draw_index++))
#define T8B_ATTACK_ROLL(purpose) unit(hash3(seed, stream ^ (0x9e3779b97f4a7c15ull * ((purpose) + 1ull)), attack_key))
    const int spread = ihi(1, ch.candidate_count - kUniversalCount);

    // throw break
    if (own.break_frames > 0 && !on(own, fBreakAttempted) && other.move >= 0 && other.pending_throw_hit >= 0) {
        const DMove& tm = move_at(m, 1 - p, other.move);
        const uint8_t rule = hit_at(m, 1 - p, tm, other.pending_throw_hit).throw_break;
        int right = cBreak12;
        if (rule == kBreakOne || rule == kBreakOneOrTwo) right = cBreak1;
        if (rule == kBreakTwo) right = cBreak2;
        int choice = right;
        if (T8B_ATTACK_ROLL(1ull) >= pr.throw_break) choice = right == cBreak12 ? cBreak1 : (right == cBreak1 ? cBreak2 : cBreak12);
        if (legal(choice)) return choice;
    }
    // getting up
    if (own.posture == kGrounded) {
        const int options[3] = {cWakeStand, cWakeRoll, cTechRoll};
        const int first = below(draw(prefix, counter * 64u + 63u), 3);
        for (int k = 0; k < 3; ++k) {
            if (legal(options[(first + k) % 3])) return options[(first + k) % 3];
        }
    }
    // defense
    if (other.move >= 0) {
        const DMove& mv = move_at(m, 1 - p, other.move);
        for (int k = 0; k < mv.hit_count; ++k) {
            if ((other.hits_landed >> static_cast<unsigned>(k)) & 1u) continue;
            const DHit& hit = hit_at(m, 1 - p, mv, k);
            if (other.action_frame >= hit.first_active_frame + hit.active_frames) continue;
            const int until = hit.first_active_frame - other.action_frame;
            const bool seen = other.action_frame >= pr.reaction;
            if (!seen || distance > hit.reach + 0.4) break;
            const double answer = T8B_ATTACK_ROLL(2ull);
            if (!(hit.flags & kHoming) && until >= 12 && answer < pr.sidestep) {
                const int side = T8B_ATTACK_ROLL(3ull) < 0.5 ? cStepLeft : cStepRight;
                if (legal(side)) return side;
            }
            if (answer < pr.sidestep + pr.block) {
                const bool crouch = hit.level == kLow || hit.level == kSpecialLow || hit.level == kThrow ||
                    (hit.level == kHigh && T8B_ATTACK_ROLL(4ull) < 0.5);
                const int guard = crouch ? cCrouch : cNeutral;
                if (legal(guard)) return guard;
            }
            break;
        }
    }
    // punish
    if (other.move >= 0 && legal.can) {
        const DMove& mv = move_at(m, 1 - p, other.move);
        int last_active = 0;
        for (int k = 0; k < mv.hit_count; ++k) {
            const DHit& hit = hit_at(m, 1 - p, mv, k);
            last_active = ihi(last_active, hit.first_active_frame + hit.active_frames);
        }
        const int remaining = mv.total_frames - other.action_frame;
        int window = 0;
        if (other.action_frame >= last_active && !on(other, fMoveHit) && !on(other, fMoveBlocked)) window = remaining;
        if (on(other, fMoveBlocked) && mv.block_advantage <= -10) window = ilo(remaining, -mv.block_advantage);
        if (window > 0 && T8B_ATTACK_ROLL(5ull) < pr.punish) {
            int best = -1;
            double best_score = -1.0;
            for (int k = 0; k < 24; ++k) {
                const int c = kUniversalCount + below(draw(prefix, counter * 64u + 32u + static_cast<uint64_t>(k)), spread);
                if (c >= ch.candidate_count) continue;
                const DFacts& fx = ch.facts[c];
                if (!(fx.bits & 1u) || (fx.bits & 16u) || fx.startup > window || fx.reach + 0.1 < distance) continue;
                const double score = fx.damage + ((fx.bits & 4u) ? 25.0 : 0.0);
                if (score > best_score && legal(c)) {
                    best = c;
                    best_score = score;
                }
            }
            if (best >= 0) return best;
        }
    }
    // Heat and Rage
    if (pr.heat_use > 0.0F && legal.can) {
        const bool want_heat = on(own, fHeatAvailable) && !on(own, fHeat) && T8B_ROLL() < 0.02 * pr.heat_use;
        const bool want_rage = on(own, fRage) && distance < 1.3 && T8B_ROLL() < 0.05 * pr.heat_use;
        if (want_heat || want_rage) {
            for (int c = kUniversalCount; c < ch.candidate_count; ++c) {
                const DFacts& fx = ch.facts[c];
                const bool wanted = want_rage ? (fx.flags & kRequiresRage) != 0 : (fx.flags & kEngagesHeat) != 0;
                if (wanted && legal(c)) return c;
            }
        }
    }
    // pressure
    if (pr.pressure > 0.0F && on(other, fInBlockstun) && legal.can && T8B_ROLL() < pr.pressure) {
        for (int k = 0; k < 16; ++k) {
            const int c = kUniversalCount + below(draw(prefix, counter * 64u + 40u + static_cast<uint64_t>(k)), spread);
            if (c >= ch.candidate_count) continue;
            const DFacts& fx = ch.facts[c];
            if ((fx.bits & 1u) && !(fx.bits & 16u) && fx.startup <= 14 && fx.reach + 0.05 >= distance &&
                legal(c)) {
                return c;
            }
        }
    }
    // fundamentals
    if (other.move >= 0) {
        const DMove& mv = move_at(m, 1 - p, other.move);
        bool incoming = false;
        for (int k = 0; k < mv.hit_count; ++k) {
            const DHit& hit = hit_at(m, 1 - p, mv, k);
            if (!((other.hits_landed >> static_cast<unsigned>(k)) & 1u) &&
                other.action_frame < hit.first_active_frame + hit.active_frames) {
                incoming = true;
            }
        }
        const bool opponent_plus = on(other, fMoveBlocked) && mv.block_advantage > 0;
        if ((incoming || opponent_plus) && distance < 2.0 && T8B_ROLL() < pr.smart) return cNeutral;
    }
    // offense and spacing
    const double reach = 1.25;
    if (pr.keepaway > 0.0F && distance > reach && distance < pr.distance + 0.6 && T8B_ROLL() < 0.025 * pr.aggression) {
        if (legal(cDash)) return cDash;
    }
    const double attack_rate = 0.12 * pr.aggression * (pr.keepaway > 0.0F ? 3.0 : 1.0);
    if (distance <= reach + 0.25 && T8B_ROLL() < attack_rate) {
        int best = -1;
        double best_score = -1e9;
        for (int k = 0; k < 12; ++k) {
            const int c = kUniversalCount + below(draw(prefix, counter * 64u + 8u + static_cast<uint64_t>(k)), spread);
            if (c >= ch.candidate_count) continue;
            const DFacts& fx = ch.facts[c];
            if (!(fx.bits & 1u) || !legal(c)) continue;
            if (fx.reach + 0.05 < distance && T8B_ROLL() < 0.3 + 0.7 * pr.smart) continue;
            double score = T8B_ROLL() * 2.0;
            if (T8B_ROLL() < pr.smart) {
                score += ((fx.bits & 2u) ? 2.0 : -1.5) + (fx.startup <= 12 ? 2.5 : (fx.startup <= 15 ? 0.5 : -2.0)) +
                    (fx.reach + 0.05 >= distance ? 1.5 : -3.0) + fx.damage / 30.0;
            }
            score += ((fx.bits & 8u) ? pr.low_bias : 0.0) + ((fx.bits & 16u) ? pr.throw_bias : 0.0);
            if (score > best_score) {
                best = c;
                best_score = score;
            }
        }
        if (best >= 0) return best;
    }
    const double r = T8B_ROLL();
    if (distance > pr.distance + 0.2) {
        const int approach = pr.aggression > 0.7F && distance > 2.0 ? cDash : cWalkForward;
        if (legal(approach)) return approach;
    }
    if (distance < pr.distance - 0.3 && pr.keepaway > 0.0F && r < 0.08 * pr.keepaway) {
        const int retreat = r < 0.03 * pr.keepaway ? cBackdash : cWalkBack;
        if (legal(retreat)) return retreat;
    }
    if (r > 1.0 - 0.05 * pr.movement) {
        const int side = r > 1.0 - 0.025 * pr.movement ? cStepLeft : cStepRight;
        if (legal(side)) return side;
    }
#undef T8B_ROLL
#undef T8B_ATTACK_ROLL
    return cNeutral;
}

// ------------------------------------------------------------------ observation
T8B_HD float c01(double v) { return static_cast<float>(clampd(v, 0.0, 1.0)); }
T8B_HD float c11(double v) { return static_cast<float>(clampd(v, -1.0, 1.0)); }

// encode_move (full_move_contract.hpp:512-527), written at out[0..7]
T8B_HD void move_features(const Match& m, const Fight& s, int p, float* out) {
    const Fighter& f = s.f[p];
    for (int k = 0; k < 8; ++k) out[k] = 0.0F;
    if (f.move < 0) return;
    const DMove& mv = move_at(m, p, f.move);
    out[0] = 1.0F;
    out[7] = c01(static_cast<double>(mv.total_frames - f.action_frame) / 60.0);
    out[6] = c11(static_cast<double>(mv.block_advantage) / 30.0);
    for (int k = 0; k < mv.hit_count; ++k) {
        if ((f.hits_landed >> static_cast<unsigned>(k)) & 1u) continue;
        const DHit& next = hit_at(m, p, mv, k);
        out[1 + level_slot(next.level)] = 1.0F;
        out[5] = c01(static_cast<double>(next.first_active_frame - f.action_frame) / 30.0);
        break;
    }
}

// encode_observation (full_move_contract.hpp:535-605); out has kObservationBase floats.
T8B_HD void observe(const Match& m, const Fight& s, int p, int round_frames, int own_id, int other_id, float* out,
                    int perception_delay) {
    const Cfg& c = *m.cfg;
    for (int k = kStateFeatures; k < kObservationBase; ++k) out[k] = 0.0F;
    if (own_id >= 0 && own_id < kRosterSlots) out[kStateFeatures + own_id] = 1.0F;
    if (other_id >= 0 && other_id < kRosterSlots) out[kStateFeatures + kRosterSlots + other_id] = 1.0F;
    const Fighter& own = s.f[p];
    const Fighter& opp = s.f[1 - p];
    const double width = s.right_wall - s.left_wall;
    const double toward = facing(s, p);
    const double behind = toward > 0.0 ? own.x - s.left_wall : s.right_wall - own.x;
    const double ahead = toward > 0.0 ? s.right_wall - opp.x : opp.x - s.left_wall;
    out[0] = c01(own.health / c.max_health);
    out[1] = c01(opp.health / c.max_health);
    out[2] = c01(own.recoverable / c.max_health);
    out[3] = c01(opp.recoverable / c.max_health);
    out[4] = c01(mag(opp.x - own.x) / 4.0);
    out[5] = c11((opp.axis - own.axis) * toward / 2.0);
    out[6] = c01(behind / hi(width, 1e-9));
    out[7] = c01(ahead / hi(width, 1e-9));
    for (int k = 0; k < 6; ++k) {
        out[8 + k] = own.posture == k ? 1.0F : 0.0F;
        out[14 + k] = opp.posture == k ? 1.0F : 0.0F;
    }
    out[20] = c01(own.stun / 60.0);
    out[21] = c01(opp.stun / 60.0);
    out[22] = on(own, fInBlockstun) ? 1.0F : 0.0F;
    out[23] = on(opp, fInBlockstun) ? 1.0F : 0.0F;
    out[24] = can_act(m, s, p) ? 1.0F : 0.0F;
    out[25] = can_act(m, s, 1 - p) ? 1.0F : 0.0F;
    out[26] = on(own, fHeat) ? 1.0F : 0.0F;
    out[27] = c01(static_cast<double>(own.heat_frames) / hi(1.0, c.heat_duration_frames));
    out[28] = on(own, fHeatAvailable) ? 1.0F : 0.0F;
    out[29] = on(own, fRage) ? 1.0F : 0.0F;
    out[30] = on(own, fRageAvailable) ? 1.0F : 0.0F;
    out[31] = on(opp, fHeat) ? 1.0F : 0.0F;
    out[32] = on(opp, fRage) ? 1.0F : 0.0F;
    const int own_stances = m.side[p]->stance_count;
    out[33] = own.stance >= 0 ? 1.0F : 0.0F;
    out[34] = own.stance >= 0 ? static_cast<float>(own.stance + 1) / static_cast<float>(own_stances + 1) : 0.0F;
    out[35] = opp.stance >= 0 ? 1.0F : 0.0F;
    const DRules& rules = m.side[p]->rules;
    out[36] = rules.resource_max > 0.0 ? c01(own.resource / rules.resource_max) : 0.0F;
    out[37] = on(own, fInstalled) ? 1.0F : 0.0F;
    out[38] = on(own, fBackTurned) ? 1.0F : 0.0F;
    out[39] = on(opp, fBackTurned) ? 1.0F : 0.0F;
    out[40] = c01(own.combo_hits / 10.0);
    out[41] = c01(opp.combo_hits / 10.0);
    out[42] = own.break_frames > 0 ? 1.0F : 0.0F;
    out[43] = own.pending_throw_hit >= 0 ? 1.0F : 0.0F;
    out[44] = own.dash_from != kNoContactFrom ? 1.0F : 0.0F;
    out[45] = c01(static_cast<double>(own.grounded_elapsed) / hi(1.0, c.knockdown_frames));
    out[46] = c01(static_cast<double>(opp.grounded_elapsed) / hi(1.0, c.knockdown_frames));
    out[47] = c01(1.0 - static_cast<double>(s.frame) / hi(1.0, round_frames));
    out[48] = own.ki_frames > 0 ? 1.0F : 0.0F;
    out[49] = opp.ki_frames > 0 ? 1.0F : 0.0F;
    move_features(m, s, 1 - p, out + 50);
    if (opp.move >= 0 && opp.action_frame < perception_delay) {
        for (int k = 50; k < 58; ++k) out[k] = 0.0F;
    }
    out[58] = own.move >= 0 ? 1.0F : 0.0F;
    out[59] = own.move >= 0 ? c01(static_cast<double>(move_at(m, p, own.move).total_frames - own.action_frame) / 60.0) : 0.0F;
    out[60] = on(own, fTechable) ? 1.0F : 0.0F;
    out[61] = c01(own.posture_frames / 60.0);
    out[62] = c01(opp.posture_frames / 60.0);
    out[63] = 1.0F;
}

// NoiseLevels (full_move_contract.hpp:787-792)
struct Noise {
    float position_sigma, flip_rate;
    int32_t latency;
    uint32_t key;
};

// draw_noise_levels (full_move_contract.hpp:805-815)
T8B_HD Noise draw_noise(const EnvCfg& ec, uint64_t seed, uint64_t stream, uint64_t counter) {
    const uint64_t base = seed ^ 0x6e6f697365ull;
    Noise n;
    n.position_sigma = static_cast<float>(ec.noise_position_max * unit(hash3(base, stream, counter * 4u)));
    n.flip_rate = static_cast<float>(ec.noise_flip_max * unit(hash3(base, stream, counter * 4u + 1u)));
    const int span = ihi(0, ec.latency_max - ec.latency_min) + 1;
    n.latency = ec.latency_min + below(hash3(base, stream, counter * 4u + 2u), span);
    n.key = static_cast<uint32_t>(hash3(base, stream, counter * 4u + 3u));
    return n;
}

// noise_gaussian (full_move_contract.hpp:818-822): Irwin-Hall sum of four uniforms.
T8B_HD double gaussian4(uint64_t key, uint64_t stream, uint64_t counter) {
    double sum = 0.0;
    for (uint64_t k = 0; k < 4u; ++k) sum += unit(hash3(key, stream, counter * 4u + k));
    return (sum - 2.0) * 1.7320508075688772;
}

// apply_observation_noise (full_move_contract.hpp:827-873)
T8B_HD void perturb(const Noise& n, const Fight& s, int p, float* out) {
    const uint64_t key = n.key;
    const uint64_t frame = static_cast<uint64_t>(s.frame);
    const uint64_t side = static_cast<uint64_t>(p) * 4096u;
    const double sigma = n.position_sigma;
    const double flip = n.flip_rate;
#define T8B_GAUSS(i) gaussian4(key, side + static_cast<uint64_t>(i), frame)
#define T8B_UNIFORM(i) unit(hash3(key, side + 2048u + static_cast<uint64_t>(i), frame))
    for (int k = 0; k < 4; ++k) out[k] = c01(out[k] + 0.005 * T8B_GAUSS(k));
    out[4] = c01(out[4] + sigma / 4.0 * T8B_GAUSS(4));
    out[5] = c11(out[5] + sigma / 2.0 * T8B_GAUSS(5));
    out[6] = c01(out[6] + sigma / 7.2 * T8B_GAUSS(6));
    out[7] = c01(out[7] + sigma / 7.2 * T8B_GAUSS(7));
    for (int who = 0; who < 2; ++who) {
        if (T8B_UNIFORM(8 + who) < flip) {
            const int wrong = below(hash3(key, side + 3000u + static_cast<uint64_t>(who), frame), 6);
            for (int k = 0; k < 6; ++k) out[8 + 6 * who + k] = k == wrong ? 1.0F : 0.0F;
        }
    }
    for (int k = 20; k < 24; ++k) {
        if (T8B_UNIFORM(k) < flip) out[k] = 0.0F;
    }
    for (int k = 24; k < 26; ++k) {
        if (T8B_UNIFORM(k) < flip) out[k] = 1.0F - out[k];
    }
    const double roll = T8B_UNIFORM(50);
    if (out[50] > 0.5F) {
        if (roll < flip) {
            for (int k = 50; k < 58; ++k) out[k] = 0.0F;
        } else if (roll < 2.0 * flip) {
            const int wrong = below(hash3(key, side + 3002u, frame), 4);
            for (int k = 0; k < 4; ++k) out[51 + k] = k == wrong ? 1.0F : 0.0F;
        }
        out[55] = c01(out[55] + 20.0 * flip / 30.0 * T8B_GAUSS(55));
    } else if (roll < 0.25 * flip) {
        out[50] = 1.0F;
        const int level = below(hash3(key, side + 3003u, frame), 4);
        for (int k = 0; k < 4; ++k) out[51 + k] = k == level ? 1.0F : 0.0F;
        out[55] = static_cast<float>(T8B_UNIFORM(55));
        out[56] = 0.0F;
        out[57] = static_cast<float>(T8B_UNIFORM(57));
    }
#undef T8B_GAUSS
#undef T8B_UNIFORM
}

// screen_view_feature / apply_screen_view (full_move_contract.hpp:897-918)
T8B_HD bool screen_feature(int k) {
    return (k >= 0 && k <= 4) || (k >= 8 && k <= 11) || (k >= 14 && k <= 17) || k == 24 || k == 29 || k == 32 ||
        k == 33 || k == 34 || k == 50 || k == 58 || k == 59 || k == 63;
}
T8B_HD void screen_view(float* out) {
    for (int base = 8; base <= 14; base += 6) {
        if (out[base + 4] > 0.5F) out[base + 3] = 1.0F;
        if (out[base + 5] > 0.5F) out[base + 0] = 1.0F;
    }
    for (int k = 0; k < kStateFeatures; ++k) {
        if (!screen_feature(k)) out[k] = 0.0F;
    }
}

// encode_noise_levels (full_move_contract.hpp:920-924)
T8B_HD void noise_features(const Noise& n, float* out) {
    out[0] = c01(n.position_sigma / 0.5);
    out[1] = c01(n.flip_rate / 0.3);
    out[2] = c01(n.latency / 10.0);
}

// ------------------------------------------------------------------ resets
enum Scenario { scNeutral = 0, scWall, scPunish, scThrowBreak, scWakeup, scJuggle, scHeat, scRage, scRange };

// env_reset + find_opponent_move (full_move_contract.hpp:966-1059)
T8B_HD void start_round(const Match& m, Fight& s, const EnvCfg& ec, uint64_t seed, uint64_t stream, uint64_t counter,
                        int scenario, int learner) {
    const Cfg& c = *m.cfg;
    double center = (2.0 * unit(hash3(seed, stream, counter * 4u)) - 1.0) * ec.start_center_range;
    double distance = ec.start_distance_min +
        unit(hash3(seed, stream, counter * 4u + 1u)) * (ec.start_distance_max - ec.start_distance_min);
    const bool flip = (hash3(seed, stream, counter * 4u + 2u) & 1u) != 0u;
    const double half = c.half_width;
    if (scenario == scWall) center = (flip ? 1.0 : -1.0) * (half - 0.9);
    if (scenario == scRange) distance = 3.0 + unit(hash3(seed, stream, counter * 4u + 3u));
    if (scenario == scPunish || scenario == scThrowBreak || scenario == scJuggle || scenario == scWakeup) {
        distance = scenario == scThrowBreak ? 0.6 : 0.9;
    }
    fresh_fight(m, s, center - distance / 2.0, center + distance / 2.0);
    const int op = 1 - learner;
    Fighter& own = s.f[learner];
    Fighter& other = s.f[op];
    const DCharacter& och = *m.side[op];
    if (scenario == scPunish || scenario == scThrowBreak) {
        if (och.candidate_count <= kUniversalCount) return;
        int found = -1;
        for (int k = 0; k < 48; ++k) {
            const int c2 = kUniversalCount +
                below(hash3(seed, stream, counter * 4u + 8u + static_cast<uint64_t>(k)), och.candidate_count - kUniversalCount);
            const int move = och.candidate_moves[c2];
            if (move < 0) continue;
            const DMove& mv = och.moves[move];
            bool want;
            if (scenario == scPunish) {
                want = mv.hit_count > 0 && mv.block_advantage <= -10 && mv.required_stance < 0 && !has(mv, kReactive);
            } else {
                want = mv.hit_count != 0 && mv.required_stance < 0;
                if (want) {
                    const DHit& first = och.hits[mv.hit_offset];
                    want = first.level == kThrow && first.throw_break != kBreakNone &&
                        mv.required_posture == kStanding && !has(mv, kReactive);
                }
            }
            if (want) {
                found = move;
                break;
            }
        }
        if (found < 0) return;
        const DMove& mv = och.moves[found];
        other.move = found;
        if (scenario == scPunish) {
            other.action_frame = ihi(0, mv.total_frames + mv.block_advantage);
            other.hits_landed = mv.hit_count >= 32 ? ~0u : (1u << static_cast<unsigned>(mv.hit_count)) - 1u;
            other.flags |= fMoveBlocked;
        } else {
            other.action_frame = och.hits[mv.hit_offset].first_active_frame;
            other.hits_landed = 1u;
            other.pending_throw_hit = 0;
            own.break_frames = c.throw_break_window;
            own.flags &= ~fBreakAttempted;
        }
        return;
    }
    switch (scenario) {
        case scWakeup:
            own.posture = kGrounded;
            own.grounded_elapsed = 0;
            own.flags &= ~fTechable;
            break;
        case scJuggle:
            other.posture = kAirborne;
            other.posture_frames = 45;
            other.combo_hits = 1;
            break;
        case scHeat:
            own.flags = (own.flags | fHeat) & ~fHeatAvailable;
            own.heat_frames = c.heat_duration_frames;
            break;
        case scRage:
            own.health = c.max_health * c.rage_health_fraction * 0.8;
            own.flags = (own.flags | fRage) & ~fRageAvailable;
            break;
        default: break;
    }
}

// ------------------------------------------------------------------ memory (--memory)
// full_move_contract.hpp:611-735: each fighter's last four moves (level, how they ended, age)
// and decaying traces of its habits, updated after every frame and appended to the observation
// (the opponent's newest move only once it is perception_delay frames old).
constexpr int kMemorySlots = 4;
constexpr int kMemorySlotFeatures = 10;  // level: high, mid, low, throw, no hit; outcome: hit, counter, blocked, missed; age
constexpr int kMemoryTraces = 5;         // crouching, backing off, sidestepping, guarding, attacking
constexpr int kMemoryFighterFeatures = kMemorySlots * kMemorySlotFeatures + kMemoryTraces;
constexpr int kMemoryFeatures = 2 * kMemoryFighterFeatures;

struct MemoryEntry {
    int16_t move_plus_one;  // 0: empty slot
    int8_t level;           // 1 high, 2 mid, 3 low, 4 throw, 5 no hit
    int8_t outcome;         // 0 pending, 1 hit, 2 counter hit, 3 blocked, 4 missed or stopped
    int32_t age;            // frames since it started
};
struct FighterMemory {
    MemoryEntry slots[kMemorySlots];  // newest first
    int32_t last_move_plus_one, last_action_frame;
    float traces[kMemoryTraces];
};
struct Memory {
    FighterMemory f[2];
};
static_assert(sizeof(Memory) == 120, "two 60-byte fighter memories");

// memory_level (full_move_contract.hpp:648-660)
T8B_HD int8_t memory_level(const Match& m, int p, int move) {
    const DMove& mv = move_at(m, p, move);
    if (mv.hit_count <= 0) return 5;
    switch (hit_at(m, p, mv, 0).level) {
        case kHigh: return 1;
        case kMid:
        case kSpecialMid: return 2;
        case kLow:
        case kSpecialLow: return 3;
        case kThrow: return 4;
        default: return 5;
    }
}

// memory_update (full_move_contract.hpp:663-712), after every engine frame with its events.
T8B_HD void memory_update(const Match& m, const Fight& s, const Events& e, int perception_delay, Memory& memory) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        FighterMemory& fm = memory.f[p];
        const Fighter& f = s.f[p];
#pragma unroll
        for (int slot = 0; slot < kMemorySlots; ++slot) {
            if (fm.slots[slot].move_plus_one != 0) ++fm.slots[slot].age;
        }
        const bool ended = f.move < 0 && fm.last_move_plus_one != 0;
        const bool started = f.move >= 0 && (f.move + 1 != fm.last_move_plus_one || f.action_frame < fm.last_action_frame);
        if ((ended || started) && fm.slots[0].move_plus_one != 0 && fm.slots[0].outcome == 0) fm.slots[0].outcome = 4;
        if (started) {
#pragma unroll
            for (int slot = kMemorySlots - 1; slot > 0; --slot) fm.slots[slot] = fm.slots[slot - 1];
            fm.slots[0] = MemoryEntry{static_cast<int16_t>(f.move + 1), memory_level(m, p, f.move), 0, 0};
        }
        if (fm.slots[0].move_plus_one != 0 && fm.slots[0].outcome == 0) {
            for (int k = 0; k < e.contact_count; ++k) {
                if (e.contacts[k].attacker != p) continue;
                switch (e.contacts[k].contact) {
                    case kHit:
                    case kThrowHeld: fm.slots[0].outcome = 1; break;
                    case kCounterHit: fm.slots[0].outcome = 2; break;
                    case kBlocked: fm.slots[0].outcome = 3; break;
                    default: fm.slots[0].outcome = 4; break;
                }
                break;
            }
        }
        const bool idle = f.move < 0;
        const float signals[kMemoryTraces] = {
            f.posture == kCrouching ? 1.0F : 0.0F,
            idle && (f.universal == kWalkBack || f.universal == kBackdash) ? 1.0F : 0.0F,
            idle && (f.universal == kSidestepLeft || f.universal == kSidestepRight) ? 1.0F : 0.0F,
            on(f, fInBlockstun) ? 1.0F : 0.0F,
            f.move >= 0 && f.action_frame >= perception_delay ? 1.0F : 0.0F,
        };
#pragma unroll
        for (int k = 0; k < kMemoryTraces; ++k) fm.traces[k] += (signals[k] - fm.traces[k]) * (1.0F / 60.0F);
        fm.last_move_plus_one = f.move + 1;
        fm.last_action_frame = f.action_frame;
    }
}

// encode_fighter_memory / encode_memory (full_move_contract.hpp:714-735); kMemoryFeatures floats.
T8B_HD void encode_fighter_memory(const FighterMemory& fm, int hide_younger_than, float* out) {
    for (int k = 0; k < kMemoryFighterFeatures; ++k) out[k] = 0.0F;
    int written = 0;
    for (int slot = 0; slot < kMemorySlots && written < kMemorySlots; ++slot) {
        const MemoryEntry& entry = fm.slots[slot];
        if (entry.move_plus_one == 0 || entry.age < hide_younger_than) continue;
        float* at = out + written * kMemorySlotFeatures;
        if (entry.level >= 1 && entry.level <= 5) at[entry.level - 1] = 1.0F;
        if (entry.outcome >= 1 && entry.outcome <= 4) at[4 + entry.outcome] = 1.0F;
        at[9] = c01(entry.age / 180.0);
        ++written;
    }
    for (int k = 0; k < kMemoryTraces; ++k) out[kMemorySlots * kMemorySlotFeatures + k] = fm.traces[k];
}
T8B_HD void encode_memory(const Memory& memory, int player, int perception_delay, float* out) {
    encode_fighter_memory(memory.f[player], 0, out);
    encode_fighter_memory(memory.f[1 - player], perception_delay, out + kMemoryFighterFeatures);
}

// ------------------------------------------------------------------ one decision
struct StepOut {
    float reward, sparse;
    int32_t terminated, outcome, frames;
};

// held_input (full_move_contract.hpp:1062-1065)
T8B_HD bool is_held(const Input& in) {
    return in.move < 0 &&
        (in.universal == kIdle || in.universal == kWalkForward || in.universal == kWalkBack || in.universal == kCrouch);
}

// How the frame loop's threads proceed: each on its own (the loop runs while this thread's
// decision runs), or, in a block whose threads all call the loop, frame by frame together: a
// block barrier at the top of every frame (until the block's last decision ends) and one between
// the scripted opponent's choice and the engine step, a thread whose decision has ended only
// passing the barriers. The warps of an SM then fetch the same code at about the same time,
// which is what bounds the frame loop (instruction fetch). Barriers inside the engine step
// measured slower.
struct FreeFrames {
    T8B_HD bool any(bool running) const { return running; }
    T8B_HD void together() const {}
};
#ifdef __CUDACC__
struct LockstepFrames {
    __device__ __forceinline__ bool any(bool running) const { return __syncthreads_or(running ? 1 : 0) != 0; }
    __device__ __forceinline__ void together() const { __syncthreads(); }
};
#endif

// env_step (full_move_contract.hpp:1071-1154) for a learner on side L. `profiles` is the
// 331-entry bot table; opponent_candidate < 0 means the scripted opponent plays. The side is a
// template argument so that every fighter index in the frame loop is a constant. With `live`
// false the thread runs no frame (it only keeps the frame barriers of a lockstep block).
template <int L, class Frames = FreeFrames>
T8B_HD StepOut decision_as(const Match& m, Fight& s, int learner_candidate, int opponent_candidate, double aggression,
                           const EnvCfg& ec, const Profile* profiles, uint64_t seed, uint64_t stream, uint64_t counter,
                           const Noise* noise, Memory* memory = nullptr, bool live = true, Frames frames = Frames{}) {
    constexpr int learner = L;
    StepOut r{0.0F, 0.0F, 0, 0, 0};
    int lag = 0;
    if (noise != nullptr && noise->latency > 0) {
        lag = noise->latency + (unit(hash3(noise->key, 0x1a7u, counter)) < 0.25 ? 1 : 0);
    }
    constexpr int op = 1 - learner;
    const double max_health = m.cfg->max_health;
    const double own_before = s.f[learner].health;
    const double opp_before = s.f[op].health;
    Input li{-1, kIdle};
    if (!candidate_ok(m, s, learner, learner_candidate) || !to_input(*m.side[learner], learner_candidate, li)) li = Input{-1, kIdle};
    const bool policy_opponent = opponent_candidate >= 0;
    Input oi{-1, kIdle};
    if (policy_opponent && (!candidate_ok(m, s, op, opponent_candidate) || !to_input(*m.side[op], opponent_candidate, oi))) {
        oi = Input{-1, kIdle};
    }
    const bool learner_held = is_held(li);
    const bool opponent_held = policy_opponent && is_held(oi);
    const int bot = bot_id(aggression);
    const uint64_t opponent_prefix = prefix_of(seed, stream);
    Events e;
    int broken = 0;
    double distance_frames = 0.0;
    bool running = live;
    for (int frame = 0; frames.any(running && frame < ec.max_frames_per_decision); ++frame) {
        const bool act = running && frame < ec.max_frames_per_decision;
        const bool landing = frame == lag;
        const bool holding = frame > lag && frame < lag + ec.hold_frames;
        const Input own = landing || (learner_held && holding) ? li : Input{-1, kIdle};
        Input other{-1, kIdle};
        if (!act) {
            // past its decision: only the barriers
        } else if (policy_opponent) {
            if (landing || (opponent_held && holding)) other = oi;
        } else if (decides(m, s, op)) {
            const uint64_t at = counter * 256u + static_cast<uint64_t>(frame);
            const int choice = bot >= 0 ? bot_choice(m, s, op, profiles[bot], seed, stream, opponent_prefix, at)
                                        : random_opponent(m, s, op, aggression, opponent_prefix, at);
            if (!to_input(*m.side[op], choice, other)) other = Input{-1, kIdle};
        }
        frames.together();
        if (!act) continue;
        frame_step(m, s, learner == 0 ? own : other, learner == 0 ? other : own, e);
        if (memory != nullptr) memory_update(m, s, e, ec.perception_delay, *memory);
        ++r.frames;
        distance_frames += mag(s.f[0].x - s.f[1].x);
        for (int k = 0; k < e.contact_count; ++k) {
            if (e.contacts[k].contact == kThrowBroken && e.contacts[k].attacker == learner) ++broken;
        }
        if (s.winner < 0 && s.frame >= ec.max_round_frames) {
            const double oh = s.f[learner].health, th = s.f[op].health;
            s.winner = oh == th ? 2 : (oh > th ? learner : op);
        }
        if (s.winner >= 0) {
            running = false;
            continue;
        }
        const int minimum = ((learner_held || opponent_held) ? ec.hold_frames : 1) + lag;
        if (frame + 1 >= minimum && (decides(m, s, learner) || (policy_opponent && decides(m, s, op)))) running = false;
    }
    const double dealt = opp_before - s.f[op].health;
    const double taken = own_before - s.f[learner].health;
    r.reward = static_cast<float>((dealt * ec.damage_dealt_weight - taken * ec.damage_taken_weight) / max_health) *
            ec.damage_reward -
        static_cast<float>(distance_frames) * (ec.distance_penalty_per_second / 60.0F) -
        static_cast<float>(broken) * ec.throw_break_penalty -
        static_cast<float>(r.frames) * (ec.time_penalty_per_second / 60.0F);
    if (s.winner >= 0) {
        r.terminated = 1;
        r.outcome = s.winner == learner ? 1 : (s.winner == op ? -1 : 0);
        r.sparse = r.outcome == 0 ? -ec.draw_penalty * ec.win_reward : static_cast<float>(r.outcome) * ec.win_reward;
        r.reward += r.sparse;
    }
    return r;
}

T8B_HD StepOut decision(const Match& m, Fight& s, int learner, int learner_candidate, int opponent_candidate,
                        double aggression, const EnvCfg& ec, const Profile* profiles, uint64_t seed, uint64_t stream,
                        uint64_t counter, const Noise* noise, Memory* memory = nullptr) {
    return learner == 0 ? decision_as<0>(m, s, learner_candidate, opponent_candidate, aggression, ec, profiles, seed,
                                         stream, counter, noise, memory)
                        : decision_as<1>(m, s, learner_candidate, opponent_candidate, aggression, ec, profiles, seed,
                                         stream, counter, noise, memory);
}

}  // namespace t8b
