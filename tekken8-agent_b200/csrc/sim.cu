// Batched fight simulator: the GpuFullMoveSimulator contract (include/t8_v2/full_move_gpu.hpp)
// as sm_100a kernels and its C ABI (include/t8b.h, t8b_sim_*).
//
// Per decision the hot path is two launches:
//   k_step   one thread per fight: load the 240 B fight state
//            once, run the whole frame loop of the decision on chip (engine.cuh /
//            contract.cuh), store it, and encode both sides' observations (screen view,
//            live noise) in the same thread;
//   k_masks  one warp per (fight, side): 32 candidates per ballot, 12 ballots cover the
//            368-candidate stride, written as 12 packed words (48 B instead of 368 B).
// reset_done adds k_reset over finished fights (plus k_masks over the same fights only:
// unchanged fights keep identical observations and masks, so recomputing them is skipped).
// Roster tables are repacked at creation into the compact DMove/DHit/DStance layout and
// the per-block character table and engine config are staged in shared memory.
#include "common.cuh"
#include "internal.cuh"
#include "contract.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>

namespace t8b {

thread_local std::string g_last_error;
void set_last_error(const std::string& message) { g_last_error = message; }

static_assert(sizeof(Fight) == sizeof(t8b_state_t), "Fight mirrors t8b_state_t");
static_assert(sizeof(Cfg) == sizeof(t8b_engine_config_t), "Cfg mirrors t8b_engine_config_t");
static_assert(sizeof(EnvCfg) == sizeof(t8b_env_config_t), "EnvCfg mirrors t8b_env_config_t");
static_assert(sizeof(Noise) == sizeof(t8b_noise_levels_t), "Noise mirrors t8b_noise_levels_t");
static_assert(sizeof(Input) == sizeof(t8b_input_t), "Input mirrors t8b_input_t");
static_assert(sizeof(Events) == sizeof(t8b_events_t), "Events mirrors t8b_events_t");
static_assert(sizeof(DMove) == 304, "compact move record");

constexpr int kMaskWords = 12;  // 368 candidates in 32-bit words
constexpr unsigned kStepThreads = 128;
// k_step runs one fight per lane: the decision loop is one dependent chain per fight and its
// lanes diverge, and fewer fights per warp (more warps, narrower path unions) measured slower
// on B200 at 32,768 fights (16 lanes +8 %, 8 lanes +35 % per step). Its blocks hold up to 8
// warps (210 registers per thread, no spills; 9 warps spill) and it runs one block per SM;
// step_grid picks the block size.
constexpr unsigned kStepMaxWarps = 8;
constexpr unsigned kMaskThreads = 256;

// Pointers every kernel needs, passed by value.
struct SimView {
    const DCharacter* chars;
    const Cfg* cfg;
    const EnvCfg* ecfg;
    const Profile* profiles;
    Fight* states;
    int32_t* p1;
    int32_t* p2;
    const uint8_t* learner_is_p1;
    const uint32_t* side_order;  // fights with the learner on P1 first, then on P2
    float* aggression;
    const int32_t* pending_opponents;
    const float* pending_aggression;
    int32_t* scenarios;
    const int32_t* pending_scenarios;
    const int32_t* pending_learners;
    Noise* noise;  // null without live noise
    Memory* memories;  // null without --memory
    float* learner_obs;
    float* opponent_obs;
    int32_t* learner_tables;
    int32_t* opponent_tables;
    uint32_t* learner_bits;
    uint32_t* opponent_bits;
    float* rewards;
    float* sparse;
    uint8_t* terminated;
    int8_t* outcomes;
    unsigned long long* frames;
    uint32_t* tally;
    uint32_t* scenario_tally;
    uint32_t* learner_tally;
    uint32_t* bot_tally;
    int roster;
    int width;  // observation floats per environment
    size_t count;
    size_t first;  // k_masks: the first environment of the range it covers (count environments)
};

// Copies the character table and configs into shared memory; returns the staged view.
struct Staged {
    const DCharacter* chars;
    const Cfg* cfg;
    const EnvCfg* ecfg;
};

__device__ Staged stage_tables(const SimView& v) {
    extern __shared__ __align__(16) unsigned char smem[];
    DCharacter* chars = reinterpret_cast<DCharacter*>(smem);
    Cfg* cfg = reinterpret_cast<Cfg*>(chars + v.roster);
    EnvCfg* ecfg = reinterpret_cast<EnvCfg*>(cfg + 1);
    const uint32_t* src = reinterpret_cast<const uint32_t*>(v.chars);
    uint32_t* dst = reinterpret_cast<uint32_t*>(chars);
    const int words = static_cast<int>(v.roster * sizeof(DCharacter) / 4);
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
    const uint32_t* csrc = reinterpret_cast<const uint32_t*>(v.cfg);
    for (int i = threadIdx.x; i < static_cast<int>(sizeof(Cfg) / 4); i += blockDim.x) reinterpret_cast<uint32_t*>(cfg)[i] = csrc[i];
    const uint32_t* esrc = reinterpret_cast<const uint32_t*>(v.ecfg);
    for (int i = threadIdx.x; i < static_cast<int>(sizeof(EnvCfg) / 4); i += blockDim.x) reinterpret_cast<uint32_t*>(ecfg)[i] = esrc[i];
    __syncthreads();
    return {chars, cfg, ecfg};
}

size_t stage_bytes(int roster) { return roster * sizeof(DCharacter) + sizeof(Cfg) + sizeof(EnvCfg); }

__device__ __forceinline__ Match match_of(const Staged& st, int p1, int p2) {
    Match m;
    m.side[0] = st.chars + p1;
    m.side[1] = st.chars + p2;
    m.cfg = st.cfg;
    return m;
}

// observe_kernel (src/full_move_gpu.cu:131-166): both sides of one fight, the learner on side L.
template <int L>
__device__ void write_observations(const SimView& v, const Staged& st, const Match& m, const Fight& s, size_t env,
                                   int p1, int p2) {
    const EnvCfg& ec = *st.ecfg;
    const int own = L == 0 ? p1 : p2;
    const int other = L == 0 ? p2 : p1;
    float* lo = v.learner_obs + env * static_cast<size_t>(v.width);
    float* oo = v.opponent_obs + env * static_cast<size_t>(v.width);
    float buf[kObservationBase + kMemoryFeatures + 3];
    const int noise_at = kObservationBase + (v.memories != nullptr ? kMemoryFeatures : 0);
#pragma unroll
    for (int side = 0; side < 2; ++side) {
        const int player = side == 0 ? L : 1 - L;
        const int me = side == 0 ? own : other;
        const int them = side == 0 ? other : own;
        observe(m, s, player, ec.max_round_frames, st.chars[me].roster_id, st.chars[them].roster_id, buf,
                ec.perception_delay);
        if (v.memories != nullptr) encode_memory(v.memories[env], player, ec.perception_delay, buf + kObservationBase);
        if (v.noise != nullptr) {
            const Noise n = v.noise[env];
            perturb(n, s, player, buf);
            noise_features(n, buf + noise_at);
        }
        if (ec.screen_view) screen_view(buf);
        float* out = side == 0 ? lo : oo;
        for (int k = 0; k < v.width; ++k) out[k] = buf[k];
    }
    v.learner_tables[env] = own;
    v.opponent_tables[env] = other;
}

__device__ __forceinline__ void write_observations(const SimView& v, const Staged& st, const Match& m, const Fight& s,
                                                   size_t env, int p1, int p2, int learner) {
    if (learner == 0) write_observations<0>(v, st, m, s, env, p1, p2);
    else write_observations<1>(v, st, m, s, env, p1, p2);
}

__device__ __forceinline__ void add_frames(const SimView& v, unsigned long long frames) {
    // one atomic per warp
    for (int offset = 16; offset > 0; offset >>= 1) frames += __shfl_down_sync(0xffffffffu, frames, offset);
    if ((threadIdx.x & 31) == 0 && frames != 0) atomicAdd(v.frames, frames);
}

// One fight's round reset (env_reset_kernel, src/full_move_gpu.cu:231-255): fresh live-noise
// levels, the pending matchup, aggression and scenario, and a new round's state, stored; p1 and
// p2 come back as the new matchup.
__device__ __forceinline__ Fight reset_fight(const SimView& v, const Staged& st, size_t env, uint64_t seed,
                                             uint64_t counter, int& p1, int& p2) {
    if (v.noise != nullptr) v.noise[env] = draw_noise(*st.ecfg, seed, env, counter);
    const bool learner_p1 = v.learner_is_p1[env] != 0;
    if (learner_p1) {
        p2 = v.pending_opponents[env];
        if (v.pending_learners[env] >= 0) p1 = v.pending_learners[env];
    } else {
        p1 = v.pending_opponents[env];
        if (v.pending_learners[env] >= 0) p2 = v.pending_learners[env];
    }
    v.p1[env] = p1;
    v.p2[env] = p2;
    v.aggression[env] = v.pending_aggression[env];
    const int scenario = v.pending_scenarios[env];
    v.scenarios[env] = scenario;
    Fight s;
    start_round(match_of(st, p1, p2), s, *st.ecfg, seed, env, counter, scenario, learner_p1 ? 0 : 1);
    v.states[env] = s;
    if (v.memories != nullptr) v.memories[env] = Memory{};
    return s;
}

// One fight's decision with the learner on side L: the state stays in registers through the
// frame loop (every fighter index is a constant), then the outcome, tallies and observations.
// With `reset`, a fight whose round ended is reset at once (reset_fight with the step's seed
// and counter, as reset_done would do next) and only the new round's observations are written.
// Every thread of the block calls it (the frame loop runs in lockstep); a thread with `live`
// false (past its side's last fight) reads fight `env` but runs no frame and writes nothing.
template <int L>
__device__ __forceinline__ unsigned long long step_fight(const SimView& v, const Staged& st, size_t env,
                                                         const int64_t* learner_candidates,
                                                         const int64_t* opponent_candidates, uint64_t seed,
                                                         uint64_t counter, bool reset, bool live) {
    const int p1 = v.p1[env], p2 = v.p2[env];
    const Match m = match_of(st, p1, p2);
    Fight s = v.states[env];
    const float aggression = v.aggression[env];
    const Noise* noise = v.noise != nullptr ? v.noise + env : nullptr;
    Memory memory;
    Memory* remembered = nullptr;
    if (v.memories != nullptr) {
        memory = v.memories[env];
        remembered = &memory;
    }
    const StepOut r = decision_as<L, LockstepFrames>(
        m, s, static_cast<int>(learner_candidates[env]),
        opponent_candidates != nullptr ? static_cast<int>(opponent_candidates[env]) : -1, aggression, *st.ecfg,
        v.profiles, seed, env, counter, noise, remembered, live);
    if (!live) return 0;
    v.rewards[env] = r.reward;
    v.sparse[env] = r.sparse;
    v.terminated[env] = r.terminated ? 1 : 0;
    v.outcomes[env] = static_cast<int8_t>(r.outcome);
    if (r.terminated) {
        const int opponent_character = L == 0 ? p2 : p1;
        const int bucket = min(4, max(0, static_cast<int>(aggression * 4.0F + 0.5F)));
        const int column = r.outcome > 0 ? 0 : (r.outcome < 0 ? 1 : 2);
        atomicAdd(&v.tally[((opponent_character * 5 + bucket) * 2 + L) * 3 + column], 1u);
        atomicAdd(&v.scenario_tally[v.scenarios[env] * 3 + column], 1u);
        atomicAdd(&v.learner_tally[(L == 0 ? p1 : p2) * 3 + column], 1u);
        const int bot = bot_id(aggression);
        if (bot >= 0 && bot < T8B_SCRIPTED_PROFILES) atomicAdd(&v.bot_tally[bot * 3 + column], 1u);
    }
    int q1 = p1, q2 = p2;
    if (reset && r.terminated) {
        s = reset_fight(v, st, env, seed, counter, q1, q2);
    } else {
        v.states[env] = s;
        if (remembered != nullptr) v.memories[env] = memory;
    }
    write_observations<L>(v, st, match_of(st, q1, q2), s, env, q1, q2);
    return static_cast<unsigned long long>(r.frames);
}

// env_step_kernel (src/full_move_gpu.cu:188-229) with the observation pass fused in.
//
// The frame loop is compiled once per learner side (step_fight<0>, step_fight<1>), and an SM
// that runs both copies at once thrashes its instruction cache. So the grid is one block per
// SM, each block takes the side its SM serves (SMs below the P1 share of the fights serve P1)
// and pulls chunks of that side, one fight per thread (side_order lists P1-learner fights
// first), from a per-side ticket; when its side runs out it helps with the other side.
__global__ void __launch_bounds__(kStepMaxWarps * 32, 1) k_step(SimView v, const int64_t* learner_candidates,
                                                            const int64_t* opponent_candidates, uint64_t seed,
                                                            uint64_t counter, unsigned* tickets, uint32_t p1_fights,
                                                            int reset) {
    const Staged st = stage_tables(v);
    __shared__ unsigned chunk;
    unsigned smid, nsmid;
    asm("mov.u32 %0, %%smid;" : "=r"(smid));
    asm("mov.u32 %0, %%nsmid;" : "=r"(nsmid));
    int side = static_cast<uint64_t>(smid) * v.count < static_cast<uint64_t>(p1_fights) * nsmid ? 0 : 1;
    unsigned long long frames = 0;
    for (int sides_done = 0; sides_done < 2;) {
        __syncthreads();
        if (threadIdx.x == 0) chunk = atomicAdd(tickets + side, 1u);
        __syncthreads();
        const size_t first = static_cast<size_t>(chunk) * blockDim.x;
        const size_t count = side == 0 ? p1_fights : v.count - p1_fights;
        if (first >= count) {
            side ^= 1;
            ++sides_done;
            continue;
        }
        const size_t in_side = first + threadIdx.x;
        const bool live = in_side < count;
        const size_t env = v.side_order[(side == 0 ? 0 : p1_fights) + (live ? in_side : first)];
        frames += side == 0
            ? step_fight<0>(v, st, env, learner_candidates, opponent_candidates, seed, counter, reset != 0, live)
            : step_fight<1>(v, st, env, learner_candidates, opponent_candidates, seed, counter, reset != 0, live);
    }
    add_frames(v, frames);
}

// k_step's launch shape: the fewest waves of one block per SM, then the fewest warps per block
// whose chunks (counted per side, as the blocks take them) fit in those waves, so every SM
// carries about the same number of warps (32,768 fights on 148 SMs: 148 blocks of 7 warps).
// One block of 7 warps per SM measured 9 % faster than two blocks of 4 per SM (108 SMs with 8
// warps, 40 with 4) at 32,768 fights.
struct StepGrid {
    unsigned blocks, threads;
};
inline StepGrid step_grid(size_t fights, size_t p1_fights, int sm_count) {
    const size_t sms = static_cast<size_t>(std::max(sm_count, 1));
    const auto chunks = [&](size_t threads) {
        return (p1_fights + threads - 1) / threads + (fights - p1_fights + threads - 1) / threads;
    };
    for (size_t waves = 1;; ++waves) {
        for (size_t warps = 1; warps <= kStepMaxWarps; ++warps) {
            const size_t c = chunks(warps * 32);
            if (c <= waves * sms) {
                return {static_cast<unsigned>(std::max<size_t>(std::min(c, sms), 1)), static_cast<unsigned>(warps * 32)};
            }
        }
    }
}

// env_reset_kernel (src/full_move_gpu.cu:231-255) with the observation pass fused in.
__global__ void __launch_bounds__(kStepThreads) k_reset(SimView v, const uint8_t* only_done, uint64_t seed,
                                                          uint64_t counter) {
    const Staged st = stage_tables(v);
    const size_t env = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (env >= v.count) return;
    if (only_done != nullptr && !only_done[env]) return;
    int p1 = v.p1[env], p2 = v.p2[env];
    const Fight s = reset_fight(v, st, env, seed, counter, p1, p2);
    write_observations(v, st, match_of(st, p1, p2), s, env, p1, p2, v.learner_is_p1[env] != 0 ? 0 : 1);
}

// Observations of every fight from its stored state (restore).
__global__ void __launch_bounds__(kStepThreads) k_observe(SimView v) {
    const Staged st = stage_tables(v);
    const size_t env = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (env >= v.count) return;
    const int p1 = v.p1[env], p2 = v.p2[env];
    const Fight s = v.states[env];
    write_observations(v, st, match_of(st, p1, p2), s, env, p1, p2, v.learner_is_p1[env] ? 0 : 1);
}

// The first finished round of every fight during an evaluation: the outcome of a fight that
// terminates for the first time is kept and `remaining` drops by one; later rounds are ignored.
__global__ void k_first_outcomes(const uint8_t* terminated, const int8_t* outcomes, size_t count, int8_t* result,
                                 uint8_t* finished, unsigned* remaining) {
    const size_t env = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool first = env < count && terminated[env] && !finished[env];
    if (first) {
        finished[env] = 1;
        result[env] = outcomes[env];
    }
    const uint32_t ballot = __ballot_sync(0xffffffffu, first);
    if ((threadIdx.x & 31) == 0 && ballot != 0) atomicSub(remaining, static_cast<unsigned>(__popc(ballot)));
}

// candidate_mask_kernel (src/full_move_gpu.cu:169-186) as one warp per (fight, side).
// `sides`: 3 both sides (items = 2 x fights), 1 the learner's, 2 the opponent's (items = fights).
__global__ void __launch_bounds__(kMaskThreads) k_masks(SimView v, const uint8_t* only, int sides) {
    const Staged st = stage_tables(v);
    __shared__ Fight fights[kMaskThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t item = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
    const size_t local = sides == 3 ? item >> 1 : item;
    const size_t env = v.first + local;
    const int side = sides == 3 ? static_cast<int>(item & 1) : sides - 1;
    const bool active = local < v.count && (only == nullptr || only[env]);
    if (active) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(v.states + env);
        uint32_t* dst = reinterpret_cast<uint32_t*>(fights + warp);
        for (int i = lane; i < static_cast<int>(sizeof(Fight) / 4); i += 32) dst[i] = src[i];
    }
    __syncwarp();
    if (!active) return;
    const int p1 = v.p1[env], p2 = v.p2[env];
    const Match m = match_of(st, p1, p2);
    const int learner = v.learner_is_p1[env] ? 0 : 1;
    const int player = side == 0 ? learner : 1 - learner;
    const int count = m.side[player]->candidate_count;
    const Fight& s = fights[warp];
    // move candidates: the gate record against the fighter's side of move_allowed, derived once
    const MoveContext context = move_context(m, s, player);
    const uint32_t universal = universal_mask(m, s, player, context.can);
    const DGate* gates = m.side[player]->gates;
    uint32_t mine = 0;
    // unrolled so the twelve gate loads issue together (12 % faster than the rolled loop)
#pragma unroll
    for (int word = 0; word < kMaskWords; ++word) {
        const int c = word * 32 + lane;
        bool legal = false;
        if (c >= kUniversalCount && c < count) {
            const DGate g = gates[c];
            legal = g.move >= 0 && s.winner < 0 &&
                context_allows(context, g.flags, g.required_posture, g.required_stance, g.heat_cost != 0);
        } else if (c < count) {
            legal = (universal >> c) & 1u;  // c < kUniversalCount: word 0
        }
        const uint32_t bits = __ballot_sync(0xffffffffu, legal);
        if (lane == word) mine = bits;
    }
    if (lane < kMaskWords) (side == 0 ? v.learner_bits : v.opponent_bits)[env * kMaskWords + lane] = mine;
}

__global__ void k_expand_masks(const uint32_t* bits, uint8_t* bytes, size_t count) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count * kMaxCandidates) return;
    const size_t env = i / kMaxCandidates;
    const int c = static_cast<int>(i % kMaxCandidates);
    bytes[i] = (bits[env * kMaskWords + (c >> 5)] >> (c & 31)) & 1u;
}

// engine_reset_kernel / engine_step_kernel / legal_mask_kernel (src/full_move_gpu.cu:93-129).
__global__ void k_engine_reset(SimView v, const double* x1, const double* x2) {
    const Staged st = stage_tables(v);
    const size_t env = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (env >= v.count) return;
    Fight s;
    fresh_fight(match_of(st, v.p1[env], v.p2[env]), s, x1[env], x2[env]);
    v.states[env] = s;
}

__global__ void k_engine_step(SimView v, const Input* inputs, const uint8_t* new_round, const double* x1,
                              const double* x2, Events* events) {
    const Staged st = stage_tables(v);
    const size_t env = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    unsigned long long frames = 0;
    if (env < v.count) {
        const Match m = match_of(st, v.p1[env], v.p2[env]);
        Fight s = v.states[env];
        if (new_round != nullptr && new_round[env]) next_round(m, s, x1[env], x2[env]);
        Events e;
        for (int k = 0; k < kMaxContacts; ++k) e.contacts[k] = ContactEvent{0, 0, 0, 0, 0.0};
        for (int k = 0; k < kMaxTransitions; ++k) e.transitions[k] = 0;
        frame_step(m, s, inputs[2 * env], inputs[2 * env + 1], e);
        v.states[env] = s;
        events[env] = e;
        frames = 1;
    }
    add_frames(v, frames);
}

__global__ void k_legal_mask(SimView v, int player, uint8_t* out) {
    const Staged st = stage_tables(v);
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= v.count * kMaxCandidates) return;
    const size_t env = i / kMaxCandidates;
    const int c = static_cast<int>(i % kMaxCandidates);
    const Match m = match_of(st, v.p1[env], v.p2[env]);
    const Fight s = v.states[env];
    out[i] = c < m.side[player]->candidate_count && candidate_ok(m, s, player, c);
}

__global__ void k_draw_noise(SimView v, uint64_t seed) {
    const size_t env = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (env >= v.count) return;
    const EnvCfg ec = *v.ecfg;
    v.noise[env] = draw_noise(ec, seed, env, 0);
}

// ------------------------------------------------------------------ engine-parity workload
// PCG-XSH-RR 64/32 (O'Neill 2014), seeded as pcg32_srandom; bounded draws by Lemire's
// multiply-shift so the draw has no rejection loop.
struct Pcg32 {
    uint64_t state, inc;
    __host__ __device__ Pcg32(uint64_t seed, uint64_t stream) : state(0), inc((stream << 1) | 1u) {
        next();
        state += seed;
        next();
    }
    __host__ __device__ uint32_t next() {
        const uint64_t old = state;
        state = old * 6364136223846793005ull + inc;
        const uint32_t shifted = static_cast<uint32_t>(((old >> 18) ^ old) >> 27);
        const uint32_t rot = static_cast<uint32_t>(old >> 59);
        return (shifted >> rot) | (shifted << ((32u - rot) & 31u));
    }
    __host__ __device__ uint32_t below(uint32_t bound) { return static_cast<uint32_t>((static_cast<uint64_t>(next()) * bound) >> 32); }
};

// FNV-1a over the 60 words of the packed state.
__host__ __device__ inline uint64_t fight_hash(const Fight& s) {
    uint32_t words[sizeof(Fight) / 4];
    memcpy(words, &s, sizeof(Fight));
    uint64_t h = 0xcbf29ce484222325ull;
    for (int i = 0; i < static_cast<int>(sizeof(Fight) / 4); ++i) h = (h ^ words[i]) * 0x100000001b3ull;
    return h;
}

// A uniformly random legal candidate (the harness's pick, tests/full_combat_random_play.hpp), with
// the candidate scan spread over a warp: every lane holds the same fight, lane
// l checks candidates l, l + 32, ...; the legal set is 12 ballot words, and the draw (the same
// PCG32 call on every lane) picks the same candidate index the scalar scan would.
__device__ __forceinline__ Input random_legal_warp(const Match& m, const Fight& s, int p, Pcg32& rng, int lane) {
    const DCharacter& ch = *m.side[p];
    constexpr int kWords = (T8B_MAX_CANDIDATES + 31) / 32;
    // candidate_ok per lane, with the fight's side of it derived once (as k_masks does)
    const MoveContext context = move_context(m, s, p);
    const uint32_t universal = universal_mask(m, s, p, context.can);
    uint32_t bits[kWords];
    int legal = 0;
#pragma unroll
    for (int w = 0; w < kWords; ++w) {
        const int c = w * 32 + lane;
        bool ok = false;
        if (c >= kUniversalCount && c < ch.candidate_count) {
            const DGate g = ch.gates[c];
            ok = g.move >= 0 && s.winner < 0 &&
                context_allows(context, g.flags, g.required_posture, g.required_stance, g.heat_cost != 0);
        } else if (c < ch.candidate_count) {
            ok = (universal >> c) & 1u;
        }
        bits[w] = __ballot_sync(0xffffffffu, ok);
        legal += __popc(bits[w]);
    }
    Input in{-1, kIdle};
    if (legal == 0) return in;
    int pick = static_cast<int>(rng.below(static_cast<uint32_t>(legal)));
#pragma unroll
    for (int w = 0; w < kWords; ++w) {
        const int count = __popc(bits[w]);
        if (pick < count) {
            uint32_t word = bits[w];
            for (int k = 0; k < pick; ++k) word &= word - 1;  // drop the lowest `pick` set bits
            const int c = w * 32 + (__ffs(static_cast<int>(word)) - 1);
            if (!to_input(ch, c, in)) in = Input{-1, kIdle};
            return in;
        }
        pick -= count;
    }
    return in;
}

// The engine-parity workload, one warp per fight. All lanes step the same state (control flow is
// the same on every lane, so the warp never diverges in the frame step), the decisions' legality
// scans are shared out over the lanes, and lane 0 writes the frame's hash. 1,024 fights are 1,024
// warps (about 7 per SM) instead of 32.
__global__ void __launch_bounds__(kStepThreads) k_random_play(SimView v, int fights, const int32_t* p1,
                                                                const int32_t* p2, const double* x1, const double* x2,
                                                                int frames, uint64_t seed, uint64_t* hashes) {
    const Staged st = stage_tables(v);
    const int lane = threadIdx.x & 31;
    const int f = static_cast<int>((static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    if (f < fights) {
        const Match m = match_of(st, p1[f], p2[f]);
        Pcg32 rng(seed, static_cast<uint64_t>(f));
        Fight s;
        fresh_fight(m, s, x1[f], x2[f]);
        Events e;
        uint64_t* out = hashes + static_cast<size_t>(f) * frames;
        for (int frame = 0; frame < frames; ++frame) {
            if (s.winner >= 0) next_round(m, s, x1[f], x2[f]);
            Input chosen[2] = {{-1, kIdle}, {-1, kIdle}};
            for (int p = 0; p < 2; ++p) {
                if (decides(m, s, p)) chosen[p] = random_legal_warp(m, s, p, rng, lane);
            }
            frame_step(m, s, chosen[0], chosen[1], e);
            if (lane == 0) out[frame] = fight_hash(s);
        }
        if (lane == 0) atomicAdd(v.frames, static_cast<unsigned long long>(frames));
    }
}

// ------------------------------------------------------------------ host: tables

// scripted_profile / generated_profile (include/t8_v2/full_move_contract.hpp:157-268), evaluated
// once on the host; the same IEEE float/double operations as the device would run.
Profile make_profile(int id) {
    Profile p{};
    p.tier = 0; p.fixed = -1; p.aggression = 0.0F; p.block = 0.0F; p.reaction = 99; p.punish = 0.0F;
    p.throw_break = 0.0F; p.sidestep = 0.0F; p.smart = 0.0F; p.distance = 1.0F; p.keepaway = 0.0F;
    p.low_bias = 0.0F; p.throw_bias = 0.0F; p.heat_use = 0.0F; p.movement = 0.3F; p.pressure = 0.0F;
    constexpr int kHandmade = 30, kTiers = 7, kPerTier = 43;
    if (id >= kHandmade) {
        const int index = id - kHandmade;
        p.tier = std::min(kTiers - 1, index / kPerTier);
        uint64_t state = 0x9e3779b97f4a7c15ull * static_cast<uint64_t>(id + 1) + 0x632be59bd9b4e5f5ull;
        auto next = [&]() {
            state = mix64(state + 0x9e3779b97f4a7c15ull);
            return static_cast<double>(state >> 11) * (1.0 / 9007199254740992.0);
        };
        auto vary = [&](double value, double low, double high) { return clampd(value * (0.9 + 0.2 * next()), low, high); };
        static const double table[kTiers][6] = {
            {0.00, 99, 0.00, 0.00, 0.00, 0.10}, {0.05, 40, 0.05, 0.08, 0.00, 0.20}, {0.42, 22, 0.30, 0.35, 0.02, 0.50},
            {0.68, 17, 0.60, 0.58, 0.10, 0.75}, {0.80, 15, 0.74, 0.72, 0.25, 0.82}, {0.91, 12, 0.90, 0.87, 0.38, 0.95},
            {0.97, 9, 0.98, 0.95, 0.50, 1.00}};
        const double* skill = table[p.tier];
        p.block = static_cast<float>(vary(skill[0], 0.0, 0.98));
        p.reaction = static_cast<int>(clampd(skill[1] + (next() * 4.0 - 2.0), 8.0, 99.0));
        p.punish = static_cast<float>(vary(skill[2], 0.0, 0.99));
        p.throw_break = static_cast<float>(vary(skill[3], 0.0, 0.98));
        p.sidestep = static_cast<float>(vary(skill[4], 0.0, 0.8));
        p.smart = static_cast<float>(vary(skill[5], 0.0, 1.0));
        const int style = static_cast<int>(next() * (p.tier >= 4 ? 9.0 : 8.0));
        p.aggression = static_cast<float>(0.35 + 0.5 * next());
        p.distance = static_cast<float>(0.85 + 0.3 * next());
        p.movement = static_cast<float>(0.1 + 0.5 * next());
        switch (style) {
            case 0: p.aggression = static_cast<float>(0.75 + 0.25 * next()); p.distance = 0.85F; break;
            case 1:
                p.aggression = static_cast<float>(0.3 + 0.2 * next());
                p.distance = 1.15F;
                p.block = static_cast<float>(lo(0.98, p.block + 0.1));
                p.punish = static_cast<float>(lo(0.99, p.punish + 0.1));
                break;
            case 2:
                p.distance = static_cast<float>(1.6 + 0.4 * next());
                p.keepaway = static_cast<float>(0.5 + 0.4 * next());
                break;
            case 3:
                p.sidestep = static_cast<float>(lo(0.9, p.sidestep + 0.25 + 0.15 * next()));
                p.movement = 0.7F;
                break;
            case 4:
                p.low_bias = static_cast<float>(0.8 + 1.2 * next());
                p.throw_bias = static_cast<float>(0.4 + 0.8 * next());
                break;
            case 5: p.heat_use = static_cast<float>(0.6 + 0.4 * next()); break;
            case 6: p.throw_bias = static_cast<float>(1.5 + 1.5 * next()); p.distance = 0.85F; break;
            case 7: p.low_bias = static_cast<float>(1.5 + 1.5 * next()); break;
            default:
                p.pressure = static_cast<float>(0.5 + 0.4 * next());
                p.aggression = static_cast<float>(0.7 + 0.2 * next());
                break;
        }
        if (p.tier == 0) {
            p.aggression = static_cast<float>(0.05 + 0.15 * next());
            p.block = p.punish = p.throw_break = p.sidestep = p.pressure = 0.0F;
            p.reaction = 99;
        }
        if (p.tier == 5 && next() < 0.5) p.pressure = static_cast<float>(hi(p.pressure, 0.3 + 0.4 * next()));
        if (p.tier == 6) p.pressure = static_cast<float>(hi(p.pressure, 0.4 + 0.4 * next()));
        return p;
    }
    auto skill = [&](int tier, float block, int reaction, float punish, float breaks, float side, float smart) {
        p.tier = tier; p.block = block; p.reaction = reaction; p.punish = punish; p.throw_break = breaks;
        p.sidestep = side; p.smart = smart;
    };
    auto rushdown = [&]() { p.aggression = 0.85F; p.distance = 0.85F; p.movement = 0.2F; };
    auto turtle = [&]() {
        p.aggression = 0.4F; p.distance = 1.15F;
        p.block = static_cast<float>(lo(0.98, p.block + 0.1));
        p.punish = static_cast<float>(lo(0.98, p.punish + 0.1));
    };
    auto keepaway = [&]() { p.aggression = 0.45F; p.distance = 1.8F; p.keepaway = 0.7F; };
    auto sidestepper = [&]() {
        p.aggression = 0.5F; p.distance = 1.1F;
        p.sidestep = static_cast<float>(lo(0.9, p.sidestep + 0.3));
        p.movement = 0.6F;
    };
    auto mixup = [&]() { p.aggression = 0.65F; p.distance = 0.95F; p.low_bias = 1.5F; p.throw_bias = 0.8F; };
    auto heat_user = [&]() { p.aggression = 0.6F; p.distance = 1.0F; p.heat_use = 1.0F; };
    const float t2[6] = {0.42F, 22, 0.30F, 0.35F, 0.02F, 0.50F};
    const float t3[6] = {0.68F, 17, 0.60F, 0.58F, 0.10F, 0.75F};
    const float t4[6] = {0.80F, 15, 0.74F, 0.72F, 0.25F, 0.82F};
    const float t5[6] = {0.91F, 12, 0.90F, 0.87F, 0.38F, 0.95F};
    const float t6[6] = {0.97F, 9, 0.98F, 0.95F, 0.50F, 1.0F};
    auto tier_skill = [&](int tier, const float* t) {
        skill(tier, t[0], static_cast<int>(t[1]), t[2], t[3], t[4], t[5]);
    };
    switch (id) {
        case 0: p.tier = 0; p.fixed = 1; break;
        case 1: p.tier = 0; p.fixed = 0; break;
        case 2: p.tier = 0; p.fixed = 5; break;
        case 3: p.tier = 1; p.aggression = 1.0F; p.distance = 1.0F; break;
        case 4: p.tier = 1; p.aggression = 0.8F; p.low_bias = 3.0F; p.smart = 0.3F; break;
        case 5: p.tier = 1; p.aggression = 0.7F; p.distance = 0.8F; p.throw_bias = 3.0F; p.smart = 0.3F; break;
        case 6: p.tier = 1; p.aggression = 0.4F; p.distance = 2.0F; p.keepaway = 0.8F; break;
        case 7: tier_skill(2, t2); rushdown(); break;
        case 8: tier_skill(2, t2); turtle(); break;
        case 9: tier_skill(2, t2); keepaway(); break;
        case 10: tier_skill(2, t2); mixup(); break;
        case 11: tier_skill(3, t3); rushdown(); break;
        case 12: tier_skill(3, t3); turtle(); break;
        case 13: tier_skill(3, t3); keepaway(); break;
        case 14: tier_skill(3, t3); sidestepper(); break;
        case 15: tier_skill(3, t3); mixup(); break;
        case 16: tier_skill(3, t3); heat_user(); break;
        case 17: tier_skill(4, t4); rushdown(); break;
        case 18: tier_skill(4, t4); turtle(); break;
        case 19: tier_skill(4, t4); keepaway(); break;
        case 20: tier_skill(4, t4); sidestepper(); break;
        case 21: tier_skill(4, t4); mixup(); break;
        case 22: tier_skill(4, t4); heat_user(); break;
        case 23: tier_skill(5, t5); rushdown(); break;
        case 24: tier_skill(5, t5); turtle(); break;
        case 25: tier_skill(5, t5); mixup(); p.heat_use = 0.7F; break;
        case 26: tier_skill(6, t6); keepaway(); p.distance = 1.7F; p.pressure = 0.3F; break;
        case 27: tier_skill(6, t6); rushdown(); p.pressure = 0.85F; p.heat_use = 1.0F; break;
        case 28: tier_skill(6, t6); turtle(); p.pressure = 0.4F; break;
        default:
            tier_skill(6, t6); mixup(); p.sidestep = 0.6F; p.pressure = 0.6F; p.heat_use = 0.8F;
            break;
    }
    return p;
}

struct HostRoster {
    std::vector<DMove> moves;
    std::vector<DHit> hits;
    std::vector<DStance> stances;
    std::vector<int2> spans;
    std::vector<int32_t> candidate_moves;
    std::vector<DFacts> facts;
    std::vector<DGate> gates;
    struct Offsets { size_t move, hit, stance, candidate; };
    std::vector<Offsets> offsets;
    std::vector<int32_t> roster_ids;
};

DMove compact_move(const t8b_move_t& m, const t8b_hit_t* hits, int hit_count, std::vector<int2>& spans) {
    DMove d;
    std::memset(&d, 0, sizeof d);
    d.flags = m.flags;
    d.hit_offset = m.hit_offset; d.hit_count = m.hit_count; d.total_frames = m.total_frames; d.recovery = m.recovery;
    d.block_advantage = m.block_advantage; d.hit_advantage = m.hit_advantage;
    d.counter_hit_advantage = m.counter_hit_advantage; d.launch_air_frames = m.launch_air_frames;
    d.back_turned_hit_advantage = m.back_turned_hit_advantage;
    d.heat_dash_block_advantage = m.heat_dash_block_advantage; d.heat_dash_hit_advantage = m.heat_dash_hit_advantage;
    d.heat_cost_frames = m.heat_cost_frames; d.required_stance = m.required_stance; d.result_stance = m.result_stance;
    d.result_stance_on_hit = m.result_stance_on_hit; d.result_stance_on_block = m.result_stance_on_block;
    for (int i = 0; i < 4; ++i) d.parry_outcomes[i] = m.parry_outcomes[i];
    d.heat_parry_outcome = m.heat_parry_outcome;
    if (m.hit_count < 0 || (m.hit_count > 0 && (m.hit_offset < 0 || m.hit_offset + m.hit_count > hit_count))) {
        raise(T8B_EINVAL, "a move's hits lie outside its character's hit table");
    }
    d.approach_frames = m.hit_count == 0 ? 0 : hits[m.hit_offset].first_active_frame - 1;
    d.hit_effect = m.hit_effect; d.counter_hit_effect = m.counter_hit_effect;
    d.back_turned_hit_effect = m.back_turned_hit_effect; d.heat_dash_hit_effect = m.heat_dash_hit_effect;
    d.required_posture = m.required_posture; d.attack_throw = m.attack_throw;
    d.parry_levels = m.parry_levels; d.heat_parry_levels = m.heat_parry_levels;
    d.travel = m.travel; d.pushback_hit = m.pushback_hit; d.pushback_block = m.pushback_block;
    d.reversal_damage = m.reversal_damage; d.attack_throw_damage = m.attack_throw_damage;
    d.recoverable_damage = m.recoverable_damage; d.rage_art_max_damage = m.rage_art_max_damage;
    d.self_damage = m.self_damage; d.self_recoverable = m.self_recoverable; d.restore_health_hit = m.restore_health_hit;
    d.restore_recoverable_hit = m.restore_recoverable_hit; d.restore_recoverable_block = m.restore_recoverable_block;
    d.resource_gain_start = m.resource_gain_start; d.resource_gain_hit = m.resource_gain_hit;
    d.resource_gain_airborne_hit = m.resource_gain_airborne_hit; d.resource_gain_block = m.resource_gain_block;
    d.resource_gain_heat_activation = m.resource_gain_heat_activation;
    d.install_damage_bonus = m.install_damage_bonus; d.install_chip_damage = m.install_chip_damage;
    d.install_reach = m.install_reach;
    for (int w = 0; w < 9; ++w) {
        const t8b_window_t& win = m.windows[w];
        if (win.count < 0 || win.count > T8B_MAX_WINDOW_SPANS) raise(T8B_EINVAL, "a move window has too many spans");
        const uint32_t first = static_cast<uint32_t>(spans.size());
        for (int k = 0; k < win.count; ++k) spans.push_back(make_int2(win.first[k], win.last[k]));
        d.windows[w] = (first << 4) | static_cast<uint32_t>(win.count);
    }
    return d;
}

// MoveFacts of every candidate (include/t8_v2/full_move_contract.hpp:292-313).
DFacts candidate_facts(const t8b_character_t& ch, int candidate) {
    DFacts out{0.0, 0.0, 0ull, 99, 0u};
    if (candidate < kUniversalCount || candidate >= ch.candidate_count) return out;
    const int move = ch.candidate_moves[candidate];
    if (move < 0) return out;
    const t8b_move_t& m = ch.moves[move];
    out.flags = m.flags;
    if (m.block_advantage >= -9) out.bits |= 2u;
    if (m.hit_effect == kLaunch) out.bits |= 4u;
    for (int k = 0; k < m.hit_count; ++k) {
        const t8b_hit_t& h = ch.hits[m.hit_offset + k];
        out.damage += h.damage;
        if (k == 0) {
            out.startup = h.first_active_frame;
            out.reach = h.reach;
            if (h.level == kLow || h.level == kSpecialLow) out.bits |= 8u;
            if (h.level == kThrow) out.bits |= 16u;
        }
    }
    if (m.hit_count > 0) out.bits |= 1u;
    return out;
}

// The legality inputs of a move candidate (DGate); universal candidates and gaps get move -1.
DGate candidate_gate(const t8b_character_t& ch, int candidate) {
    DGate g;
    std::memset(&g, 0, sizeof g);
    g.move = -1;
    const int move = candidate >= kUniversalCount ? ch.candidate_moves[candidate] : -1;
    if (move < 0) return g;
    if (move > 32767) raise(T8B_EINVAL, "a candidate's move index exceeds 32767");
    const t8b_move_t& m = ch.moves[move];
    g.flags = m.flags;
    g.required_stance = m.required_stance;
    g.required_posture = m.required_posture;
    g.heat_cost = m.heat_cost_frames != 0 ? 1 : 0;
    g.move = static_cast<int16_t>(move);
    return g;
}

// Repacks the boundary tables into the device layout (host vectors; the caller uploads).
HostRoster pack_roster(const t8b_character_t* roster, int roster_count) {
    HostRoster host;
    host.moves.push_back(DMove{});  // index -1 of the first character reads this record
    std::memset(&host.moves.front(), 0, sizeof(DMove));
    for (int c = 0; c < roster_count; ++c) {
        const t8b_character_t& ch = roster[c];
        if (ch.move_count < 0 || ch.hit_count < 0 || ch.stance_count < 0 || ch.candidate_count < 0 ||
            ch.candidate_count > T8B_MAX_CANDIDATES) {
            raise(T8B_EINVAL, "character table sizes are invalid");
        }
        host.offsets.push_back({host.moves.size(), host.hits.size(), host.stances.size(), host.candidate_moves.size()});
        for (int k = 0; k < ch.move_count; ++k) host.moves.push_back(compact_move(ch.moves[k], ch.hits, ch.hit_count, host.spans));
        for (int k = 0; k < ch.hit_count; ++k) {
            const t8b_hit_t& h = ch.hits[k];
            DHit d;
            std::memset(&d, 0, sizeof d);
            d.level = h.level; d.throw_break = h.throw_break; d.flags = h.flags;
            d.first_active_frame = h.first_active_frame; d.active_frames = h.active_frames;
            d.damage = h.damage; d.reach = h.reach; d.tracking_left = h.tracking_left;
            d.tracking_right = h.tracking_right; d.chip_damage = h.chip_damage; d.heat_chip_damage = h.heat_chip_damage;
            host.hits.push_back(d);
        }
        for (int k = 0; k < ch.stance_count; ++k) {
            const t8b_stance_t& s = ch.stances[k];
            DStance d;
            std::memset(&d, 0, sizeof d);
            d.can_guard = s.can_guard; d.has_max_frames = s.has_max_frames; d.auto_parry = s.auto_parry;
            d.max_frames = s.max_frames;
            for (int i = 0; i < 4; ++i) d.parry_outcomes[i] = s.parry_outcomes[i];
            d.pulse_interval_frames = s.pulse_interval_frames; d.pulse_recoverable = s.pulse_recoverable;
            d.pulse_resource = s.pulse_resource;
            host.stances.push_back(d);
        }
        for (int k = 0; k < ch.candidate_count; ++k) {
            if (ch.candidate_moves[k] >= ch.move_count) raise(T8B_EINVAL, "a candidate names a missing move");
            host.candidate_moves.push_back(ch.candidate_moves[k]);
            host.facts.push_back(candidate_facts(ch, k));
            host.gates.push_back(candidate_gate(ch, k));
        }
        host.roster_ids.push_back(ch.roster_id);
    }
    return host;
}

}  // namespace t8b

using namespace t8b;

struct t8b_sim {
    cudaStream_t stream = nullptr;
    size_t n = 0;
    int roster = 0;
    int width = 0;
    t8b_env_config_t config{};
    Buffer<DMove> moves;
    Buffer<DHit> hits;
    Buffer<DStance> stances;
    Buffer<int2> spans;
    Buffer<int32_t> candidate_moves;
    Buffer<DFacts> facts;
    Buffer<DGate> gates;
    Buffer<DCharacter> chars;
    Buffer<Cfg> cfg;
    Buffer<EnvCfg> ecfg;
    Buffer<Profile> profiles;
    Buffer<Fight> states;
    Buffer<Events> events;
    Buffer<Input> inputs;
    Buffer<uint8_t> new_round;
    Buffer<double> x1, x2;
    Buffer<int32_t> p1, p2, pending_opponents, pending_learners, scenarios, pending_scenarios;
    Buffer<uint8_t> learner_is_p1, terminated, truncated;
    Buffer<uint32_t> side_order;
    int sm_count = 1;
    Buffer<float> aggression, pending_aggression;
    Buffer<Noise> noise;
    Buffer<Memory> memories;  // config.memory only
    Buffer<float> learner_obs, opponent_obs;
    Buffer<int32_t> learner_tables, opponent_tables;
    Buffer<uint32_t> learner_bits, opponent_bits;
    bool opponent_bits_stale = true;
    Buffer<uint8_t> learner_bytes, opponent_bytes, legal_bytes;
    Buffer<float> rewards, sparse;
    Buffer<int8_t> outcomes;
    Buffer<unsigned long long> frames;
    Buffer<uint32_t> tally, scenario_tally, learner_tally, bot_tally;
    std::vector<int32_t> host_roster_ids;

    SimView view() const {
        SimView v{};
        v.chars = chars.data(); v.cfg = cfg.data(); v.ecfg = ecfg.data(); v.profiles = profiles.data();
        v.states = states.data(); v.p1 = p1.data(); v.p2 = p2.data(); v.learner_is_p1 = learner_is_p1.data();
        v.side_order = side_order.data();
        v.aggression = aggression.data(); v.pending_opponents = pending_opponents.data();
        v.pending_aggression = pending_aggression.data(); v.scenarios = scenarios.data();
        v.pending_scenarios = pending_scenarios.data(); v.pending_learners = pending_learners.data();
        v.noise = config.live_noise ? noise.data() : nullptr;
        v.memories = config.memory ? memories.data() : nullptr;
        v.learner_obs = learner_obs.data(); v.opponent_obs = opponent_obs.data();
        v.learner_tables = learner_tables.data(); v.opponent_tables = opponent_tables.data();
        v.learner_bits = learner_bits.data(); v.opponent_bits = opponent_bits.data();
        v.rewards = rewards.data(); v.sparse = sparse.data(); v.terminated = terminated.data();
        v.outcomes = outcomes.data(); v.frames = frames.data(); v.tally = tally.data();
        v.scenario_tally = scenario_tally.data(); v.learner_tally = learner_tally.data(); v.bot_tally = bot_tally.data();
        v.roster = roster; v.width = width; v.count = n;
        return v;
    }
    size_t smem() const { return stage_bytes(roster); }

    // Fight groups: the environments split into contiguous ranges that can be stepped on separate
    // streams (one group, all fights, unless the native rollout loop asks for more). Each group's
    // slice of side_order lists its fights with the learner on P1 first, then those on P2 (each in
    // index order), and has its own pair of k_step tickets.
    std::vector<uint8_t> host_sides;
    std::vector<size_t> group_first, group_count;
    std::vector<uint32_t> group_p1;
    Buffer<unsigned> group_tickets;

    void build_order(int groups) {
        groups = std::max(1, std::min<int>(groups, static_cast<int>(n)));
        if (host_sides.size() != n) host_sides.assign(n, 1);
        group_first.assign(static_cast<size_t>(groups), 0);
        group_count.assign(static_cast<size_t>(groups), 0);
        group_p1.assign(static_cast<size_t>(groups), 0);
        std::vector<uint32_t> order;
        order.reserve(n);
        for (int g = 0; g < groups; ++g) {
            const size_t first = n * static_cast<size_t>(g) / static_cast<size_t>(groups);
            const size_t last = n * static_cast<size_t>(g + 1) / static_cast<size_t>(groups);
            group_first[g] = first;
            group_count[g] = last - first;
            for (size_t i = first; i < last; ++i) if (host_sides[i]) order.push_back(static_cast<uint32_t>(i));
            group_p1[g] = static_cast<uint32_t>(order.size() - first);
            for (size_t i = first; i < last; ++i) if (!host_sides[i]) order.push_back(static_cast<uint32_t>(i));
        }
        if (side_order.size() < n) side_order.allocate(n);
        side_order.upload(order.data(), n, stream);
        if (group_tickets.size() < 2 * static_cast<size_t>(groups)) group_tickets.allocate(2 * static_cast<size_t>(groups));
        check(cudaStreamSynchronize(stream), "fight order");
    }
    int groups() const { return static_cast<int>(group_first.size()); }

    // Learner sides from the host, plus the fight order k_step walks.
    void set_sides(const uint8_t* host) {
        learner_is_p1.upload(host, n, stream);
        host_sides.assign(host, host + n);
        build_order(std::max(1, groups()));
    }

    // env_step over one group's fights on `st` (k_step, then the learner's masks of the group).
    void step_group(int g, const int64_t* learner, const int64_t* opponent, uint64_t seed, uint64_t counter, bool reset,
                    cudaStream_t st, bool with_masks = true) {
        SimView v = view();
        v.side_order = side_order.data() + group_first[g];
        v.count = group_count[g];
        unsigned* tickets = group_tickets.data() + 2 * static_cast<size_t>(g);
        check(cudaMemsetAsync(tickets, 0, 2 * sizeof(unsigned), st), "step tickets");
        const StepGrid grid = step_grid(group_count[g], group_p1[g], sm_count);
        launch("k_step", k_step, grid.blocks, grid.threads, smem(), st, v, learner, opponent, seed, counter, tickets,
               group_p1[g], reset ? 1 : 0);
        launched("step");
        opponent_bits_stale = true;
        if (!with_masks) return;
        v.first = group_first[g];
        const unsigned warps_per_block = kMaskThreads / 32;
        launch("k_masks", k_masks, blocks(group_count[g], warps_per_block), kMaskThreads, smem(), st, v,
               static_cast<const uint8_t*>(nullptr), 1);
        launched("candidate masks");
        opponent_bits_stale = true;
    }
    void launched(const char* what) const { check(cudaGetLastError(), what); }
    // k_masks' grid over `items` (fight, side) items: one warp each
    unsigned mask_grid(size_t items) const { return blocks(items, kMaskThreads / 32); }

    // The learner's masks after every state change; the opponent's are computed when asked for
    // (opponent_bits_stale), which a scripted-opponent trainer never does.
    void masks(const uint8_t* only) {
        const unsigned warps_per_block = kMaskThreads / 32;
        launch("k_masks", k_masks, blocks(n, warps_per_block), kMaskThreads, smem(), stream, view(), only, 1);
        launched("candidate masks");
        opponent_bits_stale = true;
    }
    const uint32_t* opponent_mask_bits() {
        if (opponent_bits_stale) {
            const unsigned warps_per_block = kMaskThreads / 32;
            launch("k_masks", k_masks, blocks(n, warps_per_block), kMaskThreads, smem(), stream, view(), nullptr, 2);
            launched("opponent masks");
            opponent_bits_stale = false;
        }
        return opponent_bits.data();
    }
    void check_characters(const int32_t* values, bool allow_keep, const char* what) const {
        for (size_t i = 0; i < n; ++i) {
            if (values[i] < (allow_keep ? -1 : 0) || values[i] >= roster) raise(T8B_ERANGE, what);
        }
    }
};

namespace {

template <typename Body>
int with_sim(t8b_sim* sim, Body&& body) {
    return guarded([&] {
        if (sim == nullptr) raise(T8B_EINVAL, "null simulator handle");
        body(*sim);
    });
}

}  // namespace

extern "C" {

const char* t8b_last_error(void) { return t8b::g_last_error.c_str(); }

int t8b_device_count(int* out) {
    return guarded([&] { check(cudaGetDeviceCount(out), "cudaGetDeviceCount"); });
}

void t8b_engine_config_default(t8b_engine_config_t* c) {
    std::memset(c, 0, sizeof *c);
    c->half_width = 3.6; c->body_radius = 0.22; c->walk_speed = 0.025; c->dash_distance = 0.7; c->dash_frames = 18;
    c->backdash_distance = 0.6; c->backdash_frames = 22; c->sidestep_distance = 0.5; c->sidestep_frames = 18;
    c->axis_realign_per_frame = 0.03; c->launch_air_frames = 60; c->juggle_window_frames = 22;
    c->juggle_window_decay = 1; c->tornado_extra_frames = 40; c->knockdown_frames = 24; c->wakeup_stand_frames = 30;
    c->wakeup_roll_frames = 24; c->wakeup_roll_distance = 0.8; c->tech_window_frames = 6; c->tech_roll_frames = 20;
    c->wall_splat_frames = 20; c->crumple_frames = 70; c->stage_break_air_frames = 55; c->wall_break_extension = 3.6;
    c->combo_scale_step = 0.10; c->combo_scale_floor = 0.30; c->counter_hit_damage_scale = 1.2;
    c->throw_break_window = 20; c->throw_break_recovery = 20; c->parry_outcome_frames = 30;
    c->side_exposure_ratio = 0.5; c->back_to_wall_distance = 0.3; c->ki_charge_frames = 300;
    c->ki_charge_damage_scale = 1.10; c->parry_stun_frames = 40; c->reversal_recovery = 30;
    c->heat_duration_frames = 600; c->heat_dash_frames = 20; c->heat_dash_distance = 1.2;
    c->rage_health_fraction = 0.25; c->rage_damage_scale = 1.10; c->wall_combo_scale = 0.70;
    c->recoverable_regain_hit = 0.50; c->recoverable_regain_block = 0.25; c->max_health = 180.0;
}

void t8b_env_config_default(t8b_env_config_t* c) {
    std::memset(c, 0, sizeof *c);
    c->max_round_frames = 3600; c->hold_frames = 4; c->max_frames_per_decision = 120;
    c->damage_reward = 1.0F; c->win_reward = 1.0F; c->damage_dealt_weight = 1.0F; c->damage_taken_weight = 1.0F;
    c->noise_position_max = 0.25F; c->noise_flip_max = 0.10F; c->latency_min = 2; c->latency_max = 6;
    c->start_center_range = 1.2; c->start_distance_min = 0.8; c->start_distance_max = 2.4;
}

int t8b_sim_create(const t8b_character_t* roster, int roster_count, const t8b_engine_config_t* engine,
                   size_t environments, const t8b_env_config_t* config, t8b_sim** out) {
    return guarded([&] {
        if (out == nullptr || engine == nullptr || config == nullptr) raise(T8B_EINVAL, "null argument");
        *out = nullptr;
        if (roster == nullptr || roster_count <= 0 || environments == 0) {
            raise(T8B_EINVAL, "full-move simulator needs characters and environments");
        }
        if (config->max_round_frames <= 0 || config->hold_frames <= 0 ||
            config->max_frames_per_decision < config->hold_frames ||
            !(config->start_distance_max >= config->start_distance_min) || !(config->start_distance_min > 0.0)) {
            raise(T8B_EINVAL, "full-move environment configuration is invalid");
        }
        auto sim = std::make_unique<t8b_sim>();
        sim->n = environments;
        {
            int device = 0;
            check(cudaGetDevice(&device), "cudaGetDevice");
            check(cudaDeviceGetAttribute(&sim->sm_count, cudaDevAttrMultiProcessorCount, device), "SM count");
        }
        sim->roster = roster_count;
        sim->config = *config;
        sim->width = kObservationBase + (config->memory ? kMemoryFeatures : 0) + (config->live_noise ? T8B_NOISE_FEATURES : 0);
        const size_t n = environments;

        HostRoster host = pack_roster(roster, roster_count);
        sim->host_roster_ids = host.roster_ids;
        if (host.spans.empty()) host.spans.push_back(make_int2(0, -1));
        if (host.hits.empty()) host.hits.push_back(DHit{});
        if (host.stances.empty()) host.stances.push_back(DStance{});
        if (host.candidate_moves.empty()) host.candidate_moves.push_back(-1);
        if (host.facts.empty()) host.facts.push_back(DFacts{});
        if (host.gates.empty()) host.gates.push_back(DGate{});
        cudaStream_t s = sim->stream;
        sim->moves.allocate(host.moves.size()); sim->moves.upload(host.moves.data(), host.moves.size(), s);
        sim->hits.allocate(host.hits.size()); sim->hits.upload(host.hits.data(), host.hits.size(), s);
        sim->stances.allocate(host.stances.size()); sim->stances.upload(host.stances.data(), host.stances.size(), s);
        sim->spans.allocate(host.spans.size()); sim->spans.upload(host.spans.data(), host.spans.size(), s);
        sim->candidate_moves.allocate(host.candidate_moves.size());
        sim->candidate_moves.upload(host.candidate_moves.data(), host.candidate_moves.size(), s);
        sim->facts.allocate(host.facts.size()); sim->facts.upload(host.facts.data(), host.facts.size(), s);
        sim->gates.allocate(host.gates.size()); sim->gates.upload(host.gates.data(), host.gates.size(), s);
        std::vector<DCharacter> chars;
        for (int c = 0; c < roster_count; ++c) {
            const auto& off = host.offsets[static_cast<size_t>(c)];
            DCharacter d{};
            d.moves = sim->moves.data() + off.move;
            d.hits = sim->hits.data() + off.hit;
            d.stances = sim->stances.data() + off.stance;
            d.spans = sim->spans.data();
            d.candidate_moves = sim->candidate_moves.data() + off.candidate;
            d.facts = sim->facts.data() + off.candidate;
            d.gates = sim->gates.data() + off.candidate;
            d.move_count = roster[c].move_count;
            d.stance_count = roster[c].stance_count;
            d.candidate_count = roster[c].candidate_count;
            d.move_candidate_inverse = roster[c].candidate_count > kUniversalCount ? 1.0 / (roster[c].candidate_count - kUniversalCount) : 0.0;
            d.roster_id = roster[c].roster_id;
            d.rules.resource_max = roster[c].rules.resource_max;
            d.rules.install_threshold = roster[c].rules.install_threshold;
            d.rules.has_install_threshold = roster[c].rules.has_install_threshold;
            d.rules.resource_persists = roster[c].rules.resource_persists;
            chars.push_back(d);
        }
        sim->chars.allocate(chars.size()); sim->chars.upload(chars.data(), chars.size(), s);
        Cfg cfg;
        std::memcpy(&cfg, engine, sizeof cfg);
        sim->cfg.allocate(1); sim->cfg.upload(&cfg, 1, s);
        EnvCfg ecfg;
        std::memcpy(&ecfg, config, sizeof ecfg);
        sim->ecfg.allocate(1); sim->ecfg.upload(&ecfg, 1, s);
        std::vector<Profile> profiles;
        for (int id = 0; id < T8B_SCRIPTED_PROFILES; ++id) profiles.push_back(make_profile(id));
        sim->profiles.allocate(profiles.size()); sim->profiles.upload(profiles.data(), profiles.size(), s);

        sim->states.allocate(n); sim->events.allocate(n); sim->inputs.allocate(2 * n); sim->new_round.allocate(n);
        sim->x1.allocate(n); sim->x2.allocate(n);
        sim->p1.allocate(n); sim->p2.allocate(n); sim->pending_opponents.allocate(n);
        sim->pending_learners.allocate(n); sim->scenarios.allocate(n); sim->pending_scenarios.allocate(n);
        sim->learner_is_p1.allocate(n); sim->terminated.allocate(n); sim->truncated.allocate(n);
        sim->aggression.allocate(n); sim->pending_aggression.allocate(n);
        if (config->memory) sim->memories.allocate(n);
        if (config->live_noise) sim->noise.allocate(n);
        sim->learner_obs.allocate(n * static_cast<size_t>(sim->width));
        sim->opponent_obs.allocate(n * static_cast<size_t>(sim->width));
        sim->learner_tables.allocate(n); sim->opponent_tables.allocate(n);
        sim->learner_bits.allocate(n * kMaskWords); sim->opponent_bits.allocate(n * kMaskWords);
        sim->rewards.allocate(n); sim->sparse.allocate(n); sim->outcomes.allocate(n);
        sim->frames.allocate(1);
        sim->tally.allocate(static_cast<size_t>(roster_count) * T8B_AGGRESSION_BUCKETS * 2 * 3);
        sim->scenario_tally.allocate(T8B_SCENARIOS * 3);
        sim->learner_tally.allocate(static_cast<size_t>(roster_count) * 3);
        sim->bot_tally.allocate(T8B_SCRIPTED_PROFILES * 3);
        const std::vector<int32_t> keep(n, -1);
        sim->pending_learners.upload(keep.data(), n, s);
        const std::vector<uint8_t> p1_learners(n, 1);
        sim->set_sides(p1_learners.data());
        const std::vector<double> left(n, -0.8), right(n, 0.8);
        sim->x1.upload(left.data(), n, s);
        sim->x2.upload(right.data(), n, s);
        launch("k_engine_reset", k_engine_reset, blocks(n, kStepThreads), kStepThreads, sim->smem(), s, sim->view(), sim->x1.data(), sim->x2.data());
        sim->launched("initial reset");
        check(cudaStreamSynchronize(s), "create simulator");
        *out = sim.release();
    });
}

int t8b_sim_destroy(t8b_sim* sim) {
    return guarded([&] {
        if (sim != nullptr) cudaStreamSynchronize(sim->stream);
        delete sim;
    });
}

int t8b_sim_set_stream(t8b_sim* sim, void* stream) {
    return with_sim(sim, [&](t8b_sim& s) { s.stream = static_cast<cudaStream_t>(stream); });
}

size_t t8b_sim_environment_count(const t8b_sim* sim) { return sim ? sim->n : 0; }
int t8b_sim_observation_size(const t8b_sim* sim) { return sim ? sim->width : 0; }

int t8b_sim_set_matchups(t8b_sim* sim, const int32_t* p1, const int32_t* p2) {
    return with_sim(sim, [&](t8b_sim& s) {
        if (p1 == nullptr || p2 == nullptr) raise(T8B_EINVAL, "one matchup per environment is required");
        s.check_characters(p1, false, "P1 character");
        s.check_characters(p2, false, "P2 character");
        s.p1.upload(p1, s.n, s.stream);
        s.p2.upload(p2, s.n, s.stream);
        check(cudaStreamSynchronize(s.stream), "set matchups");
    });
}

int t8b_sim_reset_engine(t8b_sim* sim, const double* p1_x, const double* p2_x) {
    return with_sim(sim, [&](t8b_sim& s) {
        s.x1.upload(p1_x, s.n, s.stream);
        s.x2.upload(p2_x, s.n, s.stream);
        launch("k_engine_reset", k_engine_reset, blocks(s.n, kStepThreads), kStepThreads, s.smem(), s.stream, s.view(), s.x1.data(), s.x2.data());
        s.launched("engine reset");
        check(cudaStreamSynchronize(s.stream), "engine reset");
    });
}

int t8b_sim_step_engine(t8b_sim* sim, const t8b_input_t* inputs, const uint8_t* new_round, const double* p1_x,
                        const double* p2_x) {
    return with_sim(sim, [&](t8b_sim& s) {
        s.inputs.upload(reinterpret_cast<const Input*>(inputs), 2 * s.n, s.stream);
        const bool rounds = new_round != nullptr;
        if (rounds) {
            s.new_round.upload(new_round, s.n, s.stream);
            s.x1.upload(p1_x, s.n, s.stream);
            s.x2.upload(p2_x, s.n, s.stream);
        }
        launch("k_engine_step", k_engine_step, blocks(s.n, kStepThreads), kStepThreads, s.smem(), s.stream, 
            s.view(), s.inputs.data(), rounds ? s.new_round.data() : nullptr, s.x1.data(), s.x2.data(), s.events.data());
        s.launched("engine step");
        check(cudaStreamSynchronize(s.stream), "engine step");
    });
}

int t8b_sim_download_states(t8b_sim* sim, t8b_state_t* out) {
    return with_sim(sim, [&](t8b_sim& s) { s.states.download(reinterpret_cast<Fight*>(out), s.n, s.stream); });
}

int t8b_sim_download_events(t8b_sim* sim, t8b_events_t* out) {
    return with_sim(sim, [&](t8b_sim& s) { s.events.download(reinterpret_cast<Events*>(out), s.n, s.stream); });
}

int t8b_sim_upload_states(t8b_sim* sim, const t8b_state_t* states) {
    return with_sim(sim, [&](t8b_sim& s) {
        s.states.upload(reinterpret_cast<const Fight*>(states), s.n, s.stream);
        check(cudaStreamSynchronize(s.stream), "upload states");
    });
}

int t8b_sim_download_legal_mask(t8b_sim* sim, int player, uint8_t* out) {
    return with_sim(sim, [&](t8b_sim& s) {
        if (player != 0 && player != 1) raise(T8B_ERANGE, "player must be 0 or 1");
        if (s.legal_bytes.size() == 0) s.legal_bytes.allocate(s.n * kMaxCandidates);
        launch("k_legal_mask", k_legal_mask, blocks(s.n * kMaxCandidates, 256), 256, s.smem(), s.stream, s.view(), player, s.legal_bytes.data());
        s.launched("legal mask");
        s.legal_bytes.download(out, s.n * kMaxCandidates, s.stream);
    });
}

int t8b_sim_set_learner_sides(t8b_sim* sim, const uint8_t* learner_is_p1) {
    return with_sim(sim, [&](t8b_sim& s) {
        s.set_sides(learner_is_p1);
    });
}

int t8b_sim_set_pending_opponents(t8b_sim* sim, const int32_t* characters, const float* aggression,
                                  const int32_t* scenarios) {
    return with_sim(sim, [&](t8b_sim& s) {
        s.check_characters(characters, false, "opponent");
        s.pending_opponents.upload(characters, s.n, s.stream);
        if (aggression == nullptr) {
            const std::vector<float> half(s.n, 0.5F);
            s.pending_aggression.upload(half.data(), s.n, s.stream);
            check(cudaStreamSynchronize(s.stream), "set pending opponents");
        } else {
            s.pending_aggression.upload(aggression, s.n, s.stream);
        }
        if (scenarios == nullptr) {
            const std::vector<int32_t> neutral(s.n, 0);
            s.pending_scenarios.upload(neutral.data(), s.n, s.stream);
            check(cudaStreamSynchronize(s.stream), "set pending opponents");
        } else {
            for (size_t i = 0; i < s.n; ++i) {
                if (scenarios[i] < 0 || scenarios[i] >= T8B_SCENARIOS) raise(T8B_ERANGE, "scenario");
            }
            s.pending_scenarios.upload(scenarios, s.n, s.stream);
        }
        check(cudaStreamSynchronize(s.stream), "set pending opponents");
    });
}

int t8b_sim_set_pending_learners(t8b_sim* sim, const int32_t* characters) {
    return with_sim(sim, [&](t8b_sim& s) {
        if (characters == nullptr) raise(T8B_EINVAL, "one learner per environment is required");
        s.check_characters(characters, true, "learner");
        s.pending_learners.upload(characters, s.n, s.stream);
        check(cudaStreamSynchronize(s.stream), "set pending learners");
    });
}

int t8b_sim_reset_all(t8b_sim* sim, uint64_t seed, uint64_t counter) {
    return with_sim(sim, [&](t8b_sim& s) {
        launch("k_reset", k_reset, blocks(s.n, kStepThreads), kStepThreads, s.smem(), s.stream, s.view(), nullptr, seed, counter);
        s.launched("reset all");
        s.terminated.zero(s.stream);
        s.masks(nullptr);
    });
}

int t8b_sim_reset_done(t8b_sim* sim, uint64_t seed, uint64_t counter) {
    return with_sim(sim, [&](t8b_sim& s) {
        launch("k_reset", k_reset, blocks(s.n, kStepThreads), kStepThreads, s.smem(), s.stream, s.view(), s.terminated.data(), seed, counter);
        s.launched("reset done");
        s.masks(s.terminated.data());
    });
}

namespace t8b {
static int step_launch(t8b_sim* sim, const int64_t* learner, const int64_t* opponent, uint64_t seed, uint64_t counter,
                bool reset) {
    return with_sim(sim, [&](t8b_sim& s) {
        if (learner == nullptr) raise(T8B_EINVAL, "learner candidates are required");
        for (int g = 0; g < s.groups(); ++g) s.step_group(g, learner, opponent, seed, counter, reset, s.stream);
    });
}
}  // namespace t8b

}  // extern "C"

namespace t8b::internal {

void sim_set_groups(t8b_sim* sim, int groups) {
    if (sim->groups() != groups) sim->build_order(groups);
}
size_t sim_group_first(const t8b_sim* sim, int group) { return sim->group_first[static_cast<size_t>(group)]; }
size_t sim_group_count(const t8b_sim* sim, int group) { return sim->group_count[static_cast<size_t>(group)]; }
void sim_step_group(t8b_sim* sim, int group, const int64_t* learner, const int64_t* opponent, uint64_t seed,
                    uint64_t counter, bool reset, cudaStream_t stream) {
    if (learner == nullptr) raise(T8B_EINVAL, "learner candidates are required");
    if (group < 0 || group >= sim->groups()) raise(T8B_ERANGE, "fight group");
    sim->step_group(group, learner, opponent, seed, counter, reset, stream);
}
void sim_step_without_masks(t8b_sim* sim, const int64_t* learner, const int64_t* opponent, uint64_t seed,
                            uint64_t counter, bool reset, cudaStream_t stream) {
    if (learner == nullptr) raise(T8B_EINVAL, "learner candidates are required");
    if (sim->groups() != 1) raise(T8B_ESTATE, "the fights are split into groups");
    sim->step_group(0, learner, opponent, seed, counter, reset, stream, false);
}
void sim_learner_masks(t8b_sim* sim, cudaStream_t stream) {
    launch("k_masks", k_masks, sim->mask_grid(sim->n), kMaskThreads, sim->smem(), stream, sim->view(),
           static_cast<const uint8_t*>(nullptr), 1);
    check(cudaGetLastError(), "candidate masks");
}

}  // namespace t8b::internal

extern "C" {

int t8b_sim_step(t8b_sim* sim, const int64_t* learner, const int64_t* opponent, uint64_t seed, uint64_t counter) {
    return t8b::step_launch(sim, learner, opponent, seed, counter, false);
}

int t8b_sim_step_and_reset(t8b_sim* sim, const int64_t* learner, const int64_t* opponent, uint64_t seed,
                           uint64_t counter) {
    return t8b::step_launch(sim, learner, opponent, seed, counter, true);
}

const float* t8b_sim_learner_observations(const t8b_sim* sim) { return sim ? sim->learner_obs.data() : nullptr; }
const float* t8b_sim_opponent_observations(const t8b_sim* sim) { return sim ? sim->opponent_obs.data() : nullptr; }
const uint32_t* t8b_sim_learner_mask_bits(const t8b_sim* sim) { return sim ? sim->learner_bits.data() : nullptr; }
const uint32_t* t8b_sim_opponent_mask_bits(const t8b_sim* sim) {
    if (sim == nullptr) return nullptr;
    const uint32_t* bits = nullptr;
    // the view is filled on first use after a state change (the handle is logically const)
    const int status = with_sim(const_cast<t8b_sim*>(sim), [&](t8b_sim& s) { bits = s.opponent_mask_bits(); });
    return status == T8B_OK ? bits : nullptr;
}

static const uint8_t* expand(t8b_sim* sim, bool learner) {
    const uint8_t* result = nullptr;
    const int status = with_sim(sim, [&](t8b_sim& s) {
        Buffer<uint8_t>& bytes = learner ? s.learner_bytes : s.opponent_bytes;
        if (bytes.size() == 0) bytes.allocate(s.n * kMaxCandidates);
        launch("k_expand_masks", k_expand_masks, blocks(s.n * kMaxCandidates, 256), 256, 0, s.stream, 
            learner ? s.learner_bits.data() : s.opponent_mask_bits(), bytes.data(), s.n);
        s.launched("expand masks");
        result = bytes.data();
    });
    return status == T8B_OK ? result : nullptr;
}

const uint8_t* t8b_sim_learner_masks(t8b_sim* sim) { return expand(sim, true); }
const uint8_t* t8b_sim_opponent_masks(t8b_sim* sim) { return expand(sim, false); }
const float* t8b_sim_rewards(const t8b_sim* sim) { return sim ? sim->rewards.data() : nullptr; }
const float* t8b_sim_sparse_rewards(const t8b_sim* sim) { return sim ? sim->sparse.data() : nullptr; }
const uint8_t* t8b_sim_terminated(const t8b_sim* sim) { return sim ? sim->terminated.data() : nullptr; }
const uint8_t* t8b_sim_truncated(const t8b_sim* sim) { return sim ? sim->truncated.data() : nullptr; }
const int8_t* t8b_sim_outcomes(const t8b_sim* sim) { return sim ? sim->outcomes.data() : nullptr; }
const int32_t* t8b_sim_learner_feature_tables(const t8b_sim* sim) { return sim ? sim->learner_tables.data() : nullptr; }
const int32_t* t8b_sim_opponent_feature_tables(const t8b_sim* sim) { return sim ? sim->opponent_tables.data() : nullptr; }

int t8b_sim_download_noise_levels(t8b_sim* sim, t8b_noise_levels_t* out) {
    return with_sim(sim, [&](t8b_sim& s) {
        if (!s.config.live_noise) raise(T8B_ESTATE, "live noise is off");
        s.noise.download(reinterpret_cast<Noise*>(out), s.n, s.stream);
    });
}

int t8b_sim_frames_simulated(t8b_sim* sim, uint64_t* out) {
    return with_sim(sim, [&](t8b_sim& s) {
        unsigned long long value = 0;
        s.frames.download(&value, 1, s.stream);
        *out = value;
    });
}

int t8b_sim_record_first_outcomes(t8b_sim* sim, int8_t* result, uint8_t* finished, uint32_t* remaining) {
    return with_sim(sim, [&](t8b_sim& s) {
        if (!result || !finished || !remaining) raise(T8B_EINVAL, "first-outcome buffers are required");
        launch("k_first_outcomes", k_first_outcomes, blocks(s.n, 256), 256, 0, s.stream, s.terminated.data(),
               s.outcomes.data(), s.n, result, finished, remaining);
        s.launched("first outcomes");
    });
}

int t8b_sim_download_and_clear_tally(t8b_sim* sim, uint32_t* tally, uint32_t* scenario_tally, uint32_t* learner_tally,
                                     uint32_t* bot_tally) {
    return with_sim(sim, [&](t8b_sim& s) {
        std::vector<uint32_t> scratch;
        auto grab = [&](Buffer<uint32_t>& buffer, uint32_t* out) {
            if (out != nullptr) {
                buffer.download(out, buffer.size(), s.stream);
            }
            buffer.zero(s.stream);
        };
        grab(s.tally, tally);
        grab(s.scenario_tally, scenario_tally);
        grab(s.learner_tally, learner_tally);
        grab(s.bot_tally, bot_tally);
        check(cudaStreamSynchronize(s.stream), "clear tallies");
    });
}

int t8b_sim_snapshot(t8b_sim* sim, t8b_state_t* states, int32_t* p1, int32_t* p2, uint8_t* learner_is_p1,
                     float* aggression, int32_t* pending_opponents, float* pending_aggression, uint8_t* terminated,
                     int32_t* scenarios, int32_t* pending_scenarios, int32_t* pending_learners) {
    return with_sim(sim, [&](t8b_sim& s) {
        s.states.download(reinterpret_cast<Fight*>(states), s.n, s.stream);
        s.p1.download(p1, s.n, s.stream);
        s.p2.download(p2, s.n, s.stream);
        s.learner_is_p1.download(learner_is_p1, s.n, s.stream);
        s.aggression.download(aggression, s.n, s.stream);
        s.pending_opponents.download(pending_opponents, s.n, s.stream);
        s.pending_aggression.download(pending_aggression, s.n, s.stream);
        s.terminated.download(terminated, s.n, s.stream);
        s.scenarios.download(scenarios, s.n, s.stream);
        s.pending_scenarios.download(pending_scenarios, s.n, s.stream);
        s.pending_learners.download(pending_learners, s.n, s.stream);
    });
}

// restore (src/full_move_gpu.cu:657-682): noise levels are redrawn with seed 0x5eed.
int t8b_sim_restore(t8b_sim* sim, const t8b_state_t* states, const int32_t* p1, const int32_t* p2,
                    const uint8_t* learner_is_p1, const float* aggression, const int32_t* pending_opponents,
                    const float* pending_aggression, const uint8_t* terminated, const int32_t* scenarios,
                    const int32_t* pending_scenarios, const int32_t* pending_learners) {
    return with_sim(sim, [&](t8b_sim& s) {
        s.check_characters(p1, false, "P1 character");
        s.check_characters(p2, false, "P2 character");
        s.check_characters(pending_opponents, false, "opponent");
        s.check_characters(pending_learners, true, "learner");
        s.p1.upload(p1, s.n, s.stream);
        s.p2.upload(p2, s.n, s.stream);
        s.states.upload(reinterpret_cast<const Fight*>(states), s.n, s.stream);
        s.set_sides(learner_is_p1);
        s.aggression.upload(aggression, s.n, s.stream);
        s.pending_opponents.upload(pending_opponents, s.n, s.stream);
        s.pending_aggression.upload(pending_aggression, s.n, s.stream);
        s.scenarios.upload(scenarios, s.n, s.stream);
        s.pending_scenarios.upload(pending_scenarios, s.n, s.stream);
        s.pending_learners.upload(pending_learners, s.n, s.stream);
        s.terminated.upload(terminated, s.n, s.stream);
        if (s.config.live_noise) {
            launch("k_draw_noise", k_draw_noise, blocks(s.n, 256), 256, 0, s.stream, s.view(), 0x5eedull);
            s.launched("draw noise levels");
        }
        if (s.config.memory) s.memories.zero(s.stream);  // memory is not part of a snapshot: it restarts empty
        launch("k_observe", k_observe, blocks(s.n, kStepThreads), kStepThreads, s.smem(), s.stream, s.view());
        s.launched("observe");
        s.masks(nullptr);
        check(cudaStreamSynchronize(s.stream), "restore");
    });
}

int t8b_sim_synchronize(t8b_sim* sim) {
    return with_sim(sim, [&](t8b_sim& s) { check(cudaStreamSynchronize(s.stream), "synchronize simulator"); });
}

int t8b_sim_random_play(t8b_sim* sim, int fights, const int32_t* p1, const int32_t* p2, const double* p1_x,
                        const double* p2_x, int frames, uint64_t seed, uint64_t* hashes, uint64_t* frames_done) {
    return with_sim(sim, [&](t8b_sim& s) {
        if (fights <= 0 || frames <= 0 || !p1 || !p2 || !p1_x || !p2_x || !hashes) raise(T8B_EINVAL, "random play arguments");
        launch("k_random_play", k_random_play, blocks(static_cast<size_t>(fights) * 32, kStepThreads), kStepThreads, s.smem(), s.stream, 
            s.view(), fights, p1, p2, p1_x, p2_x, frames, seed, hashes);
        s.launched("random play");
        if (frames_done != nullptr) *frames_done = static_cast<uint64_t>(fights) * static_cast<uint64_t>(frames);
    });
}

}  // extern "C"
