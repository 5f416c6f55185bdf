/*
 * t8b.h - C ABI of the B200-native self-play hot path (simulator, policy, rollout).
 *
 * Every entry point is plain C: opaque handles, plain pointers and sizes, int status
 * codes. Host pointers are read during the call only; device pointers are borrowed for
 * the call and must address memory on the handle's device. A pointer returned by a
 * `*_view` function stays valid until the next mutating call on the same handle.
 *
 * The C++ classes of the reference (t8::v2::GpuFullMoveSimulator,
 * t8::v2::GpuActorCritic, t8::v2::GpuRolloutBuffer) map one method to one entry
 * point here; each declaration names the reference member it replaces.
 *
 * Status codes: 0 ok; T8B_EINVAL (std::invalid_argument in the reference),
 * T8B_ERANGE (std::out_of_range), T8B_ECUDA (std::runtime_error from a CUDA call),
 * T8B_ENONFINITE (std::runtime_error on non-finite data), T8B_ESTATE
 * (std::logic_error). t8b_last_error() gives the message of the calling thread's
 * last failure.
 */
#ifndef T8B_H
#define T8B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    T8B_OK = 0,
    T8B_EINVAL = 1,
    T8B_ERANGE = 2,
    T8B_ECUDA = 3,
    T8B_ENONFINITE = 4,
    T8B_ESTATE = 5,
};

enum { T8B_UNIVERSAL_COUNT = 22, T8B_MAX_CANDIDATES = 368, T8B_FEATURE_SIZE = 32, T8B_ROSTER_SLOTS = 42 };
enum { T8B_STATE_FEATURES = 64, T8B_NOISE_FEATURES = 3, T8B_MAX_WINDOW_SPANS = 8, T8B_MAX_CONTACTS = 8 };
enum { T8B_SCRIPTED_PROFILES = 331, T8B_SCENARIOS = 9, T8B_AGGRESSION_BUCKETS = 5 };

/* ------------------------------------------------------------------ tables
 * One fighter's compiled move tables, field for field the values of the reference's
 * full_core::Move / Hit / Stance / Rules (include/t8_v2/full_combat_core.hpp:37-171)
 * and FullEngineConfig (include/t8_v2/full_combat_engine.hpp:236-289). Enumerations
 * are their uint8 values. The library repacks them into its own device layout. */

typedef struct t8b_window {
    int32_t count;
    int32_t first[T8B_MAX_WINDOW_SPANS];
    int32_t last[T8B_MAX_WINDOW_SPANS];
} t8b_window_t;

typedef struct t8b_hit {
    uint8_t level;       /* FullHitLevel: High Mid Low SpecialMid SpecialLow Throw */
    uint8_t throw_break; /* FullThrowBreak: None One Two OneTwo OneOrTwo */
    uint16_t flags;      /* homing, ground hit, wall splat, wall break, floor break, balcony break,
                            tornado, spike, unparryable, reversal break, has heat chip */
    int32_t first_active_frame;
    int32_t active_frames;
    double damage, reach, tracking_left, tracking_right, chip_damage, heat_chip_damage;
} t8b_hit_t;

typedef struct t8b_move {
    uint64_t flags; /* the 35 move flags of full_core::MoveFlag, same bit positions */
    int32_t hit_offset, hit_count, total_frames, recovery, block_advantage, hit_advantage;
    int32_t counter_hit_advantage, launch_air_frames, back_turned_hit_advantage;
    int32_t heat_dash_block_advantage, heat_dash_hit_advantage, heat_cost_frames;
    int32_t required_stance, result_stance, result_stance_on_hit, result_stance_on_block;
    int32_t parry_outcomes[4];
    int32_t heat_parry_outcome;
    uint8_t hit_effect, counter_hit_effect, back_turned_hit_effect, heat_dash_hit_effect;
    uint8_t required_posture, attack_throw, parry_levels, heat_parry_levels;
    double travel, pushback_hit, pushback_block, reversal_damage, attack_throw_damage;
    double recoverable_damage, rage_art_max_damage, self_damage, self_recoverable;
    double restore_health_hit, restore_recoverable_hit, restore_recoverable_block;
    double resource_gain_start, resource_gain_hit, resource_gain_airborne_hit, resource_gain_block;
    double resource_gain_heat_activation, install_damage_bonus, install_chip_damage, install_reach;
    /* high crush, low crush, power crush, armor, parry, reversal, invincible, airborne, heat parry */
    t8b_window_t windows[9];
} t8b_move_t;

typedef struct t8b_stance {
    uint8_t can_guard, has_max_frames, auto_parry, pad;
    int32_t max_frames;
    int32_t parry_outcomes[4];
    int32_t pulse_interval_frames;
    double pulse_recoverable, pulse_resource;
} t8b_stance_t;

typedef struct t8b_rules {
    double resource_max;
    double install_threshold;
    uint8_t has_install_threshold, resource_persists, install_consumes, pad[5];
} t8b_rules_t;

typedef struct t8b_engine_config {
    double half_width, body_radius, walk_speed, dash_distance;
    int32_t dash_frames;
    int32_t backdash_frames;
    double backdash_distance, sidestep_distance;
    int32_t sidestep_frames;
    int32_t launch_air_frames;
    double axis_realign_per_frame;
    int32_t juggle_window_frames, juggle_window_decay, tornado_extra_frames, knockdown_frames;
    int32_t wakeup_stand_frames, wakeup_roll_frames;
    double wakeup_roll_distance;
    int32_t tech_window_frames, tech_roll_frames, wall_splat_frames, crumple_frames, stage_break_air_frames;
    int32_t pad0;
    double wall_break_extension, combo_scale_step, combo_scale_floor, counter_hit_damage_scale;
    int32_t throw_break_window, throw_break_recovery, parry_outcome_frames;
    int32_t pad1;
    double side_exposure_ratio, back_to_wall_distance;
    int32_t ki_charge_frames;
    int32_t pad2;
    double ki_charge_damage_scale;
    int32_t parry_stun_frames, reversal_recovery, heat_duration_frames, heat_dash_frames;
    double heat_dash_distance, rage_health_fraction, rage_damage_scale, wall_combo_scale;
    double recoverable_regain_hit, recoverable_regain_block, max_health;
} t8b_engine_config_t;

/* One roster character: FullMoveCharacter (include/t8_v2/full_move_roster.hpp:56-67) with
 * its side-0 tables. candidate_features is [candidate_count, 32]. */
typedef struct t8b_character {
    const t8b_move_t* moves;
    const t8b_hit_t* hits;
    const t8b_stance_t* stances;
    const int32_t* candidate_moves;
    const float* candidate_features;
    int32_t move_count, hit_count, stance_count, candidate_count;
    int32_t roster_id;
    int32_t pad;
    t8b_rules_t rules;
} t8b_character_t;

/* ------------------------------------------------------------------ state
 * full_core::State (include/t8_v2/full_combat_core.hpp:179-228) in a packed form: the
 * fighter's bools are bits of `flags`, in this order. */
enum {
    T8B_F_HEAT = 1u << 0, T8B_F_HEAT_AVAILABLE = 1u << 1, T8B_F_RAGE = 1u << 2, T8B_F_RAGE_AVAILABLE = 1u << 3,
    T8B_F_THROW_BREAK_ATTEMPTED = 1u << 4, T8B_F_INSTALLED = 1u << 5, T8B_F_MOVE_HIT = 1u << 6,
    T8B_F_MOVE_BLOCKED = 1u << 7, T8B_F_RESOURCE_GAINED = 1u << 8, T8B_F_BACK_TURNED = 1u << 9,
    T8B_F_MOVE_IN_HEAT = 1u << 10, T8B_F_KI_CHARGE_BOOST = 1u << 11, T8B_F_MOVE_BOOSTED = 1u << 12,
    T8B_F_IN_BLOCKSTUN = 1u << 13, T8B_F_TORNADO_USED = 1u << 14, T8B_F_WALL_SPLAT_USED = 1u << 15,
    T8B_F_WALL_SCALED = 1u << 16, T8B_F_TECHABLE = 1u << 17, T8B_F_CRUMPLED = 1u << 18,
};
enum {
    T8B_S_LEFT_WALL_BREAKABLE = 1u << 0, T8B_S_RIGHT_WALL_BREAKABLE = 1u << 1, T8B_S_LEFT_BALCONY = 1u << 2,
    T8B_S_RIGHT_BALCONY = 1u << 3, T8B_S_FLOOR_BREAKABLE = 1u << 4,
};

typedef struct t8b_fighter {
    double health, recoverable_health, x, axis, resource;
    uint8_t posture, universal;
    int8_t heat_dash_from;
    uint8_t pad;
    uint32_t flags;
    int32_t stance, heat_frames, throw_break_frames, pending_throw_hit, pending_throw_elapsed;
    int32_t move, action_frame;
    uint32_t hits_landed;
    int32_t stance_frames, ki_charge_frames, stun, posture_frames, grounded_elapsed, combo_hits;
} t8b_fighter_t; /* 104 bytes */

typedef struct t8b_state {
    t8b_fighter_t fighters[2];
    double left_wall, right_wall;
    uint32_t stage_flags;
    int32_t stage_level;
    int32_t frame, winner;
} t8b_state_t; /* 240 bytes */

typedef struct t8b_input {
    int32_t move;      /* -1: the universal action */
    int32_t universal; /* FullUniversal */
} t8b_input_t;

typedef struct t8b_contact {
    int32_t attacker, hit_index, contact, pad;
    double damage;
} t8b_contact_t;

typedef struct t8b_events {
    int32_t contact_count, transition_count;
    t8b_contact_t contacts[T8B_MAX_CONTACTS];
    uint8_t transitions[4];
    uint8_t heat_activated[2], rage_activated[2];
} t8b_events_t;

/* full_core::EnvConfig (include/t8_v2/full_move_contract.hpp:737-773). */
typedef struct t8b_env_config {
    int32_t max_round_frames, hold_frames, max_frames_per_decision;
    float damage_reward, win_reward, draw_penalty, throw_break_penalty, time_penalty_per_second;
    float damage_dealt_weight, damage_taken_weight, distance_penalty_per_second;
    int32_t perception_delay;
    uint8_t memory, live_noise, screen_view, pad;
    float noise_position_max, noise_flip_max;
    int32_t latency_min, latency_max;
    int32_t pad2;
    double start_center_range, start_distance_min, start_distance_max;
} t8b_env_config_t;

/* full_core::NoiseLevels (include/t8_v2/full_move_contract.hpp:787-792). */
typedef struct t8b_noise_levels {
    float position_sigma, flip_rate;
    int32_t latency;
    uint32_t key;
} t8b_noise_levels_t;

/* Fills defaults equal to the reference's default member initialisers. */
void t8b_engine_config_default(t8b_engine_config_t* out);
void t8b_env_config_default(t8b_env_config_t* out);

const char* t8b_last_error(void);
int t8b_device_count(int* out);

/* ------------------------------------------------------------------ simulator
 * class GpuFullMoveSimulator (include/t8_v2/full_move_gpu.hpp:42-141). */
typedef struct t8b_sim t8b_sim;

/* GpuFullMoveSimulator(roster, environments, config)  full_move_gpu.hpp:44-45 */
int t8b_sim_create(const t8b_character_t* roster, int roster_count, const t8b_engine_config_t* engine,
                   size_t environments, const t8b_env_config_t* config, t8b_sim** out);
int t8b_sim_destroy(t8b_sim* sim);
/* Stream for every following call (the reference always uses the default stream). */
int t8b_sim_set_stream(t8b_sim* sim, void* stream);
size_t t8b_sim_environment_count(const t8b_sim* sim);            /* full_move_gpu.hpp:52 */
int t8b_sim_observation_size(const t8b_sim* sim);                /* full_move_gpu.hpp:58 */
/* set_matchups  full_move_gpu.hpp:61 (host arrays [environments]) */
int t8b_sim_set_matchups(t8b_sim* sim, const int32_t* p1_characters, const int32_t* p2_characters);
/* reset_engine / step_engine / download_states / download_events / upload_states /
 * download_legal_mask  full_move_gpu.hpp:64-74 (host arrays) */
int t8b_sim_reset_engine(t8b_sim* sim, const double* p1_x, const double* p2_x);
int t8b_sim_step_engine(t8b_sim* sim, const t8b_input_t* inputs, const uint8_t* new_round, const double* p1_x,
                        const double* p2_x);
int t8b_sim_download_states(t8b_sim* sim, t8b_state_t* out);
int t8b_sim_download_events(t8b_sim* sim, t8b_events_t* out);
int t8b_sim_upload_states(t8b_sim* sim, const t8b_state_t* states);
int t8b_sim_download_legal_mask(t8b_sim* sim, int player, uint8_t* out);
/* set_learner_sides / set_pending_opponents / set_pending_learners  full_move_gpu.hpp:79-86.
 * aggression and scenarios may be NULL (0.5 and neutral, as the reference). */
int t8b_sim_set_learner_sides(t8b_sim* sim, const uint8_t* learner_is_p1);
int t8b_sim_set_pending_opponents(t8b_sim* sim, const int32_t* characters, const float* aggression,
                                  const int32_t* scenarios);
int t8b_sim_set_pending_learners(t8b_sim* sim, const int32_t* characters);
/* reset_all / reset_done / step  full_move_gpu.hpp:87-93. learner/opponent candidates are
 * device int64 [environments]; opponent NULL = scripted opponent. */
int t8b_sim_reset_all(t8b_sim* sim, uint64_t seed, uint64_t counter);
int t8b_sim_reset_done(t8b_sim* sim, uint64_t seed, uint64_t counter);
int t8b_sim_step(t8b_sim* sim, const int64_t* learner_candidates, const int64_t* opponent_candidates, uint64_t seed,
                 uint64_t counter);
/* No reference counterpart: t8b_sim_step followed by t8b_sim_reset_done with the same seed and
 * counter, in one launch sequence. A fight whose round ends is reset inside the step, so its
 * terminal observations are never written; states, matchups, noise levels, rewards,
 * terminations, outcomes, tallies, and the observations and masks after the call equal those
 * after the two calls. (The trainer reads no terminal observation except at the last decision
 * of a rollout, where it bootstraps from them before resetting.) */
int t8b_sim_step_and_reset(t8b_sim* sim, const int64_t* learner_candidates, const int64_t* opponent_candidates,
                           uint64_t seed, uint64_t counter);
/* Device views  full_move_gpu.hpp:96-112. Masks are uint8 [env][368] as in the
 * reference; t8b_sim_learner_mask_bits gives the packed form the library keeps
 * (12 uint32 words per environment, bit c of word c/32 = candidate c). The opponent's masks
 * are computed on the simulator's stream the first time they are asked for after a state
 * change (a scripted-opponent trainer never reads them). */
const float* t8b_sim_learner_observations(const t8b_sim* sim);
const float* t8b_sim_opponent_observations(const t8b_sim* sim);
const uint8_t* t8b_sim_learner_masks(t8b_sim* sim);
const uint8_t* t8b_sim_opponent_masks(t8b_sim* sim);
const uint32_t* t8b_sim_learner_mask_bits(const t8b_sim* sim);
const uint32_t* t8b_sim_opponent_mask_bits(const t8b_sim* sim);
const float* t8b_sim_rewards(const t8b_sim* sim);
const float* t8b_sim_sparse_rewards(const t8b_sim* sim);
const uint8_t* t8b_sim_terminated(const t8b_sim* sim);
const uint8_t* t8b_sim_truncated(const t8b_sim* sim);
const int8_t* t8b_sim_outcomes(const t8b_sim* sim);
const int32_t* t8b_sim_learner_feature_tables(const t8b_sim* sim);
const int32_t* t8b_sim_opponent_feature_tables(const t8b_sim* sim);
/* download_noise_levels  full_move_gpu.hpp:110 */
int t8b_sim_download_noise_levels(t8b_sim* sim, t8b_noise_levels_t* out);
/* frames_simulated  full_move_gpu.hpp:120 */
int t8b_sim_frames_simulated(t8b_sim* sim, uint64_t* out);
/* Evaluation bookkeeping on the device (no reference counterpart: the reference's evaluate and
 * head_to_head, src/full_move_train.cpp:921-1044, download terminated and outcomes after every
 * step). After a step, every fight that has terminated for the first time since the caller
 * zeroed `finished` gets its outcome in result[env], finished[env] = 1, and *remaining drops by
 * one. All pointers are device memory ([environments] int8 / uint8, one uint32). */
int t8b_sim_record_first_outcomes(t8b_sim* sim, int8_t* result, uint8_t* finished, uint32_t* remaining);
/* download_and_clear_tally and the three tallies cleared with it  full_move_gpu.hpp:124-131.
 * tally: [roster][5][2][3]; scenario: [9][3]; learner: [roster][3]; bot: [331][3]. */
int t8b_sim_download_and_clear_tally(t8b_sim* sim, uint32_t* tally, uint32_t* scenario_tally,
                                     uint32_t* learner_tally, uint32_t* bot_tally);
/* snapshot / restore  full_move_gpu.hpp:134-136 (host arrays [environments]). */
int t8b_sim_snapshot(t8b_sim* sim, t8b_state_t* states, int32_t* p1, int32_t* p2, uint8_t* learner_is_p1,
                     float* aggression, int32_t* pending_opponents, float* pending_aggression, uint8_t* terminated,
                     int32_t* scenarios, int32_t* pending_scenarios, int32_t* pending_learners);
int t8b_sim_restore(t8b_sim* sim, const t8b_state_t* states, const int32_t* p1, const int32_t* p2,
                    const uint8_t* learner_is_p1, const float* aggression, const int32_t* pending_opponents,
                    const float* pending_aggression, const uint8_t* terminated, const int32_t* scenarios,
                    const int32_t* pending_scenarios, const int32_t* pending_learners);
int t8b_sim_synchronize(t8b_sim* sim);

/* Engine-parity workload (no reference counterpart: the reference's tests drive fights
 * from the host one frame at a time, tests/full_combat_random_play.hpp:181-201). Every
 * fight plays `frames` frames; whenever a fighter has a decision it picks a uniformly
 * random legal candidate with a PCG32 stream (seed, stream = fight index); a finished
 * round restarts with next_round at the fight's start positions. hashes[fight*frames+f]
 * is the FNV-1a hash of the packed state after frame f. All pointers are device. */
int t8b_sim_random_play(t8b_sim* sim, int fights, const int32_t* p1, const int32_t* p2, const double* p1_x,
                        const double* p2_x, int frames, uint64_t seed, uint64_t* hashes, uint64_t* frames_done);

/* Test hook for the tcgen05 GEMM (no reference counterpart): c[m][n] = sum_k a . b^T in fp32,
 * a bf16 [m][k] (or [k][m] when a_mn_major), b bf16 [n][k] (or [k][n]); bn is the tile width
 * (64, 192 or 256) and splits the split-K factor. All pointers are device. */
int t8b_debug_gemm(const void* a, int a_mn_major, const void* b, int b_mn_major, float* c, int m, int n, int k,
                   int bn, int splits, void* stream);

/* Test hook for the bounded waits (no reference counterpart): one thread waits on a
 * shared-memory mbarrier with the GEMM's wait loop, giving up after spin_limit polls. With
 * arrive = 1 the barrier's phase completes first and *timed_out = 0; with arrive = 0 nothing
 * ever arrives, the wait runs out and *timed_out = 1 (the kernel returns; the context stays
 * usable). */
int t8b_debug_bounded_wait(int arrive, uint32_t spin_limit, int* timed_out);

/* Launch accounting (no reference counterpart). t8b_launch_count is the number of kernels the
 * library has launched since it was loaded. t8b_profile_enable(1) clears earlier results and
 * brackets every later launch with a pair of CUDA events on the launch's stream (0 stops);
 * t8b_profile_report synchronises the device, adds the elapsed times up per kernel label and
 * writes one "label launches total_ms" line per label into `text` (NUL-terminated, truncated
 * to `capacity`); it returns the size the whole report needs. */
uint64_t t8b_launch_count(void);
void t8b_profile_enable(int on);
size_t t8b_profile_report(char* text, size_t capacity);
/* Restricts the event bracketing to launches labelled `label` (copied; NULL brackets every
 * launch again), so one kernel can be timed inside a run without events around the others. */
void t8b_profile_only(const char* label);

/* ------------------------------------------------------------------ policy and PPO
 * class GpuActorCritic (include/t8_v2/ppo.hpp:112-193). Every matrix product runs bf16 x bf16
 * with fp32 accumulation on the tensor cores whatever matmul_precision asks (the reference's
 * fp32 | tf32 | bf16 choice; storage, accumulation and the optimizer stay fp32 as there). */
typedef struct t8b_actor_config { /* ActorCriticConfig (include/t8_v2/ppo.hpp:15-46) */
    int32_t observation_size, action_count, hidden_size, action_feature_size, universal_action_count;
    int32_t shared_layers, head_layers;
    uint8_t observation_normalization, orthogonal_initialization, pad[2];
    float observation_clip, observation_epsilon;
    int32_t matmul_precision; /* 0 fp32, 1 tf32, 2 bf16 (recorded; products run bf16) */
} t8b_actor_config_t;

typedef struct t8b_ppo_config { /* PpoUpdateConfig (include/t8_v2/ppo.hpp:60-73) */
    int32_t epochs, pad;
    uint64_t minibatch_size;
    float learning_rate, clip_range, value_clip_range, target_kl, value_coefficient, entropy_coefficient;
    float max_gradient_norm, adam_beta1, adam_beta2, adam_epsilon;
} t8b_ppo_config_t;

typedef struct t8b_ppo_metrics { /* PpoUpdateMetrics (include/t8_v2/ppo.hpp:75-95) */
    float policy_loss, value_loss, entropy, approximate_kl, clip_fraction, gradient_norm;
    float decision_fraction, decision_entropy, rollout_decision_entropy, pad;
    uint64_t minibatches;
    int32_t epochs_completed, early_stopped;
} t8b_ppo_metrics_t;

typedef struct t8b_policy_output { /* GpuPolicyOutputView (include/t8_v2/ppo.hpp:48-56) */
    const float* logits; /* [n][368] candidate scores, when requested */
    const int64_t* actions;
    const float* log_probabilities;
    const float* values;
    const float* entropies;
    size_t environment_count;
} t8b_policy_output_t;

typedef struct t8b_rollout_view { /* GpuRolloutView (include/t8_v2/ppo.hpp:195-212) */
    const float* observations;       /* [step][env][observation] */
    const uint8_t* action_masks;     /* [step][env][368] */
    const int64_t* actions;
    const float* old_log_probabilities;
    const float* old_values;
    const float* rewards;
    const uint8_t* terminated;
    const uint8_t* truncated;
    const float* next_values;
    const float* advantages;
    const float* returns;
    size_t environment_count, horizon, sample_count;
    const int32_t* feature_tables;
    const float* entropies;
    const uint32_t* action_mask_bits; /* [step][env][12] packed masks; used instead of action_masks when set */
} t8b_rollout_view_t;

/* Collectives for data parallelism (no reference counterpart: the reference is single-GPU).
 * The library calls allreduce_sum_* on device buffers, on `stream`, wherever the ranks must
 * agree: the minibatch gradient (then divided by world_size), the per-epoch KL, and the
 * rollout statistics (advantage moments, return moments, observation moments). */
typedef struct t8b_comm {
    void (*allreduce_sum_f32)(float* data, size_t count, void* stream, void* user);
    void (*allreduce_sum_f64)(double* data, size_t count, void* stream, void* user);
    void* user;
    int32_t world_size, rank;
} t8b_comm_t;

/* A native communicator for t8b_comm_t (no reference counterpart): NCCL (loaded at run time,
 * libnccl.so.2) over the ranks of one job, one process per GPU. Rank 0 makes the 128-byte unique
 * id with t8b_comm_unique_id and hands it to every rank by any means (a file, a socket, an MPI
 * broadcast); each rank, with its device current, calls t8b_comm_init with it, which fills `out`
 * with hooks that sum over the ranks with ncclAllReduce on the library's stream (the host never
 * waits). Set `out` on the policy and the rollout buffer (t8b_policy_set_comm,
 * t8b_rollout_set_comm). A hook that fails records the error; t8b_comm_status reports it and
 * NCCL's asynchronous errors. t8b_comm_destroy frees the communicator (after its last use on the
 * GPU) and zeroes `comm`. */
int t8b_comm_unique_id(void* id, size_t size);
int t8b_comm_init(const void* id, size_t size, int world_size, int rank, t8b_comm_t* out);
int t8b_comm_status(const t8b_comm_t* comm);
int t8b_comm_allreduce_sum_f32(const t8b_comm_t* comm, float* data, size_t count, void* stream);
int t8b_comm_destroy(t8b_comm_t* comm);

void t8b_actor_config_default(t8b_actor_config_t* out); /* full-move defaults of the trainer */
void t8b_ppo_config_default(t8b_ppo_config_t* out);

typedef struct t8b_policy t8b_policy;
/* GpuActorCritic(capacity, config, initialization_seed)  ppo.hpp:114-117 */
int t8b_policy_create(size_t capacity, const t8b_actor_config_t* config, uint64_t initialization_seed, t8b_policy** out);
int t8b_policy_destroy(t8b_policy* policy);
size_t t8b_policy_capacity(const t8b_policy* policy);        /* ppo.hpp:125 */
size_t t8b_policy_parameter_count(const t8b_policy* policy); /* ppo.hpp:126 */
int t8b_policy_action_feature_tables(const t8b_policy* policy);
/* set_action_feature_tables  ppo.hpp:137 (host features [tables][368][32]) */
int t8b_policy_set_action_feature_tables(t8b_policy* policy, const float* features, int tables, void* stream);
/* forward  ppo.hpp:146-154. Device inputs; masks uint8 [n][368] or mask_bits [n][12]. */
int t8b_policy_forward(t8b_policy* policy, const float* observations, const uint8_t* masks, const uint32_t* mask_bits,
                       size_t environment_count, uint64_t sampling_seed, uint64_t sampling_step, int deterministic,
                       void* stream, const int32_t* feature_tables, int want_logits, t8b_policy_output_t* out);
/* update_ppo  ppo.hpp:156-160 */
int t8b_policy_update_ppo(t8b_policy* policy, const t8b_rollout_view_t* rollout, const t8b_ppo_config_t* config,
                          uint64_t shuffle_seed, void* stream, t8b_ppo_metrics_t* metrics);
/* Starts computing update_ppo's host permutations in the background (no reference counterpart;
 * the same std::shuffle permutations, ready when the update starts). */
int t8b_policy_prepare_shuffle(t8b_policy* policy, size_t sample_count, int epochs, uint64_t shuffle_seed);
int t8b_policy_set_comm(t8b_policy* policy, const t8b_comm_t* comm);
/* save_checkpoint / load_checkpoint  ppo.hpp:162-166, the reference's .t8ppo format
 * (src/ppo.cu:1704-1845): files written by either implementation load in the other. The
 * contract's text fields are those of ActorCriticConfig (catalog_sha256, roster_version,
 * observation_contract, action_contract); null means the reference's defaults. Saving
 * refuses to overwrite an existing file (T8B_ESTATE) and non-finite tensors; loading checks
 * the architecture, the contract, the normaliser block, the size and the FNV-1a checksum,
 * adopts the file's normaliser setting, and with load_optimizer_state 0 zeroes Adam's moments
 * and step. */
typedef struct t8b_checkpoint_contract { /* CheckpointContract text (src/ppo.cu:1719-1726) */
    char catalog_sha256[64];
    char roster_version[24];
    char observation_contract[32];
    char action_contract[32];
} t8b_checkpoint_contract_t;
int t8b_policy_save_checkpoint(t8b_policy* policy, const char* path, const t8b_checkpoint_contract_t* contract,
                               void* stream);
int t8b_policy_load_checkpoint(t8b_policy* policy, const char* path, int load_optimizer_state,
                               const t8b_checkpoint_contract_t* contract, void* stream);
/* Parameters, gradients and Adam state in the canonical order w1, b1, ..., w_out, b_out
 * (the checkpoint payload of src/ppo.cu:1780-1845). */
int t8b_policy_get_parameters(t8b_policy* policy, float* host, size_t count);
int t8b_policy_set_parameters(t8b_policy* policy, const float* host, size_t count);
int t8b_policy_get_gradients(t8b_policy* policy, float* host, size_t count);
int t8b_policy_get_optimizer_state(t8b_policy* policy, float* first_moment, float* second_moment, uint64_t* step);
int t8b_policy_set_optimizer_state(t8b_policy* policy, const float* first_moment, const float* second_moment,
                                   uint64_t step);
/* observation_count / download_observation_statistics  ppo.hpp:174-177 */
int t8b_policy_get_observation_statistics(t8b_policy* policy, float* mean, float* variance, uint64_t* count);
int t8b_policy_set_observation_statistics(t8b_policy* policy, const float* mean, const float* variance, uint64_t count);
/* Test aid: the last forward's network outputs [n][feature_size + 1] (query, value). */
int t8b_policy_download_outputs(t8b_policy* policy, float* host, size_t n);
/* Test aid: an intermediate of the last forward/backward as fp32 rows (which: 0 layer-1 input,
 * 1 hidden activation, 2 its pre-activation gradient, 3 output-layer gradient). */
int t8b_policy_download_activation(t8b_policy* policy, int which, int layer, float* host, size_t n);
int t8b_policy_synchronize(t8b_policy* policy, void* stream);
/* config  ppo.hpp:127: the configuration in force (load_checkpoint adopts the file's
 * observation_normalization). */
int t8b_policy_get_config(const t8b_policy* policy, t8b_actor_config_t* out);
/* Test aid behind debug_backprop_relative_error (ppo.hpp:139-142): the network alone on n device
 * observations (normalised as forward does). Writes the raw outputs [n][feature_size + 1] to
 * `outputs` (device, may be NULL); with `output_gradients` (device [n][feature_size + 1] fp32)
 * runs the backward pass from them into the gradient buffer (t8b_policy_get_gradients). */
int t8b_policy_debug_network(t8b_policy* policy, const float* observations, size_t n, const float* output_gradients,
                             float* outputs, void* stream);

/* debug_ppo_objective_gradient (include/t8_v2/ppo.hpp:100-108), batched: d(objective)/d(logits,
 * value) of the clipped PPO objective for raw [n][k + 1] outputs. Device pointers. metric_sums
 * (8 doubles: policy loss, value loss, entropy, KL, clip fraction, -, decisions, decision
 * entropy) may be NULL. The call returns once the work is queued on `stream` (its metric
 * partials come from the library's stream-ordered pool on the current device). */
int t8b_ppo_output_gradient(const float* outputs, const uint8_t* masks, const int64_t* actions,
                            const float* old_log_probabilities, const float* old_values, const float* advantages,
                            const float* returns, size_t n, int action_count, const t8b_ppo_config_t* config,
                            float* gradients, double* metric_sums, void* stream);

/* No counterpart in the reference. t8b_ppo_output_gradient without allocating device memory,
 * for callers that cannot call cudaMalloc (a host whose memory manager owns the whole GPU, a
 * loop that must not pay cudaMalloc/cudaFree's implicit device synchronisation mid-step). The
 * metric partials use a static 4 MiB device array instead of a per-call buffer: at most 524,288
 * samples per call (T8B_EINVAL beyond); the first call on a device looks the array up and should
 * come before any stream capture; calls overlapping on the GPU race on the shared array.
 * The call returns once the work is queued: gradients and metric_sums are ordered on `stream`
 * only, so synchronise it (or record an event on it) before the host or another stream reads them.
 * `stream` must belong to the current device, and the device's primary context (the runtime
 * API's) must be current: the array's address is kept per device index. */
int t8b_ppo_output_gradient_static(const float* outputs, const uint8_t* masks, const int64_t* actions,
                                   const float* old_log_probabilities, const float* old_values, const float* advantages,
                                   const float* returns, size_t n, int action_count, const t8b_ppo_config_t* config,
                                   float* gradients, double* metric_sums, void* stream);

/* ------------------------------------------------------------------ rollout buffer
 * class GpuRolloutBuffer (include/t8_v2/ppo.hpp:223-291). */
typedef struct t8b_rollout t8b_rollout;
int t8b_rollout_create(size_t environments, size_t horizon, const t8b_actor_config_t* config, t8b_rollout** out);
int t8b_rollout_destroy(t8b_rollout* rollout);
/* device_view  ppo.hpp:239. When steps were recorded with packed masks since the last view, the
 * uint8 masks are expanded first; the expansion waits for those recordings on whatever stream
 * they were queued and is complete when the call returns. */
int t8b_rollout_device_view(const t8b_rollout* rollout, t8b_rollout_view_t* out);
/* The same view with packed masks only (action_masks NULL): no uint8 expansion (no reference
 * counterpart; update_ppo reads action_mask_bits). */
int t8b_rollout_packed_view(const t8b_rollout* rollout, t8b_rollout_view_t* out);
/* record_policy_device  ppo.hpp:241-250 (uint8 masks), or packed masks with mask_bits. */
int t8b_rollout_record_policy_device(t8b_rollout* rollout, size_t step, const float* observations, const uint8_t* masks,
                                     const uint32_t* mask_bits, const int64_t* actions, const float* log_probabilities,
                                     const float* values, void* stream, const int32_t* feature_tables,
                                     const float* entropies);
/* record_outcome_device  ppo.hpp:252-259 */
int t8b_rollout_record_outcome_device(t8b_rollout* rollout, size_t step, const float* rewards, const uint8_t* terminated,
                                      const uint8_t* truncated, const float* next_values, float reward_scale,
                                      void* stream);
/* compute_gae  ppo.hpp:261-265 */
int t8b_rollout_compute_gae(t8b_rollout* rollout, float gamma, float gae_lambda, int normalize_advantages, void* stream);
/* normalize_rewards  ppo.hpp:271 (returns the standard deviation used) */
int t8b_rollout_normalize_rewards(t8b_rollout* rollout, float gamma, float clip, void* stream, float* std_out);
/* mean_reward  ppo.hpp:274 */
int t8b_rollout_mean_reward(t8b_rollout* rollout, void* stream, double* out);
/* return_normalizer_state / restore  ppo.hpp:275-276; returns [environments] host floats */
int t8b_rollout_return_normalizer_state(t8b_rollout* rollout, uint64_t* count, double* mean, double* variance,
                                        float* discounted_returns);
int t8b_rollout_restore_return_normalizer_state(t8b_rollout* rollout, uint64_t count, double mean, double variance,
                                                const float* discounted_returns);
int t8b_rollout_set_comm(t8b_rollout* rollout, const t8b_comm_t* comm);
/* The trainer's rollout loop as one call (no reference counterpart: src/full_move_train.cpp:
 * 1374-1400 runs it in C++ around the three objects). For each of `horizon` decisions with
 * counter = update * horizon + step: the learner's forward on its observations, packed masks
 * and feature tables (seed + 1, sampling), the previous decision's outcome recorded with this
 * forward's values as its bootstrap, the decision recorded, the simulator stepped (counter + 1;
 * with `opponent`, a frozen policy's forward with seed + 2 on a second stream chooses the
 * opponent side's candidates), and finished rounds reset; after the last decision a
 * deterministic forward (seed + 3) gives the final bootstrap. Everything is queued on `stream`
 * (the simulator's stream is set to it). */
int t8b_collect_rollout(t8b_sim* sim, t8b_policy* policy, t8b_rollout* rollout, t8b_policy* opponent, uint64_t seed,
                        uint64_t update, size_t horizon, float reward_scale, void* stream);
int t8b_rollout_synchronize(t8b_rollout* rollout, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* T8B_H */
