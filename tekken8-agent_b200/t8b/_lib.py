"""ctypes binding of include/t8b.h: struct layouts, prototypes, status handling.

The shared library is loaded from ../lib/libt8b.so (built in-tree by build.py), or from the
path in the T8B_LIBRARY environment variable. There is no fallback: importing this module
without the library raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("T8B_LIBRARY") or Path(__file__).resolve().parent.parent / "lib" / "libt8b.so")

T8B_OK, T8B_EINVAL, T8B_ERANGE, T8B_ECUDA, T8B_ENONFINITE, T8B_ESTATE = range(6)
UNIVERSAL_COUNT, MAX_CANDIDATES, FEATURE_SIZE, ROSTER_SLOTS = 22, 368, 32, 42
SCRIPTED_PROFILES, SCENARIOS, AGGRESSION_BUCKETS = 331, 9, 5
MASK_WORDS = 12


class Window(C.Structure):
    _fields_ = [("count", C.c_int32), ("first", C.c_int32 * 8), ("last", C.c_int32 * 8)]


class Hit(C.Structure):
    _fields_ = [("level", C.c_uint8), ("throw_break", C.c_uint8), ("flags", C.c_uint16),
                ("first_active_frame", C.c_int32), ("active_frames", C.c_int32)] + \
               [(n, C.c_double) for n in ("damage", "reach", "tracking_left", "tracking_right", "chip_damage",
                                          "heat_chip_damage")]


_MOVE_INTS = ("hit_offset", "hit_count", "total_frames", "recovery", "block_advantage", "hit_advantage",
              "counter_hit_advantage", "launch_air_frames", "back_turned_hit_advantage",
              "heat_dash_block_advantage", "heat_dash_hit_advantage", "heat_cost_frames", "required_stance",
              "result_stance", "result_stance_on_hit", "result_stance_on_block")
_MOVE_BYTES = ("hit_effect", "counter_hit_effect", "back_turned_hit_effect", "heat_dash_hit_effect",
               "required_posture", "attack_throw", "parry_levels", "heat_parry_levels")
_MOVE_DOUBLES = ("travel", "pushback_hit", "pushback_block", "reversal_damage", "attack_throw_damage",
                 "recoverable_damage", "rage_art_max_damage", "self_damage", "self_recoverable",
                 "restore_health_hit", "restore_recoverable_hit", "restore_recoverable_block",
                 "resource_gain_start", "resource_gain_hit", "resource_gain_airborne_hit", "resource_gain_block",
                 "resource_gain_heat_activation", "install_damage_bonus", "install_chip_damage", "install_reach")


class Move(C.Structure):
    _fields_ = [("flags", C.c_uint64)] + [(n, C.c_int32) for n in _MOVE_INTS] + \
               [("parry_outcomes", C.c_int32 * 4), ("heat_parry_outcome", C.c_int32)] + \
               [(n, C.c_uint8) for n in _MOVE_BYTES] + [(n, C.c_double) for n in _MOVE_DOUBLES] + \
               [("windows", Window * 9)]


class Stance(C.Structure):
    _fields_ = [("can_guard", C.c_uint8), ("has_max_frames", C.c_uint8), ("auto_parry", C.c_uint8),
                ("pad", C.c_uint8), ("max_frames", C.c_int32), ("parry_outcomes", C.c_int32 * 4),
                ("pulse_interval_frames", C.c_int32), ("pulse_recoverable", C.c_double),
                ("pulse_resource", C.c_double)]


class Rules(C.Structure):
    _fields_ = [("resource_max", C.c_double), ("install_threshold", C.c_double),
                ("has_install_threshold", C.c_uint8), ("resource_persists", C.c_uint8),
                ("install_consumes", C.c_uint8), ("pad", C.c_uint8 * 5)]


class EngineConfig(C.Structure):
    _fields_ = [("half_width", C.c_double), ("body_radius", C.c_double), ("walk_speed", C.c_double),
                ("dash_distance", C.c_double), ("dash_frames", C.c_int32), ("backdash_frames", C.c_int32),
                ("backdash_distance", C.c_double), ("sidestep_distance", C.c_double),
                ("sidestep_frames", C.c_int32), ("launch_air_frames", C.c_int32),
                ("axis_realign_per_frame", C.c_double), ("juggle_window_frames", C.c_int32),
                ("juggle_window_decay", C.c_int32), ("tornado_extra_frames", C.c_int32),
                ("knockdown_frames", C.c_int32), ("wakeup_stand_frames", C.c_int32),
                ("wakeup_roll_frames", C.c_int32), ("wakeup_roll_distance", C.c_double),
                ("tech_window_frames", C.c_int32), ("tech_roll_frames", C.c_int32),
                ("wall_splat_frames", C.c_int32), ("crumple_frames", C.c_int32),
                ("stage_break_air_frames", C.c_int32), ("pad0", C.c_int32),
                ("wall_break_extension", C.c_double), ("combo_scale_step", C.c_double),
                ("combo_scale_floor", C.c_double), ("counter_hit_damage_scale", C.c_double),
                ("throw_break_window", C.c_int32), ("throw_break_recovery", C.c_int32),
                ("parry_outcome_frames", C.c_int32), ("pad1", C.c_int32),
                ("side_exposure_ratio", C.c_double), ("back_to_wall_distance", C.c_double),
                ("ki_charge_frames", C.c_int32), ("pad2", C.c_int32), ("ki_charge_damage_scale", C.c_double),
                ("parry_stun_frames", C.c_int32), ("reversal_recovery", C.c_int32),
                ("heat_duration_frames", C.c_int32), ("heat_dash_frames", C.c_int32),
                ("heat_dash_distance", C.c_double), ("rage_health_fraction", C.c_double),
                ("rage_damage_scale", C.c_double), ("wall_combo_scale", C.c_double),
                ("recoverable_regain_hit", C.c_double), ("recoverable_regain_block", C.c_double),
                ("max_health", C.c_double)]


class Character(C.Structure):
    _fields_ = [("moves", C.POINTER(Move)), ("hits", C.POINTER(Hit)), ("stances", C.POINTER(Stance)),
                ("candidate_moves", C.POINTER(C.c_int32)), ("candidate_features", C.POINTER(C.c_float)),
                ("move_count", C.c_int32), ("hit_count", C.c_int32), ("stance_count", C.c_int32),
                ("candidate_count", C.c_int32), ("roster_id", C.c_int32), ("pad", C.c_int32),
                ("rules", Rules)]


class Fighter(C.Structure):
    _fields_ = [(n, C.c_double) for n in ("health", "recoverable_health", "x", "axis", "resource")] + \
               [("posture", C.c_uint8), ("universal", C.c_uint8), ("heat_dash_from", C.c_int8), ("pad", C.c_uint8),
                ("flags", C.c_uint32)] + \
               [(n, C.c_int32) for n in ("stance", "heat_frames", "throw_break_frames", "pending_throw_hit",
                                          "pending_throw_elapsed", "move", "action_frame")] + \
               [("hits_landed", C.c_uint32)] + \
               [(n, C.c_int32) for n in ("stance_frames", "ki_charge_frames", "stun", "posture_frames",
                                          "grounded_elapsed", "combo_hits")]


class State(C.Structure):
    _fields_ = [("fighters", Fighter * 2), ("left_wall", C.c_double), ("right_wall", C.c_double),
                ("stage_flags", C.c_uint32), ("stage_level", C.c_int32), ("frame", C.c_int32),
                ("winner", C.c_int32)]


class Input(C.Structure):
    _fields_ = [("move", C.c_int32), ("universal", C.c_int32)]


class ContactEvent(C.Structure):
    _fields_ = [("attacker", C.c_int32), ("hit_index", C.c_int32), ("contact", C.c_int32), ("pad", C.c_int32),
                ("damage", C.c_double)]


class Events(C.Structure):
    _fields_ = [("contact_count", C.c_int32), ("transition_count", C.c_int32), ("contacts", ContactEvent * 8),
                ("transitions", C.c_uint8 * 4), ("heat_activated", C.c_uint8 * 2), ("rage_activated", C.c_uint8 * 2)]


class EnvConfig(C.Structure):
    _fields_ = [("max_round_frames", C.c_int32), ("hold_frames", C.c_int32), ("max_frames_per_decision", C.c_int32)] + \
               [(n, C.c_float) for n in ("damage_reward", "win_reward", "draw_penalty", "throw_break_penalty",
                                          "time_penalty_per_second", "damage_dealt_weight", "damage_taken_weight",
                                          "distance_penalty_per_second")] + \
               [("perception_delay", C.c_int32), ("memory", C.c_uint8), ("live_noise", C.c_uint8),
                ("screen_view", C.c_uint8), ("pad", C.c_uint8), ("noise_position_max", C.c_float),
                ("noise_flip_max", C.c_float), ("latency_min", C.c_int32), ("latency_max", C.c_int32),
                ("pad2", C.c_int32), ("start_center_range", C.c_double), ("start_distance_min", C.c_double),
                ("start_distance_max", C.c_double)]


class NoiseLevels(C.Structure):
    _fields_ = [("position_sigma", C.c_float), ("flip_rate", C.c_float), ("latency", C.c_int32), ("key", C.c_uint32)]


SIZES = {"t8b_move_t": 880, "t8b_hit_t": 64, "t8b_stance_t": 48, "t8b_rules_t": 24, "t8b_engine_config_t": 280,
         "t8b_state_t": 240, "t8b_events_t": 208, "t8b_env_config_t": 96, "t8b_character_t": 88,
         "t8b_noise_levels_t": 16, "t8b_input_t": 8}
for _name, _cls in (("t8b_move_t", Move), ("t8b_hit_t", Hit), ("t8b_stance_t", Stance), ("t8b_rules_t", Rules),
                    ("t8b_engine_config_t", EngineConfig), ("t8b_state_t", State), ("t8b_events_t", Events),
                    ("t8b_env_config_t", EnvConfig), ("t8b_character_t", Character),
                    ("t8b_noise_levels_t", NoiseLevels), ("t8b_input_t", Input)):
    assert C.sizeof(_cls) == SIZES[_name], (_name, C.sizeof(_cls))

vp = C.c_void_p
u64 = C.c_uint64
i32p = C.POINTER(C.c_int32)

# name -> (restype, argtypes); restype int = status.
PROTOTYPES = {
    "t8b_last_error": (C.c_char_p, []),
    "t8b_device_count": (C.c_int, [i32p]),
    "t8b_engine_config_default": (None, [C.POINTER(EngineConfig)]),
    "t8b_env_config_default": (None, [C.POINTER(EnvConfig)]),
    "t8b_sim_create": (C.c_int, [C.POINTER(Character), C.c_int, C.POINTER(EngineConfig), C.c_size_t,
                                 C.POINTER(EnvConfig), C.POINTER(vp)]),
    "t8b_sim_destroy": (C.c_int, [vp]),
    "t8b_sim_set_stream": (C.c_int, [vp, vp]),
    "t8b_sim_environment_count": (C.c_size_t, [vp]),
    "t8b_sim_observation_size": (C.c_int, [vp]),
    "t8b_sim_set_matchups": (C.c_int, [vp, vp, vp]),
    "t8b_sim_reset_engine": (C.c_int, [vp, vp, vp]),
    "t8b_sim_step_engine": (C.c_int, [vp, vp, vp, vp, vp]),
    "t8b_sim_download_states": (C.c_int, [vp, vp]),
    "t8b_sim_download_events": (C.c_int, [vp, vp]),
    "t8b_sim_upload_states": (C.c_int, [vp, vp]),
    "t8b_sim_download_legal_mask": (C.c_int, [vp, C.c_int, vp]),
    "t8b_sim_set_learner_sides": (C.c_int, [vp, vp]),
    "t8b_sim_set_pending_opponents": (C.c_int, [vp, vp, vp, vp]),
    "t8b_sim_set_pending_learners": (C.c_int, [vp, vp]),
    "t8b_sim_reset_all": (C.c_int, [vp, u64, u64]),
    "t8b_sim_reset_done": (C.c_int, [vp, u64, u64]),
    "t8b_sim_step": (C.c_int, [vp, vp, vp, u64, u64]),
    "t8b_sim_step_and_reset": (C.c_int, [vp, vp, vp, u64, u64]),
    "t8b_sim_learner_observations": (vp, [vp]),
    "t8b_sim_opponent_observations": (vp, [vp]),
    "t8b_sim_learner_masks": (vp, [vp]),
    "t8b_sim_opponent_masks": (vp, [vp]),
    "t8b_sim_learner_mask_bits": (vp, [vp]),
    "t8b_sim_opponent_mask_bits": (vp, [vp]),
    "t8b_sim_rewards": (vp, [vp]),
    "t8b_sim_sparse_rewards": (vp, [vp]),
    "t8b_sim_terminated": (vp, [vp]),
    "t8b_sim_truncated": (vp, [vp]),
    "t8b_sim_outcomes": (vp, [vp]),
    "t8b_sim_learner_feature_tables": (vp, [vp]),
    "t8b_sim_opponent_feature_tables": (vp, [vp]),
    "t8b_sim_download_noise_levels": (C.c_int, [vp, vp]),
    "t8b_sim_frames_simulated": (C.c_int, [vp, C.POINTER(u64)]),
    "t8b_sim_record_first_outcomes": (C.c_int, [vp, vp, vp, vp]),
    "t8b_sim_download_and_clear_tally": (C.c_int, [vp, vp, vp, vp, vp]),
    "t8b_sim_snapshot": (C.c_int, [vp] * 12),
    "t8b_sim_restore": (C.c_int, [vp] * 12),
    "t8b_sim_synchronize": (C.c_int, [vp]),
    "t8b_sim_random_play": (C.c_int, [vp, C.c_int, vp, vp, vp, vp, C.c_int, u64, vp, C.POINTER(u64)]),
}


class T8bError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"status {status}: {message}")
        self.status = status


_lib = None


def lib():
    """The loaded library with prototypes applied (loads on first use)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run tekken8-agent_b200/build.py (no CPU fallback exists)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def call(name: str, *args):
    """Calls a status-returning entry point; raises T8bError on failure."""
    status = getattr(lib(), name)(*args)
    if status != T8B_OK:
        raise T8bError(status, lib().t8b_last_error().decode())


# ------------------------------------------------------------------ policy / rollout
class ActorConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("observation_size", "action_count", "hidden_size", "action_feature_size",
                                          "universal_action_count", "shared_layers", "head_layers")] + \
               [("observation_normalization", C.c_uint8), ("orthogonal_initialization", C.c_uint8),
                ("pad", C.c_uint8 * 2), ("observation_clip", C.c_float), ("observation_epsilon", C.c_float),
                ("matmul_precision", C.c_int32)]


class PpoConfig(C.Structure):
    _fields_ = [("epochs", C.c_int32), ("pad", C.c_int32), ("minibatch_size", C.c_uint64)] + \
               [(n, C.c_float) for n in ("learning_rate", "clip_range", "value_clip_range", "target_kl",
                                          "value_coefficient", "entropy_coefficient", "max_gradient_norm",
                                          "adam_beta1", "adam_beta2", "adam_epsilon")]


class PpoMetrics(C.Structure):
    _fields_ = [(n, C.c_float) for n in ("policy_loss", "value_loss", "entropy", "approximate_kl", "clip_fraction",
                                          "gradient_norm", "decision_fraction", "decision_entropy",
                                          "rollout_decision_entropy", "pad")] + \
               [("minibatches", C.c_uint64), ("epochs_completed", C.c_int32), ("early_stopped", C.c_int32)]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_ if name != "pad"}


class PolicyOutput(C.Structure):
    _fields_ = [("logits", C.c_void_p), ("actions", C.c_void_p), ("log_probabilities", C.c_void_p),
                ("values", C.c_void_p), ("entropies", C.c_void_p), ("environment_count", C.c_size_t)]


class RolloutView(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("observations", "action_masks", "actions", "old_log_probabilities",
                                           "old_values", "rewards", "terminated", "truncated", "next_values",
                                           "advantages", "returns")] + \
               [("environment_count", C.c_size_t), ("horizon", C.c_size_t), ("sample_count", C.c_size_t),
                ("feature_tables", C.c_void_p), ("entropies", C.c_void_p), ("action_mask_bits", C.c_void_p)]


ALLREDUCE_F32 = C.CFUNCTYPE(None, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p)
ALLREDUCE_F64 = C.CFUNCTYPE(None, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p)


class Comm(C.Structure):
    _fields_ = [("allreduce_sum_f32", ALLREDUCE_F32), ("allreduce_sum_f64", ALLREDUCE_F64), ("user", C.c_void_p),
                ("world_size", C.c_int32), ("rank", C.c_int32)]


class CheckpointContract(C.Structure):
    _fields_ = [("catalog_sha256", C.c_char * 64), ("roster_version", C.c_char * 24),
                ("observation_contract", C.c_char * 32), ("action_contract", C.c_char * 32)]


SIZES.update({"t8b_checkpoint_contract_t": 152})
SIZES.update({"t8b_actor_config_t": 44, "t8b_ppo_config_t": 56, "t8b_ppo_metrics_t": 56, "t8b_policy_output_t": 48,
              "t8b_rollout_view_t": 136, "t8b_comm_t": 32})
for _name, _cls in (("t8b_actor_config_t", ActorConfig), ("t8b_ppo_config_t", PpoConfig),
                    ("t8b_ppo_metrics_t", PpoMetrics), ("t8b_policy_output_t", PolicyOutput),
                    ("t8b_rollout_view_t", RolloutView), ("t8b_comm_t", Comm),
                    ("t8b_checkpoint_contract_t", CheckpointContract)):
    assert C.sizeof(_cls) == SIZES[_name], (_name, C.sizeof(_cls))

fp = C.POINTER(C.c_float)
PROTOTYPES.update({
    "t8b_debug_gemm": (C.c_int, [vp, C.c_int, vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp]),
    "t8b_debug_bounded_wait": (C.c_int, [C.c_int, C.c_uint32, C.POINTER(C.c_int)]),
    "t8b_launch_count": (u64, []),
    "t8b_profile_enable": (None, [C.c_int]),
    "t8b_profile_report": (C.c_size_t, [C.c_char_p, C.c_size_t]),
    "t8b_profile_only": (None, [C.c_char_p]),
    "t8b_actor_config_default": (None, [C.POINTER(ActorConfig)]),
    "t8b_ppo_config_default": (None, [C.POINTER(PpoConfig)]),
    "t8b_policy_create": (C.c_int, [C.c_size_t, C.POINTER(ActorConfig), u64, C.POINTER(vp)]),
    "t8b_policy_destroy": (C.c_int, [vp]),
    "t8b_policy_capacity": (C.c_size_t, [vp]),
    "t8b_policy_parameter_count": (C.c_size_t, [vp]),
    "t8b_policy_action_feature_tables": (C.c_int, [vp]),
    "t8b_policy_set_action_feature_tables": (C.c_int, [vp, vp, C.c_int, vp]),
    "t8b_policy_forward": (C.c_int, [vp, vp, vp, vp, C.c_size_t, u64, u64, C.c_int, vp, vp, C.c_int,
                                     C.POINTER(PolicyOutput)]),
    "t8b_policy_update_ppo": (C.c_int, [vp, C.POINTER(RolloutView), C.POINTER(PpoConfig), u64, vp,
                                        C.POINTER(PpoMetrics)]),
    "t8b_policy_prepare_shuffle": (C.c_int, [vp, C.c_size_t, C.c_int, u64]),
    "t8b_policy_set_comm": (C.c_int, [vp, C.POINTER(Comm)]),
    "t8b_policy_save_checkpoint": (C.c_int, [vp, C.c_char_p, C.POINTER(CheckpointContract), vp]),
    "t8b_policy_load_checkpoint": (C.c_int, [vp, C.c_char_p, C.c_int, C.POINTER(CheckpointContract), vp]),
    "t8b_policy_get_parameters": (C.c_int, [vp, vp, C.c_size_t]),
    "t8b_policy_set_parameters": (C.c_int, [vp, vp, C.c_size_t]),
    "t8b_policy_get_gradients": (C.c_int, [vp, vp, C.c_size_t]),
    "t8b_policy_get_optimizer_state": (C.c_int, [vp, vp, vp, C.POINTER(u64)]),
    "t8b_policy_set_optimizer_state": (C.c_int, [vp, vp, vp, u64]),
    "t8b_policy_get_observation_statistics": (C.c_int, [vp, vp, vp, C.POINTER(u64)]),
    "t8b_policy_set_observation_statistics": (C.c_int, [vp, vp, vp, u64]),
    "t8b_policy_download_outputs": (C.c_int, [vp, vp, C.c_size_t]),
    "t8b_policy_synchronize": (C.c_int, [vp, vp]),
    "t8b_policy_download_activation": (C.c_int, [vp, C.c_int, C.c_int, vp, C.c_size_t]),
    "t8b_ppo_output_gradient": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, C.c_size_t, C.c_int, C.POINTER(PpoConfig),
                                          vp, vp, vp]),
    "t8b_ppo_output_gradient_static": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, C.c_size_t, C.c_int,
                                                 C.POINTER(PpoConfig), vp, vp, vp]),
    "t8b_rollout_create": (C.c_int, [C.c_size_t, C.c_size_t, C.POINTER(ActorConfig), C.POINTER(vp)]),
    "t8b_rollout_destroy": (C.c_int, [vp]),
    "t8b_rollout_device_view": (C.c_int, [vp, C.POINTER(RolloutView)]),
    "t8b_rollout_packed_view": (C.c_int, [vp, C.POINTER(RolloutView)]),
    "t8b_rollout_record_policy_device": (C.c_int, [vp, C.c_size_t, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "t8b_rollout_record_outcome_device": (C.c_int, [vp, C.c_size_t, vp, vp, vp, vp, C.c_float, vp]),
    "t8b_rollout_compute_gae": (C.c_int, [vp, C.c_float, C.c_float, C.c_int, vp]),
    "t8b_rollout_normalize_rewards": (C.c_int, [vp, C.c_float, C.c_float, vp, fp]),
    "t8b_rollout_mean_reward": (C.c_int, [vp, vp, C.POINTER(C.c_double)]),
    "t8b_rollout_return_normalizer_state": (C.c_int, [vp, C.POINTER(u64), C.POINTER(C.c_double),
                                                      C.POINTER(C.c_double), vp]),
    "t8b_rollout_restore_return_normalizer_state": (C.c_int, [vp, u64, C.c_double, C.c_double, vp]),
    "t8b_rollout_set_comm": (C.c_int, [vp, C.POINTER(Comm)]),
    "t8b_comm_unique_id": (C.c_int, [vp, C.c_size_t]),
    "t8b_comm_init": (C.c_int, [vp, C.c_size_t, C.c_int, C.c_int, C.POINTER(Comm)]),
    "t8b_comm_status": (C.c_int, [C.POINTER(Comm)]),
    "t8b_comm_allreduce_sum_f32": (C.c_int, [C.POINTER(Comm), vp, C.c_size_t, vp]),
    "t8b_comm_destroy": (C.c_int, [C.POINTER(Comm)]),
    "t8b_policy_get_config": (C.c_int, [vp, C.POINTER(ActorConfig)]),
    "t8b_policy_debug_network": (C.c_int, [vp, vp, C.c_size_t, vp, vp, vp]),
    "t8b_collect_rollout": (C.c_int, [vp, vp, vp, vp, u64, u64, C.c_size_t, C.c_float, vp]),
    "t8b_rollout_synchronize": (C.c_int, [vp, vp]),
})
