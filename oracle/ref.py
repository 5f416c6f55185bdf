"""Test infrastructure (not product code): ctypes access to oracle/_ref/libt8ref.so, the
reference's own CPU engine and environment contract compiled from its sources by
oracle/Makefile. Used only by tests/, __graft_entry__.smoke() and bench.py's CPU legs."""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libt8ref.so"
# The reference checkout: $T8B_REFERENCE when set, else ../reference beside this repository.
REFERENCE = Path(os.environ.get("T8B_REFERENCE", HERE.parent.parent / "reference"))


class EnvConfig(C.Structure):
    """t8b_env_config_t of include/t8b.h, the struct the harness converts to full_core::EnvConfig."""
    _fields_ = [("max_round_frames", C.c_int32), ("hold_frames", C.c_int32), ("max_frames_per_decision", C.c_int32)] + \
               [(n, C.c_float) for n in ("damage_reward", "win_reward", "draw_penalty", "throw_break_penalty",
                                          "time_penalty_per_second", "damage_dealt_weight", "damage_taken_weight",
                                          "distance_penalty_per_second")] + \
               [("perception_delay", C.c_int32), ("memory", C.c_uint8), ("live_noise", C.c_uint8),
                ("screen_view", C.c_uint8), ("pad", C.c_uint8), ("noise_position_max", C.c_float),
                ("noise_flip_max", C.c_float), ("latency_min", C.c_int32), ("latency_max", C.c_int32),
                ("pad2", C.c_int32), ("start_center_range", C.c_double), ("start_distance_min", C.c_double),
                ("start_distance_max", C.c_double)]


def env_config(**overrides) -> EnvConfig:
    """full_core::EnvConfig with the reference's own defaults, then the given fields."""
    config = EnvConfig()
    lib().t8ref_env_config_default(C.byref(config))
    for key, value in overrides.items():
        setattr(config, key, value)
    return config


def config4_env(**overrides) -> EnvConfig:
    """The trainer's measured self-play environment (training.ini through src/train_launcher.cpp:
    106-160): screen-only observation with live noise (sigma 0.28 m, 10 % flips, latency 2-6),
    perception delay 12, 8-frame holds and the anti-stalling reward terms."""
    base = dict(screen_view=1, live_noise=1, noise_position_max=0.28, noise_flip_max=0.10, latency_min=2,
                latency_max=6, perception_delay=12, hold_frames=8, draw_penalty=0.5, throw_break_penalty=0.03,
                time_penalty_per_second=0.01, max_round_frames=3600)
    base.update(overrides)
    return env_config(**base)


def build() -> Path:
    """Builds the reference library when the reference sources are present (not on GPU boxes)."""
    if (REFERENCE / "src").exists():
        subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REFERENCE}"], check=True)
    if not LIB.exists():
        raise RuntimeError(f"{LIB} is missing and the reference sources are not here to build it")
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        h = C.CDLL(str(LIB))
        vp = C.c_void_p
        h.t8ref_last_error.restype = C.c_char_p
        h.t8ref_export_roster.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p]
        h.t8ref_roster_parse.restype = vp
        h.t8ref_roster_parse.argtypes = [C.c_char_p, C.c_size_t]
        h.t8ref_roster_free.argtypes = [vp]
        h.t8ref_roster_count.argtypes = [vp]
        h.t8ref_random_play.argtypes = [vp, C.c_int, vp, vp, vp, vp, C.c_int, C.c_uint64, vp, vp, vp, vp, C.c_int]
        h.t8ref_engine_step.argtypes = [vp, C.c_int, vp, vp, vp, vp, vp]
        h.t8ref_reset_state.argtypes = [vp, C.c_int, C.c_int, C.c_double, C.c_double, vp]
        h.t8ref_state_hash.restype = C.c_uint64
        h.t8ref_state_hash.argtypes = [vp]
        h.t8ref_env_create.restype = vp
        h.t8ref_env_create.argtypes = [vp, C.c_size_t, vp, C.c_int]
        h.t8ref_env_free.argtypes = [vp]
        h.t8ref_env_observation_size.argtypes = [vp]
        h.t8ref_env_setup.argtypes = [vp] * 8
        h.t8ref_env_reset_all.argtypes = [vp, C.c_uint64, C.c_uint64]
        h.t8ref_env_reset_done.argtypes = [vp, C.c_uint64, C.c_uint64]
        h.t8ref_env_step.argtypes = [vp, vp, vp, C.c_uint64, C.c_uint64, C.c_int]
        h.t8ref_env_read.argtypes = [vp] * 14
        h.t8ref_env_upload_states.argtypes = [vp, vp]
        h.t8ref_env_config_default.restype = None
        h.t8ref_env_config_default.argtypes = [vp]
        h.t8ref_roster_features.argtypes = [vp, vp, C.c_int]
        _lib = h
    return _lib


def _check(status):
    if status != 0:
        raise RuntimeError(lib().t8ref_last_error().decode())


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def export_roster(generated_dir: str, out_path: str, slugs: str | None = None):
    _check(lib().t8ref_export_roster(generated_dir.encode(), slugs.encode() if slugs else None, out_path.encode()))


class RefRoster:
    def __init__(self, raw: bytes):
        self._raw = raw
        self.handle = lib().t8ref_roster_parse(raw, len(raw))
        if not self.handle:
            raise RuntimeError(lib().t8ref_last_error().decode())

    def __del__(self):
        if getattr(self, "handle", None):
            lib().t8ref_roster_free(self.handle)
            self.handle = None

    def feature_tables(self, stride: int = 368) -> np.ndarray:
        """[characters, stride, 32] float32 candidate features, zero past each character's candidates."""
        count = lib().t8ref_roster_count(self.handle)
        out = np.zeros((count, stride, 32), np.float32)
        _check(lib().t8ref_roster_features(self.handle, _p(out), stride))
        return out

    def random_play(self, p1, p2, x1, x2, frames: int, seed: int, threads: int = 8, states=False, inputs=False):
        p1 = np.ascontiguousarray(p1, np.int32)
        p2 = np.ascontiguousarray(p2, np.int32)
        x1 = np.ascontiguousarray(x1, np.float64)
        x2 = np.ascontiguousarray(x2, np.float64)
        n = p1.shape[0]
        hashes = np.zeros((n, frames), np.uint64)
        st = np.zeros((n, frames, 240), np.uint8) if states else None
        ins = np.zeros((n, frames, 2, 2), np.int32) if inputs else None
        _check(lib().t8ref_random_play(self.handle, n, _p(p1), _p(p2), _p(x1), _p(x2), frames, seed, _p(hashes),
                                       _p(st), _p(ins), None, threads))
        return hashes, st, ins

    def reset_state(self, p1, p2, x1, x2) -> np.ndarray:
        out = np.zeros(240, np.uint8)
        _check(lib().t8ref_reset_state(self.handle, p1, p2, x1, x2, _p(out)))
        return out

    def engine_step(self, p1, p2, states: np.ndarray, inputs: np.ndarray):
        """states: uint8 [n, 240] (updated in place); inputs int32 [n, 2, 2]. Returns events bytes [n, 208]."""
        n = states.shape[0]
        events = np.zeros((n, 208), np.uint8)
        p1 = np.ascontiguousarray(p1, np.int32)
        p2 = np.ascontiguousarray(p2, np.int32)
        inputs = np.ascontiguousarray(inputs, np.int32)
        _check(lib().t8ref_engine_step(self.handle, n, _p(p1), _p(p2), _p(states), _p(inputs), _p(events)))
        return events


class RefEnv:
    """The GpuFullMoveSimulator contract on the host (reference functions only)."""

    def __init__(self, roster: RefRoster, n: int, config, threads: int = 8):
        self.roster = roster
        self.n = n
        self._config = config
        self.handle = lib().t8ref_env_create(roster.handle, n, C.byref(config), threads)
        if not self.handle:
            raise RuntimeError(lib().t8ref_last_error().decode())
        self.width = lib().t8ref_env_observation_size(self.handle)

    def __del__(self):
        if getattr(self, "handle", None):
            lib().t8ref_env_free(self.handle)
            self.handle = None

    def setup(self, p1=None, p2=None, learner_is_p1=None, opponents=None, aggression=None, scenarios=None,
              learners=None):
        args = [None if v is None else np.ascontiguousarray(v, t) for v, t in
                ((p1, np.int32), (p2, np.int32), (learner_is_p1, np.uint8), (opponents, np.int32),
                 (aggression, np.float32), (scenarios, np.int32), (learners, np.int32))]
        _check(lib().t8ref_env_setup(self.handle, *[_p(a) for a in args]))

    def reset_all(self, seed, counter):
        _check(lib().t8ref_env_reset_all(self.handle, seed, counter))

    def reset_done(self, seed, counter):
        _check(lib().t8ref_env_reset_done(self.handle, seed, counter))

    def step(self, learner, opponent=None, seed=0, counter=0, observe=True):
        a = np.ascontiguousarray(learner, np.int64)
        b = None if opponent is None else np.ascontiguousarray(opponent, np.int64)
        _check(lib().t8ref_env_step(self.handle, _p(a), _p(b), seed, counter, 1 if observe else 0))

    def read(self):
        n, w = self.n, self.width
        out = {
            "learner_obs": np.zeros((n, w), np.float32), "opponent_obs": np.zeros((n, w), np.float32),
            "learner_masks": np.zeros((n, 368), np.uint8), "opponent_masks": np.zeros((n, 368), np.uint8),
            "rewards": np.zeros(n, np.float32), "sparse": np.zeros(n, np.float32),
            "terminated": np.zeros(n, np.uint8), "outcomes": np.zeros(n, np.int8),
            "states": np.zeros((n, 240), np.uint8), "noise": np.zeros((n, 16), np.uint8),
            "p1": np.zeros(n, np.int32), "p2": np.zeros(n, np.int32),
        }
        frames = C.c_uint64()
        _check(lib().t8ref_env_read(self.handle, *[_p(out[k]) for k in
                                                   ("learner_obs", "opponent_obs", "learner_masks", "opponent_masks",
                                                    "rewards", "sparse", "terminated", "outcomes", "states", "noise",
                                                    "p1", "p2")], C.byref(frames)))
        out["frames"] = frames.value
        return out
