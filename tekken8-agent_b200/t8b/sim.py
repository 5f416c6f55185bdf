"""GpuFullMoveSimulator: the reference class (include/t8_v2/full_move_gpu.hpp:42-141) over
the t8b_sim_* entry points. Host arrays are numpy; device views are torch tensors aliasing
the simulator's buffers."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import EnvConfig, EngineConfig, MAX_CANDIDATES, MASK_WORDS, State, Events, NoiseLevels, Input, call
from .device import view, ptr


def env_config(**overrides) -> EnvConfig:
    """full_core::EnvConfig defaults (include/t8_v2/full_move_contract.hpp:737-773) plus overrides."""
    config = EnvConfig()
    _lib.lib().t8b_env_config_default(C.byref(config))
    for key, value in overrides.items():
        if not hasattr(config, key):
            raise AttributeError(key)
        setattr(config, key, value)
    return config


def _arr(values, dtype):
    out = np.ascontiguousarray(values, dtype=dtype)
    return out, out.ctypes.data_as(C.c_void_p)


class GpuFullMoveSimulator:
    candidate_stride = MAX_CANDIDATES

    def __init__(self, roster, environments: int, config: EnvConfig | None = None, characters=None):
        self._roster = roster
        self._chars = roster.c_array(characters)
        self.roster_count = len(self._chars)
        self.config = config if config is not None else env_config()
        self.n = int(environments)
        handle = C.c_void_p()
        engine = EngineConfig.from_buffer_copy(bytes(roster.config))
        call("t8b_sim_create", self._chars, self.roster_count, C.byref(engine), self.n, C.byref(self.config),
             C.byref(handle))
        self._handle = handle
        self.device = torch.cuda.current_device()

    def close(self):
        if getattr(self, "_handle", None):
            call("t8b_sim_destroy", self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._handle

    def environment_count(self) -> int:
        return self.n

    def observation_size(self) -> int:
        return _lib.lib().t8b_sim_observation_size(self._handle)

    # ---- setup
    def set_matchups(self, p1, p2):
        a, pa = _arr(p1, np.int32)
        b, pb = _arr(p2, np.int32)
        self._check_len(a, b)
        call("t8b_sim_set_matchups", self._handle, pa, pb)

    def set_learner_sides(self, learner_is_p1):
        a, pa = _arr(learner_is_p1, np.uint8)
        self._check_len(a)
        call("t8b_sim_set_learner_sides", self._handle, pa)

    def set_pending_opponents(self, characters, aggression=None, scenarios=None):
        a, pa = _arr(characters, np.int32)
        self._check_len(a)
        keep = [a]
        pb = pc = None
        if aggression is not None:
            b, pb = _arr(aggression, np.float32)
            self._check_len(b)
            keep.append(b)
        if scenarios is not None:
            c, pc = _arr(scenarios, np.int32)
            self._check_len(c)
            keep.append(c)
        call("t8b_sim_set_pending_opponents", self._handle, pa, pb, pc)

    def set_pending_learners(self, characters):
        a, pa = _arr(characters, np.int32)
        self._check_len(a)
        call("t8b_sim_set_pending_learners", self._handle, pa)

    def _check_len(self, *arrays):
        for a in arrays:
            if a.shape[0] != self.n:
                raise ValueError("one value per environment is required")

    # ---- engine level
    def reset_engine(self, p1_x, p2_x):
        a, pa = _arr(p1_x, np.float64)
        b, pb = _arr(p2_x, np.float64)
        call("t8b_sim_reset_engine", self._handle, pa, pb)

    def step_engine(self, inputs, new_round=None, p1_x=None, p2_x=None):
        """inputs: int32 [env, 2, 2] (move, universal) per fighter."""
        i, pi = _arr(inputs, np.int32)
        if new_round is None:
            call("t8b_sim_step_engine", self._handle, pi, None, None, None)
        else:
            r, pr = _arr(new_round, np.uint8)
            a, pa = _arr(p1_x, np.float64)
            b, pb = _arr(p2_x, np.float64)
            call("t8b_sim_step_engine", self._handle, pi, pr, pa, pb)

    def download_states(self):
        out = (State * self.n)()
        call("t8b_sim_download_states", self._handle, out)
        return out

    def download_state_bytes(self) -> np.ndarray:
        return np.frombuffer(bytes(self.download_states()), np.uint8).reshape(self.n, 240)

    def upload_states(self, states):
        call("t8b_sim_upload_states", self._handle, states)

    def download_events(self):
        out = (Events * self.n)()
        call("t8b_sim_download_events", self._handle, out)
        return out

    def download_legal_mask(self, player: int) -> np.ndarray:
        out = np.zeros((self.n, MAX_CANDIDATES), np.uint8)
        call("t8b_sim_download_legal_mask", self._handle, player, out.ctypes.data_as(C.c_void_p))
        return out

    # ---- environment level
    def reset_all(self, seed: int, counter: int):
        call("t8b_sim_reset_all", self._handle, seed, counter)

    def reset_done(self, seed: int, counter: int):
        call("t8b_sim_reset_done", self._handle, seed, counter)

    def step(self, learner_candidates: torch.Tensor, opponent_candidates: torch.Tensor | None, seed: int, counter: int):
        assert learner_candidates.dtype == torch.int64
        call("t8b_sim_step", self._handle, ptr(learner_candidates),
             ptr(opponent_candidates) if opponent_candidates is not None else None, seed, counter)

    def step_and_reset(self, learner_candidates: torch.Tensor, opponent_candidates: torch.Tensor | None, seed: int,
                       counter: int):
        """step then reset_done with the same seed and counter; finished fights' terminal
        observations are never written."""
        assert learner_candidates.dtype == torch.int64
        call("t8b_sim_step_and_reset", self._handle, ptr(learner_candidates),
             ptr(opponent_candidates) if opponent_candidates is not None else None, seed, counter)

    def _view(self, name, shape, dtype):
        return view(getattr(_lib.lib(), name)(self._handle), shape, dtype, self.device)

    def learner_observations(self):
        return self._view("t8b_sim_learner_observations", (self.n, self.observation_size()), torch.float32)

    def opponent_observations(self):
        return self._view("t8b_sim_opponent_observations", (self.n, self.observation_size()), torch.float32)

    def learner_masks(self):
        return self._view("t8b_sim_learner_masks", (self.n, MAX_CANDIDATES), torch.uint8)

    def opponent_masks(self):
        return self._view("t8b_sim_opponent_masks", (self.n, MAX_CANDIDATES), torch.uint8)

    def learner_mask_bits(self):
        return self._view("t8b_sim_learner_mask_bits", (self.n, MASK_WORDS), torch.int32)

    def opponent_mask_bits(self):
        return self._view("t8b_sim_opponent_mask_bits", (self.n, MASK_WORDS), torch.int32)

    def rewards(self):
        return self._view("t8b_sim_rewards", (self.n,), torch.float32)

    def sparse_rewards(self):
        return self._view("t8b_sim_sparse_rewards", (self.n,), torch.float32)

    def terminated(self):
        return self._view("t8b_sim_terminated", (self.n,), torch.uint8)

    def truncated(self):
        return self._view("t8b_sim_truncated", (self.n,), torch.uint8)

    def outcomes(self):
        return self._view("t8b_sim_outcomes", (self.n,), torch.int8)

    def learner_feature_tables(self):
        return self._view("t8b_sim_learner_feature_tables", (self.n,), torch.int32)

    def opponent_feature_tables(self):
        return self._view("t8b_sim_opponent_feature_tables", (self.n,), torch.int32)

    def download_noise_levels(self):
        out = (NoiseLevels * self.n)()
        call("t8b_sim_download_noise_levels", self._handle, out)
        return out

    def frames_simulated(self) -> int:
        value = C.c_uint64()
        call("t8b_sim_frames_simulated", self._handle, C.byref(value))
        return value.value

    def download_and_clear_tally(self):
        r = self.roster_count
        tally = np.zeros(r * 5 * 2 * 3, np.uint32)
        scenario = np.zeros(9 * 3, np.uint32)
        learner = np.zeros(r * 3, np.uint32)
        bot = np.zeros(331 * 3, np.uint32)
        call("t8b_sim_download_and_clear_tally", self._handle, *(a.ctypes.data_as(C.c_void_p)
                                                                   for a in (tally, scenario, learner, bot)))
        return tally, scenario, learner, bot

    def synchronize(self):
        call("t8b_sim_synchronize", self._handle)

    def random_play(self, p1, p2, p1_x, p2_x, frames: int, seed: int) -> torch.Tensor:
        """The engine-parity workload (include/t8b.h t8b_sim_random_play); returns hashes [fights, frames]."""
        dev = f"cuda:{self.device}"
        p1 = torch.as_tensor(np.asarray(p1, np.int32), device=dev)
        p2 = torch.as_tensor(np.asarray(p2, np.int32), device=dev)
        x1 = torch.as_tensor(np.asarray(p1_x, np.float64), device=dev)
        x2 = torch.as_tensor(np.asarray(p2_x, np.float64), device=dev)
        hashes = torch.empty((p1.shape[0], frames), dtype=torch.int64, device=dev)
        call("t8b_sim_random_play", self._handle, int(p1.shape[0]), ptr(p1), ptr(p2), ptr(x1), ptr(x2), frames,
             seed, ptr(hashes), None)
        return hashes
