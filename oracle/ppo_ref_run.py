"""Test infrastructure (not product code): ctypes access to oracle/_ref/libt8ppo_ref.so, the
reference's own GpuActorCritic and GpuRolloutBuffer (src/ppo.cu) built for sm_100a by
oracle/Makefile, so GPU tests can run the reference beside the library on the same inputs.
Used only by tests/."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libt8ppo_ref.so"


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("observation_size", "action_count", "hidden_size", "action_feature_size",
                                       "universal_action_count", "shared_layers", "head_layers",
                                       "observation_normalization", "orthogonal_initialization")] + \
               [("observation_clip", C.c_float), ("observation_epsilon", C.c_float),
                ("matmul_precision", C.c_char * 8)]


class Ppo(C.Structure):
    _fields_ = [("epochs", C.c_int), ("minibatch_size", C.c_size_t)] + \
               [(n, C.c_float) for n in ("learning_rate", "clip_range", "value_clip_range", "target_kl",
                                         "value_coefficient", "entropy_coefficient", "max_gradient_norm",
                                         "adam_beta1", "adam_beta2", "adam_epsilon")]


METRICS = ("policy_loss", "value_loss", "entropy", "approximate_kl", "clip_fraction", "gradient_norm",
           "decision_fraction", "decision_entropy", "rollout_decision_entropy", "minibatches", "epochs_completed",
           "early_stopped")

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            from oracle import ref
            ref.build()
        h = C.CDLL(str(LIB))
        vp, sz, u64 = C.c_void_p, C.c_size_t, C.c_uint64
        h.t8pr_last_error.restype = C.c_char_p
        h.t8pr_policy_create.argtypes = [C.POINTER(Config), sz, u64, C.POINTER(vp)]
        h.t8pr_policy_destroy.argtypes = [vp]
        h.t8pr_policy_parameter_count.restype = sz
        h.t8pr_policy_parameter_count.argtypes = [vp]
        h.t8pr_policy_set_features.argtypes = [vp, vp, sz, C.c_int]
        h.t8pr_policy_forward.argtypes = [vp, vp, vp, sz, u64, u64, C.c_int, vp, C.POINTER(vp)]
        h.t8pr_policy_update.argtypes = [vp, C.POINTER(vp), sz, sz, sz, C.POINTER(Ppo), u64, C.POINTER(C.c_double)]
        h.t8pr_policy_save.argtypes = [vp, C.c_char_p]
        h.t8pr_policy_load.argtypes = [vp, C.c_char_p, C.c_int]
        h.t8pr_policy_observation_statistics.argtypes = [vp, vp, C.POINTER(u64)]
        h.t8pr_rollout_create.argtypes = [sz, sz, C.POINTER(Config), C.POINTER(vp)]
        h.t8pr_rollout_destroy.argtypes = [vp]
        h.t8pr_rollout_record_policy.argtypes = [vp, sz, vp, vp, vp, vp, vp, vp, vp]
        h.t8pr_rollout_record_outcome.argtypes = [vp, sz, vp, vp, vp, vp, C.c_float]
        h.t8pr_rollout_compute_gae.argtypes = [vp, C.c_float, C.c_float, C.c_int]
        h.t8pr_rollout_normalize_rewards.argtypes = [vp, C.c_float, C.c_float, C.POINTER(C.c_float)]
        h.t8pr_rollout_download.argtypes = [vp, vp, vp, vp]
        h.t8pr_rollout_view.argtypes = [vp, C.POINTER(vp)]
        _lib = h
    return _lib


def _ok(status):
    if status != 0:
        raise RuntimeError(lib().t8pr_last_error().decode())


def config_from(actor, matmul: str = "bf16") -> Config:
    """The reference ActorCriticConfig matching the library's t8b_actor_config_t."""
    return Config(actor.observation_size, actor.action_count, actor.hidden_size, actor.action_feature_size,
                  actor.universal_action_count, actor.shared_layers, actor.head_layers,
                  actor.observation_normalization, actor.orthogonal_initialization, actor.observation_clip,
                  actor.observation_epsilon, matmul.encode())


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


class RefPolicy:
    def __init__(self, config: Config, capacity: int, seed: int):
        self.config = config
        handle = C.c_void_p()
        _ok(lib().t8pr_policy_create(C.byref(config), capacity, seed, C.byref(handle)))
        self.handle = handle

    def __del__(self):
        if getattr(self, "handle", None) and _lib is not None:
            _lib.t8pr_policy_destroy(self.handle)
            self.handle = None

    def parameter_count(self) -> int:
        return lib().t8pr_policy_parameter_count(self.handle)

    def set_features(self, features: np.ndarray):
        f = np.ascontiguousarray(features, np.float32)
        _ok(lib().t8pr_policy_set_features(self.handle, f.ctypes.data, f.size, f.shape[0]))

    def forward(self, obs, masks, n, seed, step, deterministic=False, tables=None):
        """Device tensors in; host copies of actions, log-probabilities, values, entropies out."""
        import torch
        from t8b.device import view
        out = (C.c_void_p * 5)()
        _ok(lib().t8pr_policy_forward(self.handle, _ptr(obs), _ptr(masks), n, seed, step, 1 if deterministic else 0,
                                      _ptr(tables), out))
        device = torch.cuda.current_device()
        return {"logits": view(out[0], (n, self.config.action_count), torch.float32, device).cpu().numpy(),
                "actions": view(out[1], (n,), torch.int64, device).cpu().numpy(),
                "log_probabilities": view(out[2], (n,), torch.float32, device).cpu().numpy(),
                "values": view(out[3], (n,), torch.float32, device).cpu().numpy(),
                "entropies": view(out[4], (n,), torch.float32, device).cpu().numpy()}

    def update(self, pointers, environments, horizon, samples, ppo: Ppo, shuffle_seed):
        arr = (C.c_void_p * 13)(*pointers)
        metrics = (C.c_double * 12)()
        _ok(lib().t8pr_policy_update(self.handle, arr, environments, horizon, samples, C.byref(ppo), shuffle_seed,
                                     metrics))
        return dict(zip(METRICS, list(metrics)))

    def save(self, path):
        _ok(lib().t8pr_policy_save(self.handle, str(path).encode()))

    def load(self, path, load_optimizer_state=True):
        _ok(lib().t8pr_policy_load(self.handle, str(path).encode(), 1 if load_optimizer_state else 0))

    def observation_statistics(self):
        w = self.config.observation_size
        buf = np.zeros(2 * w, np.float32)
        count = C.c_uint64()
        _ok(lib().t8pr_policy_observation_statistics(self.handle, buf.ctypes.data, C.byref(count)))
        return buf[:w], buf[w:], count.value


class RefRollout:
    def __init__(self, environments: int, horizon: int, config: Config):
        self.environments, self.horizon = environments, horizon
        handle = C.c_void_p()
        _ok(lib().t8pr_rollout_create(environments, horizon, C.byref(config), C.byref(handle)))
        self.handle = handle

    def __del__(self):
        if getattr(self, "handle", None) and _lib is not None:
            _lib.t8pr_rollout_destroy(self.handle)
            self.handle = None

    def record_policy(self, step, obs, masks, actions, log_probs, values, tables=None, entropies=None):
        _ok(lib().t8pr_rollout_record_policy(self.handle, step, _ptr(obs), _ptr(masks), _ptr(actions), _ptr(log_probs),
                                             _ptr(values), _ptr(tables), _ptr(entropies)))

    def record_outcome(self, step, rewards, terminated, truncated, next_values, reward_scale=1.0):
        _ok(lib().t8pr_rollout_record_outcome(self.handle, step, _ptr(rewards), _ptr(terminated), _ptr(truncated),
                                              _ptr(next_values), reward_scale))

    def compute_gae(self, gamma, gae_lambda, normalize=True):
        _ok(lib().t8pr_rollout_compute_gae(self.handle, gamma, gae_lambda, 1 if normalize else 0))

    def normalize_rewards(self, gamma, clip=10.0) -> float:
        out = C.c_float()
        _ok(lib().t8pr_rollout_normalize_rewards(self.handle, gamma, clip, C.byref(out)))
        return out.value

    def download(self):
        shape = (self.horizon, self.environments)
        a, r, w = (np.zeros(shape, np.float32) for _ in range(3))
        _ok(lib().t8pr_rollout_download(self.handle, a.ctypes.data, r.ctypes.data, w.ctypes.data))
        return a, r, w

    def view(self):
        out = (C.c_void_p * 13)()
        _ok(lib().t8pr_rollout_view(self.handle, out))
        return list(out)
