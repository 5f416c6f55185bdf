"""GpuActorCritic and GpuRolloutBuffer: the reference classes (include/t8_v2/ppo.hpp:112-291)
over the t8b_policy_* / t8b_rollout_* entry points. Device data are torch tensors or raw
device pointers; host data are numpy arrays."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import ActorConfig, CheckpointContract, PpoConfig, PpoMetrics, PolicyOutput, RolloutView, Comm, call
from .device import view, ptr


def actor_config(**overrides) -> ActorConfig:
    """ActorCriticConfig with the full-move trainer's settings (src/full_move_train.cpp:1158-1172)."""
    config = ActorConfig()
    _lib.lib().t8b_actor_config_default(C.byref(config))
    for key, value in overrides.items():
        if not hasattr(config, key):
            raise AttributeError(key)
        setattr(config, key, value)
    return config


def ppo_config(**overrides) -> PpoConfig:
    config = PpoConfig()
    _lib.lib().t8b_ppo_config_default(C.byref(config))
    for key, value in overrides.items():
        if not hasattr(config, key):
            raise AttributeError(key)
        setattr(config, key, value)
    return config


def _p(value):
    if value is None:
        return None
    if isinstance(value, int):
        return value
    return ptr(value)


def checkpoint_contract(catalog_sha256: str = "0" * 64, roster_version: str = "compatibility",
                        observation_contract: str = "v2-observation",
                        action_contract: str = "fixed-24-compatibility") -> CheckpointContract:
    """The text fields a checkpoint must agree on (the reference ActorCriticConfig's defaults)."""
    return CheckpointContract(catalog_sha256.encode(), roster_version.encode(), observation_contract.encode(),
                              action_contract.encode())


class TorchComm:
    """t8b_comm_t over torch.distributed: sum all-reduces on tensors aliasing the library's
    buffers. On CUDA (NCCL) the reduce is ordered on the stream the library passes; with
    device="cpu" the buffers are host memory (gloo), which is how the hooks are exercised
    without a GPU."""

    def __init__(self, group=None, device: str = "cuda"):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.host = device == "cpu"
        self.device = None if self.host else torch.cuda.current_device()

        def f32(pointer, count, stream, user):
            self._reduce(pointer, count, torch.float32, stream)

        def f64(pointer, count, stream, user):
            self._reduce(pointer, count, torch.float64, stream)

        self._f32 = _lib.ALLREDUCE_F32(f32)
        self._f64 = _lib.ALLREDUCE_F64(f64)
        self.struct = Comm(self._f32, self._f64, None, self.world, self.rank)

    def _reduce(self, pointer, count, dtype, stream):
        if count == 0:
            return
        if self.host:
            ctype = C.c_float if dtype == torch.float32 else C.c_double
            tensor = torch.frombuffer((ctype * count).from_address(pointer), dtype=dtype)
            self.dist.all_reduce(tensor, op=self.dist.ReduceOp.SUM, group=self.group)
            return
        tensor = view(pointer, (count,), dtype, self.device)
        if stream:
            with torch.cuda.stream(torch.cuda.ExternalStream(stream, device=self.device)):
                self.dist.all_reduce(tensor, op=self.dist.ReduceOp.SUM, group=self.group)
        else:
            self.dist.all_reduce(tensor, op=self.dist.ReduceOp.SUM, group=self.group)


class NativeComm:
    """t8b_comm_t from the library's own NCCL communicator (t8b_comm_init): the all-reduces are
    queued in C on the library's stream, with no Python between the kernels. torch.distributed
    (any backend) only carries rank 0's 128-byte unique id to the other ranks."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        box = [None]
        if self.rank == 0:
            raw = (C.c_char * 128)()
            call("t8b_comm_unique_id", raw, 128)
            box[0] = bytes(raw)
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        self.struct = Comm()
        call("t8b_comm_init", box[0], 128, self.world, self.rank, C.byref(self.struct))

    def status(self):
        call("t8b_comm_status", C.byref(self.struct))

    def close(self):
        if self.struct.user:
            call("t8b_comm_destroy", C.byref(self.struct))


class GpuActorCritic:
    def __init__(self, capacity: int, config: ActorConfig | None = None, seed: int = 2027):
        self.config = config if config is not None else actor_config()
        handle = C.c_void_p()
        call("t8b_policy_create", capacity, C.byref(self.config), seed, C.byref(handle))
        self._handle = handle
        self.capacity = capacity
        self.device = torch.cuda.current_device()
        self._comm = None

    def close(self):
        if getattr(self, "_handle", None):
            call("t8b_policy_destroy", self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._handle

    def parameter_count(self) -> int:
        return _lib.lib().t8b_policy_parameter_count(self._handle)

    def set_action_feature_tables(self, features: np.ndarray, stream=None):
        features = np.ascontiguousarray(features, np.float32)
        call("t8b_policy_set_action_feature_tables", self._handle, features.ctypes.data_as(C.c_void_p),
             int(features.shape[0]), stream)

    def forward(self, observations, masks=None, n=None, seed=0, step=0, deterministic=False, stream=None, tables=None,
                mask_bits=None, want_logits=False) -> dict:
        n = int(n if n is not None else observations.shape[0])
        out = PolicyOutput()
        call("t8b_policy_forward", self._handle, _p(observations), _p(masks), _p(mask_bits), n, seed, step,
             1 if deterministic else 0, stream, _p(tables), 1 if want_logits else 0, C.byref(out))
        d = self.device
        result = {"actions": view(out.actions, (n,), torch.int64, d),
                  "log_probabilities": view(out.log_probabilities, (n,), torch.float32, d),
                  "values": view(out.values, (n,), torch.float32, d),
                  "entropies": view(out.entropies, (n,), torch.float32, d)}
        if want_logits:
            result["logits"] = view(out.logits, (n, self.config.action_count), torch.float32, d)
        return result

    def prepare_shuffle(self, samples: int, epochs: int, seed: int):
        call("t8b_policy_prepare_shuffle", self._handle, samples, epochs, seed)

    def update_ppo(self, rollout_view: RolloutView, config: PpoConfig | None = None, shuffle_seed: int = 2027,
                   stream=None) -> dict:
        metrics = PpoMetrics()
        call("t8b_policy_update_ppo", self._handle, C.byref(rollout_view), C.byref(config or ppo_config()),
             shuffle_seed, stream, C.byref(metrics))
        return metrics.as_dict()

    def set_comm(self, comm: TorchComm | None):
        self._comm = comm
        call("t8b_policy_set_comm", self._handle, C.byref(comm.struct) if comm else None)

    def save_checkpoint(self, path, contract: CheckpointContract | None = None, stream=None):
        """GpuActorCritic::save_checkpoint: the reference's .t8ppo file (refuses to overwrite)."""
        call("t8b_policy_save_checkpoint", self._handle, str(path).encode(), C.byref(contract) if contract else None,
             stream)

    def load_checkpoint(self, path, load_optimizer_state: bool = True, contract: CheckpointContract | None = None,
                        stream=None):
        """GpuActorCritic::load_checkpoint; adopts the file's observation-normaliser setting."""
        call("t8b_policy_load_checkpoint", self._handle, str(path).encode(), 1 if load_optimizer_state else 0,
             C.byref(contract) if contract else None, stream)

    def _host(self, name, count, dtype=np.float32):
        out = np.zeros(count, dtype)
        call(name, self._handle, out.ctypes.data_as(C.c_void_p), count)
        return out

    def parameters(self) -> np.ndarray:
        return self._host("t8b_policy_get_parameters", self.parameter_count())

    def set_parameters(self, values: np.ndarray):
        values = np.ascontiguousarray(values, np.float32)
        call("t8b_policy_set_parameters", self._handle, values.ctypes.data_as(C.c_void_p), values.size)

    def gradients(self) -> np.ndarray:
        return self._host("t8b_policy_get_gradients", self.parameter_count())

    def optimizer_state(self):
        n = self.parameter_count()
        m1, m2 = np.zeros(n, np.float32), np.zeros(n, np.float32)
        step = C.c_uint64()
        call("t8b_policy_get_optimizer_state", self._handle, m1.ctypes.data_as(C.c_void_p),
             m2.ctypes.data_as(C.c_void_p), C.byref(step))
        return m1, m2, step.value

    def observation_statistics(self):
        w = self.config.observation_size
        mean, var = np.zeros(w, np.float32), np.zeros(w, np.float32)
        count = C.c_uint64()
        call("t8b_policy_get_observation_statistics", self._handle, mean.ctypes.data_as(C.c_void_p),
             var.ctypes.data_as(C.c_void_p), C.byref(count))
        return mean, var, count.value

    def set_observation_statistics(self, mean, variance, count):
        mean = np.ascontiguousarray(mean, np.float32)
        variance = np.ascontiguousarray(variance, np.float32)
        call("t8b_policy_set_observation_statistics", self._handle, mean.ctypes.data_as(C.c_void_p),
             variance.ctypes.data_as(C.c_void_p), count)

    def outputs(self, n: int) -> np.ndarray:
        width = self.config.action_feature_size + 1
        out = np.zeros((n, width), np.float32)
        call("t8b_policy_download_outputs", self._handle, out.ctypes.data_as(C.c_void_p), n)
        return out

    def activation(self, which: int, layer: int, n: int) -> np.ndarray:
        width = {0: (self.config.observation_size + 63) // 64 * 64, 3: 64}.get(which, self.config.hidden_size)
        out = np.zeros((n, width), np.float32)
        call("t8b_policy_download_activation", self._handle, which, layer, out.ctypes.data_as(C.c_void_p), n)
        return out

    def synchronize(self, stream=None):
        call("t8b_policy_synchronize", self._handle, stream)


class GpuRolloutBuffer:
    def __init__(self, environments: int, horizon: int, config: ActorConfig | None = None):
        self.config = config if config is not None else actor_config()
        handle = C.c_void_p()
        call("t8b_rollout_create", environments, horizon, C.byref(self.config), C.byref(handle))
        self._handle = handle
        self.environments = environments
        self.horizon = horizon
        self.samples = environments * horizon
        self.device = torch.cuda.current_device()

    def close(self):
        if getattr(self, "_handle", None):
            call("t8b_rollout_destroy", self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_view(self, packed: bool = False) -> RolloutView:
        """GpuRolloutView; packed=True leaves the uint8 masks unexpanded (action_masks NULL)."""
        v = RolloutView()
        call("t8b_rollout_packed_view" if packed else "t8b_rollout_device_view", self._handle, C.byref(v))
        return v

    def record_policy_device(self, step, observations, masks=None, actions=None, log_probabilities=None, values=None,
                             stream=None, feature_tables=None, entropies=None, mask_bits=None):
        call("t8b_rollout_record_policy_device", self._handle, step, _p(observations), _p(masks), _p(mask_bits),
             _p(actions), _p(log_probabilities), _p(values), stream, _p(feature_tables), _p(entropies))

    def record_outcome_device(self, step, rewards, terminated, truncated, next_values, reward_scale=1.0, stream=None):
        call("t8b_rollout_record_outcome_device", self._handle, step, _p(rewards), _p(terminated), _p(truncated),
             _p(next_values), reward_scale, stream)

    def compute_gae(self, gamma=0.997, gae_lambda=0.95, normalize=True, stream=None):
        call("t8b_rollout_compute_gae", self._handle, gamma, gae_lambda, 1 if normalize else 0, stream)

    def normalize_rewards(self, gamma, clip=10.0, stream=None) -> float:
        out = C.c_float()
        call("t8b_rollout_normalize_rewards", self._handle, gamma, clip, stream, C.byref(out))
        return out.value

    def mean_reward(self, stream=None) -> float:
        out = C.c_double()
        call("t8b_rollout_mean_reward", self._handle, stream, C.byref(out))
        return out.value

    def return_normalizer_state(self):
        count, mean, var = C.c_uint64(), C.c_double(), C.c_double()
        returns = np.zeros(self.environments, np.float32)
        call("t8b_rollout_return_normalizer_state", self._handle, C.byref(count), C.byref(mean), C.byref(var),
             returns.ctypes.data_as(C.c_void_p))
        return count.value, mean.value, var.value, returns

    def restore_return_normalizer_state(self, count, mean, variance, returns):
        returns = np.ascontiguousarray(returns, np.float32)
        call("t8b_rollout_restore_return_normalizer_state", self._handle, count, mean, variance,
             returns.ctypes.data_as(C.c_void_p))

    def set_comm(self, comm: TorchComm | None):
        self._comm = comm
        call("t8b_rollout_set_comm", self._handle, C.byref(comm.struct) if comm else None)

    def tensor(self, name: str) -> torch.Tensor:
        """A zero-copy torch view of one field of the device view ([horizon, envs] or
        [horizon, envs, width])."""
        v = self.device_view(packed=name != "action_masks")  # the uint8 masks are expanded only when asked for
        t, n = self.horizon, self.environments
        spec = {
            "observations": ((t, n, self.config.observation_size), torch.float32),
            "action_masks": ((t, n, self.config.action_count), torch.uint8),
            "action_mask_bits": ((t, n, 12), torch.int32),
            "actions": ((t, n), torch.int64), "old_log_probabilities": ((t, n), torch.float32),
            "old_values": ((t, n), torch.float32), "rewards": ((t, n), torch.float32),
            "terminated": ((t, n), torch.uint8), "truncated": ((t, n), torch.uint8),
            "next_values": ((t, n), torch.float32), "advantages": ((t, n), torch.float32),
            "returns": ((t, n), torch.float32), "feature_tables": ((t, n), torch.int32),
            "entropies": ((t, n), torch.float32),
        }[name]
        return view(getattr(v, name), spec[0], spec[1], self.device)


def ppo_output_gradient(outputs: torch.Tensor, masks: torch.Tensor, actions: torch.Tensor, old_lp: torch.Tensor,
                        old_v: torch.Tensor, adv: torch.Tensor, ret: torch.Tensor, config: PpoConfig | None = None,
                        stream=None, metrics: bool = True):
    """debug_ppo_objective_gradient (include/t8_v2/ppo.hpp:100-108) over a batch: returns the
    [n, k + 1] gradient and the eight metric sums."""
    n, width = outputs.shape
    grads = torch.empty_like(outputs)
    sums = torch.zeros(8, dtype=torch.float64, device=outputs.device) if metrics else None
    call("t8b_ppo_output_gradient", ptr(outputs), ptr(masks), ptr(actions), ptr(old_lp), ptr(old_v), ptr(adv),
         ptr(ret), n, width - 1, C.byref(config or ppo_config()), ptr(grads), ptr(sums) if metrics else None, stream)
    return grads, sums
