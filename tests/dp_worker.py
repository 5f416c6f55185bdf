"""Data-parallel worker, run as `torchrun --nproc-per-node 2 tests/dp_worker.py` (one rank per
GPU, NCCL): the PPO update and the rollout statistics with the gradient, KL, observation
normaliser and advantage moments summed over ranks. With T8B_DP_BACKEND=gloo every rank runs on
cuda:0 and the hooks' sums go through gloo (host copies), so the same checks run on a one-GPU
machine; the library's own NCCL communicator needs a GPU per rank and is checked only with NCCL.

Checks, printing "DP OK" on rank 0 when all hold:
  * identical shards on every rank give bit-identical parameters, Adam state, normaliser mean
    and variance and advantages to a single-GPU run on one shard (a mean of equal gradients is
    the gradient; merged equal moments are the moments);
  * different shards keep the replicas bit-identical after several updates."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tekken8-agent_b200"))
sys.path.insert(0, str(ROOT / "tests"))

import lzma  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


BACKEND = os.environ.get("T8B_DP_BACKEND", "nccl")


def gather(array: np.ndarray) -> list[np.ndarray]:
    t = torch.as_tensor(np.ascontiguousarray(array))
    if BACKEND == "nccl":
        t = t.cuda()
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.cpu().numpy() for o in out]


def main():
    local = int(os.environ["LOCAL_RANK"]) if BACKEND == "nccl" else 0
    torch.cuda.set_device(local)
    if BACKEND == "nccl":
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    else:
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    from t8b import roster as roster_module
    from t8b.policy import GpuActorCritic, GpuRolloutBuffer, TorchComm, actor_config, ppo_config
    from test_ppo_gpu import rollout_inputs, view_of
    roster = roster_module.parse(lzma.decompress((ROOT / "tests" / "golden" / "roster41.bin.xz").read_bytes()))
    features = roster.feature_tables()
    comm = TorchComm()
    n = 4096
    cfg = ppo_config(epochs=2, minibatch_size=n // 4, target_kl=0.0)

    # identical shards: DP equals one GPU
    runs = {}
    for name, use_comm in (("single", False), ("dp", True)):
        policy = GpuActorCritic(n, seed=31)
        policy.set_action_feature_tables(features)
        if use_comm:
            policy.set_comm(comm)
        arrays = rollout_inputs(policy, features, n, np.random.default_rng(8))
        view, keep = view_of(arrays)
        policy.update_ppo(view, cfg, shuffle_seed=5)
        mean, var, count = policy.observation_statistics()
        m1, m2, step = policy.optimizer_state()
        runs[name] = (policy.parameters(), m1, m2, mean, var, count)
    s, d = runs["single"], runs["dp"]
    for k in range(5):
        assert np.array_equal(s[k], d[k]), f"identical shards: item {k} differs from the single-GPU run"
    assert d[5] == world * s[5]

    # rollout advantages with statistics over ranks: identical shards give the single-GPU values
    t, envs = 8, 512
    rng = np.random.default_rng(3)
    rewards = torch.as_tensor(rng.normal(size=(t, envs)).astype(np.float32)).cuda()
    values = torch.as_tensor(rng.normal(size=(t, envs)).astype(np.float32)).cuda()
    done = torch.as_tensor((rng.random((t, envs)) < 0.05).astype(np.uint8)).cuda()
    zeros = torch.zeros((t, envs), dtype=torch.uint8, device="cuda")
    advantages = []
    for use_comm in (False, True):
        buf = GpuRolloutBuffer(envs, t, actor_config())
        if use_comm:
            buf.set_comm(comm)
        for step in range(t):
            buf.record_outcome_device(step, rewards[step], done[step], zeros[step], values[step])
        buf.compute_gae(0.99, 0.95, True)
        advantages.append(buf.tensor("advantages").cpu().numpy().copy())
    assert np.array_equal(advantages[0], advantages[1]), "advantage normalisation differs over ranks"

    # different shards: replicas stay identical
    policy = GpuActorCritic(n, seed=33)
    policy.set_action_feature_tables(features)
    policy.set_comm(comm)
    for update in range(3):
        arrays = rollout_inputs(policy, features, n, np.random.default_rng(100 + 10 * rank + update))
        view, keep = view_of(arrays)
        policy.update_ppo(view, cfg, shuffle_seed=50 + update)
    params = gather(policy.parameters())
    mean = gather(policy.observation_statistics()[0])
    for r in range(1, world):
        assert np.array_equal(params[0], params[r]), f"rank {r} parameters diverged"
        assert np.array_equal(mean[0], mean[r]), f"rank {r} normaliser diverged"

    # the library's own NCCL communicator (t8b_comm_init) gives the same replicas as the
    # torch.distributed hooks: the same sums in the same order, queued from C
    if BACKEND == "nccl":
        from t8b.policy import NativeComm
        native = NativeComm()
        twin = GpuActorCritic(n, seed=33)
        twin.set_action_feature_tables(features)
        twin.set_comm(native)
        for update in range(3):
            arrays = rollout_inputs(twin, features, n, np.random.default_rng(100 + 10 * rank + update))
            view, keep = view_of(arrays)
            twin.update_ppo(view, cfg, shuffle_seed=50 + update)
        torch.cuda.synchronize()
        native.status()
        assert np.array_equal(twin.parameters(), policy.parameters()), "native communicator differs from torch's"
        assert np.array_equal(twin.observation_statistics()[0], policy.observation_statistics()[0])
        native.close()
    dist.barrier()
    if rank == 0:
        print("DP OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
