"""Data parallelism: the t8b_comm_t hooks over torch.distributed, exercised on CPU with gloo
ranks (world size 2, host buffers), and the update through tests/dp_worker.py: NCCL on two GPUs,
or two gloo ranks sharing one GPU."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _hooks_rank(rank, world, port, out):
    import ctypes as C
    sys.path.insert(0, str(ROOT / "tekken8-agent_b200"))
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                           timeout=timedelta(seconds=60))
    from t8b.policy import TorchComm
    comm = TorchComm(device="cpu")
    assert comm.struct.world_size == world and comm.struct.rank == rank
    f32 = np.arange(1000, dtype=np.float32) * (rank + 1)
    f64 = np.full(7, 0.5 + rank, dtype=np.float64)
    # the library calls the hooks through these function pointers
    comm.struct.allreduce_sum_f32(f32.ctypes.data_as(C.c_void_p), f32.size, None, None)
    comm.struct.allreduce_sum_f64(f64.ctypes.data_as(C.c_void_p), f64.size, None, None)
    comm.struct.allreduce_sum_f64(f64.ctypes.data_as(C.c_void_p), 0, None, None)
    out.put((rank, f32.copy(), f64.copy()))
    dist.barrier()
    dist.destroy_process_group()


def test_comm_hooks_sum_over_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    world, port = 2, free_port()
    out = ctx.Queue()
    procs = [ctx.Process(target=_hooks_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = [out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want32 = np.arange(1000, dtype=np.float32) * 3
    for rank, f32, f64 in results:
        assert np.array_equal(f32, want32)
        assert np.array_equal(f64, np.full(7, 2.0))


def test_native_communicator_makes_unique_ids_without_a_gpu():
    """t8b_comm_unique_id loads NCCL at run time and makes the 128-byte id rank 0 hands to the
    others; a smaller buffer and a null communicator are refused."""
    import ctypes as C
    sys.path.insert(0, str(ROOT / "tekken8-agent_b200"))
    from t8b import _lib
    lib = _lib.lib()
    first, second = (C.c_char * 128)(), (C.c_char * 128)()
    assert lib.t8b_comm_unique_id(first, 128) == 0, lib.t8b_last_error()
    assert lib.t8b_comm_unique_id(second, 128) == 0
    assert bytes(first) != bytes(second) and any(bytes(first))
    assert lib.t8b_comm_unique_id(first, 64) == _lib.T8B_EINVAL
    assert lib.t8b_comm_status(None) == _lib.T8B_EINVAL
    assert lib.t8b_comm_destroy(None) == 0


def _max_rank(rank, world, port, out):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                           timeout=timedelta(seconds=60))
    import bench
    out.put(bench.max_over_ranks([10.0 + rank, 5.0 - rank], "cpu"))
    dist.destroy_process_group()


def test_bench_times_are_the_max_over_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    world, port = 2, free_port()
    out = ctx.Queue()
    procs = [ctx.Process(target=_max_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = [out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r == [11.0, 5.0] for r in results)


@pytest.mark.gpu
def test_data_parallel_update_on_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "dp_worker.py")]
    run = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-3000:]
    assert "DP OK" in run.stdout


@pytest.mark.gpu
def test_data_parallel_update_two_ranks_on_one_gpu():
    """The data-parallel semantics of tests/dp_worker.py on a one-GPU machine: two ranks share
    cuda:0 and the library's sum hooks go through gloo (no device-side waits between the ranks).
    Identical shards equal the single-rank run bit for bit, the rank-merged advantage statistics
    equal the single-rank ones, and different shards keep the replicas bit-identical."""
    env = dict(os.environ, T8B_DP_BACKEND="gloo")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "dp_worker.py")]
    run = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-3000:]
    assert "DP OK" in run.stdout
