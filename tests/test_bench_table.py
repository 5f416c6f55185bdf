"""bench.py's per-kernel roofline table (CPU, no GPU): the algorithmic work it charges each
kernel label with. With the fused inference forward (k_forward_tc) in the profile, the layer
GEMMs' forward labels count the update's samples only and the fused kernel the rollout's; the
fused forward is tensor bound, the frame step and the objective HBM bound."""
import importlib.util
from pathlib import Path
from types import SimpleNamespace

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def table(bench, profile, steps=2):
    args = SimpleNamespace(envs=32768, horizon=128, epochs=4, minibatches=8)
    rows = bench.kernel_table(args, profile, steps, (6450.6, 1425.6))
    return {row["kernel"]: row for row in rows}


def test_fused_forward_counts_rollout_samples(bench):
    steps = 2
    rows = table(bench, {"k_forward_tc": (129 * steps, 9.4 * steps), "gemm_forward_hidden": (64 * steps, 15.0 * steps),
                         "k_step": (128 * steps, 237.0 * steps)}, steps)
    rollout = 129 * 32768
    update = 4 * 128 * 32768
    fused = rows["k_forward_tc"]
    flops = bench.GEMM_FLOPS_PER_SAMPLE["k_forward_tc"]
    assert flops == 2 * (151 * 512 + 512 * 512 + 512 * 33)
    assert fused["bound"] == "tensor" and fused["unit"] == "TFLOP/s"
    assert fused["achieved"] == pytest.approx(flops * rollout / 9.4e-3 / 1e12)
    assert fused["frac"] == pytest.approx(fused["achieved"] / 1425.6)
    hidden = rows["gemm_forward_hidden"]
    assert hidden["tensor_tflops"] == pytest.approx(bench.GEMM_FLOPS_PER_SAMPLE["gemm_forward_hidden"] * update / 15.0e-3 / 1e12)
    step = rows["k_step"]
    assert step["bound"] == "hbm"
    assert step["achieved"] == pytest.approx(bench.STEP_BYTES_PER_ENV * 32768 * 128 / 237.0e-3 / 1e9)
    assert sum(row["share"] for row in rows.values()) == pytest.approx(1.0)


def test_layer_gemms_count_the_rollout_without_the_fused_forward(bench):
    rows = table(bench, {"gemm_forward_hidden": (322, 25.0)}, 1)
    samples = 129 * 32768 + 4 * 128 * 32768
    want = bench.GEMM_FLOPS_PER_SAMPLE["gemm_forward_hidden"] * samples / 25.0e-3 / 1e12
    assert rows["gemm_forward_hidden"]["tensor_tflops"] == pytest.approx(want)
