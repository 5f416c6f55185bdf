"""The reference's own driver programs, unchanged, running on the library (the drop-in check).

oracle/Makefile (target `relinked`) compiles the reference's full-move benchmark
(benchmarks/full_move_throughput.cpp), trainer (src/full_move_train.cpp) and arena
(src/full_move_arena.cpp) against the reference's headers and links them with the shim
(tekken8-agent_b200/shim: GpuFullMoveSimulator, GpuActorCritic and GpuRolloutBuffer over
include/t8b.h) and libt8b.so, in place of src/full_move_gpu.cu and src/ppo.cu. These tests run
those binaries on the GPU:
  * the benchmark prints its JSON line (benchmarks/full_move_throughput.cpp:128-138);
  * the trainer resumes exactly: a run resumed from its update-2 checkpoint writes an update-4
    checkpoint byte-identical to the uninterrupted run's, through scripted and mirror self-play
    updates (the property the reference's tests/full_move_resume_smoke.py:42-79 checks), and a
    resume with a different gamma is refused;
  * the arena plays the trainer's checkpoints (read through their .t8fmstate) and writes its CSV.
The trainer's network is 128 wide (the library's hidden sizes are multiples of 128)."""
import json
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

RELINKED = ROOT / "oracle" / "_ref" / "relinked"
DATA = ROOT / "oracle" / "_ref" / "data" / "generated"


def program(name):
    path = RELINKED / name
    if not path.exists():
        pytest.fail(f"{path} is missing: build it with `make -C oracle relinked` where the reference is present")
    return str(path)


def run(arguments, timeout=600):
    return subprocess.run(arguments, capture_output=True, text=True, timeout=timeout)


def test_reference_benchmark_runs_on_the_library(cuda):
    done = run([program("t8_v2_full_move_benchmark"), "--envs", "32768", "--horizon", "16", "--updates", "2",
                "--minibatch", "131072", "--epochs", "1", "--hidden", "512", "--data-dir", str(DATA)])
    assert done.returncode == 0, done.stderr
    line = json.loads(done.stdout.strip().splitlines()[-1])
    print("relinked benchmark:", line)
    assert line["environments"] == 32768 and line["updates"] == 2
    for key in ("simulator_decisions_per_second", "training_decisions_per_second", "simulator_frames_per_second"):
        assert line[key] > 0, key


COMMON = ["--envs", "64", "--horizon", "8", "--epochs", "1", "--minibatch", "256", "--hidden", "128",
          "--eval-interval", "2", "--eval-episodes", "16", "--checkpoint-interval", "2", "--anneal-updates", "6",
          "--learner-character", "jun,king", "--opponents", "jun,king,alisa", "--allow-provisional",
          "--entropy-target", "6", "--draw-penalty", "0.5", "--throw-break-penalty", "0.03", "--time-penalty", "0.01",
          "--hold-frames", "6", "--self-play-share", "0.5", "--self-play-start", "1", "--seed", "4401"]


def test_reference_trainer_resumes_exactly_on_the_library(cuda, tmp_path):
    trainer = program("t8_v2_full_move_train")
    common = COMMON + ["--data-dir", str(DATA)]
    straight, resumed = tmp_path / "straight", tmp_path / "resumed"
    done = run([trainer, *common, "--updates", "4", "--run-dir", str(straight)])
    assert done.returncode == 0, done.stderr[-2000:]
    done = run([trainer, *common, "--updates", "2", "--run-dir", str(resumed)])
    assert done.returncode == 0, done.stderr[-2000:]
    checkpoint = resumed / "checkpoints" / "update_2.t8ppo"
    assert checkpoint.exists()
    refused = run([trainer, *common, "--updates", "4", "--gamma", "0.9", "--run-dir", str(resumed),
                   "--resume", str(checkpoint)])
    assert refused.returncode != 0, "the trainer resumed with a different gamma"
    done = run([trainer, *common, "--updates", "4", "--run-dir", str(resumed), "--resume", str(checkpoint)])
    assert done.returncode == 0, done.stderr[-2000:]
    name = "update_4.t8ppo"
    assert (straight / "checkpoints" / name).read_bytes() == (resumed / "checkpoints" / name).read_bytes()
    modes = (straight / "metrics.jsonl").read_text()
    assert "self_play_mirror" in modes and "scripted_full_move" in modes
    # the arena over the trainer's checkpoints
    table = tmp_path / "arena.csv"
    done = run([program("t8_v2_full_move_arena"), "--output", str(table), "--rounds-per-pair", "8",
                "--allow-provisional", "--data-dir", str(DATA), "--hold-frames", "6",
                str(straight / "checkpoints" / "update_2.t8ppo"), str(straight / "checkpoints" / name)])
    assert done.returncode == 0, done.stderr[-2000:]
    rows = table.read_text().strip().splitlines()
    assert len(rows) >= 2, rows
