"""Regenerates the golden fixtures from the reference itself (run where the reference checkout is).

  roster41.bin.xz   the 41 fighters with moves, loaded by the reference's own loader
                    (src/full_move_roster.cpp:51, stand-in geometry as the trainer's
                    allow_provisional) and written in the include/t8b.h boundary layout;
  engine_trace.npz  the engine-parity workload (include/t8b.h t8b_sim_random_play) on the
                    reference's full_core::step: per-frame FNV-1a state hashes;
  env_trace.npz     the environment contract (screen view + live noise, scripted bots and the
                    random opponent, every scenario) run by the reference's functions: per-step
                    digests of observations, masks, rewards, flags and states.
The oracle library oracle/_ref/libt8ref.so is built by oracle/Makefile from the reference
sources; this script only calls it.
"""
from __future__ import annotations

import hashlib
import lzma
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tekken8-agent_b200"))

from oracle import ref  # noqa: E402

GENERATED = str(ref.REFERENCE / "data" / "generated")


def digest(array: np.ndarray) -> bytes:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).digest()[:8]


def env_run(raw: bytes, n: int, steps: int, config, seed: int, opponents, aggression, scenarios, learner_is_p1, p1, p2,
            pick_seed: int):
    """Drives the reference environment with learner picks derived from its own masks; returns
    the digests per step and the learner actions taken."""
    roster = ref.RefRoster(raw)
    env = ref.RefEnv(roster, n, config, threads=8)
    env.setup(p1=p1, p2=p2, learner_is_p1=learner_is_p1, opponents=opponents, aggression=aggression,
              scenarios=scenarios, learners=np.full(n, -1))
    env.reset_all(seed, 0)
    rng = np.random.default_rng(pick_seed)
    rows, actions = [], []
    for step in range(1, steps + 1):
        out = env.read()
        masks = out["learner_masks"]
        act = np.zeros(n, np.int64)
        for e in range(n):
            legal = np.nonzero(masks[e])[0]
            act[e] = legal[rng.integers(len(legal))] if len(legal) else 0
        actions.append(act)
        pre = [digest(out["learner_obs"]), digest(out["opponent_obs"]), digest(masks), digest(out["opponent_masks"])]
        env.step(act, None, seed, step)
        post = env.read()
        rows.append(pre + [digest(post["rewards"]), digest(post["terminated"]), digest(post["outcomes"]),
                           digest(post["states"])])
        env.reset_done(seed, step)
    return np.frombuffer(b"".join(b"".join(r) for r in rows), np.uint8).reshape(steps, 8, 8), np.stack(actions)


def env_case(n: int):
    idx = np.arange(n)
    learner_is_p1 = (idx % 2 == 0).astype(np.uint8)
    opponents = (idx * 7) % 41
    learners = (idx * 11 + 3) % 41
    p1 = np.where(learner_is_p1 == 1, learners, opponents)
    p2 = np.where(learner_is_p1 == 1, opponents, learners)
    # both opponent kinds: the random opponent (aggression in [0, 1]) and tiered bots (-(id + 1))
    aggression = np.where(idx % 3 == 0, -((idx * 13) % 331 + 1), (idx % 5) / 4.0).astype(np.float32)
    scenarios = idx % 9
    return p1, p2, learner_is_p1, opponents, aggression, scenarios


def main():
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "roster.bin"
        ref.export_roster(GENERATED, str(path))
        raw = path.read_bytes()
    (HERE / "roster41.bin.xz").write_bytes(lzma.compress(raw, preset=9))
    print("roster", len(raw), "bytes")

    roster = ref.RefRoster(raw)
    rng = np.random.default_rng(0)
    fights = 16
    p1 = rng.integers(0, 41, fights).astype(np.int32)
    p2 = rng.integers(0, 41, fights).astype(np.int32)
    start = np.where(np.arange(fights) % 2 == 1, 2.4, -0.6 + 0.1 * (np.arange(fights) % 5))
    x1, x2 = start, start + 0.9
    frames = 600
    hashes, _, _ = roster.random_play(p1, p2, x1, x2, frames, 0)
    np.savez_compressed(HERE / "engine_trace.npz", p1=p1, p2=p2, x1=x1, x2=x2, frames=frames, seed=0, hashes=hashes)
    print("engine trace", hashes.shape)

    sys.path.insert(0, str(ROOT / "tekken8-agent_b200"))
    from t8b._lib import EnvConfig  # layout only; no library load

    n, steps = 48, 60
    config = EnvConfig()
    config.max_round_frames = 900
    config.hold_frames = 8
    config.max_frames_per_decision = 120
    config.damage_reward = 1.0
    config.win_reward = 1.0
    config.draw_penalty = 0.5
    config.throw_break_penalty = 0.03
    config.time_penalty_per_second = 0.01
    config.damage_dealt_weight = 1.0
    config.damage_taken_weight = 1.0
    config.perception_delay = 12
    config.live_noise = 1
    config.screen_view = 1
    config.noise_position_max = 0.25
    config.noise_flip_max = 0.10
    config.latency_min = 2
    config.latency_max = 6
    config.start_center_range = 1.2
    config.start_distance_min = 0.8
    config.start_distance_max = 2.4
    case = env_case(n)
    digests, actions = env_run(raw, n, steps, config, 99, case[3], case[4], case[5], case[2], case[0], case[1], 7)
    np.savez_compressed(HERE / "env_trace.npz", digests=digests, actions=actions, n=n, steps=steps, seed=99,
                        config=np.frombuffer(bytes(config), np.uint8), p1=case[0], p2=case[1],
                        learner_is_p1=case[2], opponents=case[3], aggression=case[4], scenarios=case[5])
    print("env trace", digests.shape)


if __name__ == "__main__":
    main()
