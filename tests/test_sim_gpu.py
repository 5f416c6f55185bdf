"""GPU simulator parity against the reference (tests/full_move_gpu_tests.cpp in spirit):
engine traces bit for bit, the engine-level API replaying recorded inputs, and the
environment contract (observations with screen view and live noise, masks, rewards,
terminations, resets, scripted opponents) step for step against the reference CPU
contract in oracle/_ref and against the golden fixtures."""
import sys

import numpy as np
import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
import make_golden  # noqa: E402

pytestmark = pytest.mark.gpu


def first_mismatch(a, b):
    bad = np.argwhere(a != b)
    return None if bad.size == 0 else tuple(int(v) for v in bad[0])


def test_random_play_matches_golden(cuda, roster):
    from t8b.sim import GpuFullMoveSimulator
    g = np.load(GOLDEN / "engine_trace.npz")
    sim = GpuFullMoveSimulator(roster, 1)
    hashes = sim.random_play(g["p1"], g["p2"], g["x1"], g["x2"], int(g["frames"]), int(g["seed"]))
    got = hashes.cpu().numpy().view(np.uint64)
    assert first_mismatch(got, g["hashes"]) is None


def test_random_play_config1_matches_reference(cuda, roster, ref_roster):
    """The engine-parity workload: 1,024 fights over uniform pairs of the 41 fighters, 3,600 frames,
    PCG32 seed 0 per fight index; per-frame state hashes equal the reference CPU engine's."""
    from t8b.sim import GpuFullMoveSimulator
    rng = np.random.default_rng(0)
    fights, frames = 1024, 3600
    p1 = rng.integers(0, 41, fights).astype(np.int32)
    p2 = rng.integers(0, 41, fights).astype(np.int32)
    start = rng.uniform(-1.2, 1.2, fights)
    x1, x2 = start - 0.45, start + 0.45
    sim = GpuFullMoveSimulator(roster, 1)
    got = sim.random_play(p1, p2, x1, x2, frames, 0).cpu().numpy().view(np.uint64)
    want, _, _ = ref_roster.random_play(p1, p2, x1, x2, frames, 0, threads=16)
    assert first_mismatch(got, want) is None


def test_engine_level_replay(cuda, roster, ref_roster):
    """Recorded inputs replayed through reset_engine/step_engine match state and events every frame."""
    from t8b.sim import GpuFullMoveSimulator
    rng = np.random.default_rng(5)
    fights, frames = 48, 500
    p1 = rng.integers(0, 41, fights).astype(np.int32)
    p2 = rng.integers(0, 41, fights).astype(np.int32)
    start = np.where(np.arange(fights) % 2 == 1, 2.4, -0.6 + 0.1 * (np.arange(fights) % 5))
    x1, x2 = start, start + 0.9
    _, states, inputs = ref_roster.random_play(p1, p2, x1, x2, frames, 11, states=True, inputs=True)
    sim = GpuFullMoveSimulator(roster, fights)
    sim.set_matchups(p1, p2)
    sim.reset_engine(x1, x2)
    ref_state = np.stack([ref_roster.reset_state(int(a), int(b), float(c), float(d)) for a, b, c, d in zip(p1, p2, x1, x2)])
    assert np.array_equal(sim.download_state_bytes(), ref_state)
    winner_prev = np.full(fights, -1)
    for frame in range(frames):
        new_round = (winner_prev >= 0).astype(np.uint8)
        sim.step_engine(inputs[:, frame], new_round, x1, x2)
        got = sim.download_state_bytes()
        assert first_mismatch(got, states[:, frame]) is None, f"frame {frame}"
        winner_prev = states[:, frame].view(np.int32)[:, 59]
    # events of the last frame against a reference step from the same states
    sim2 = GpuFullMoveSimulator(roster, fights)
    sim2.set_matchups(p1, p2)
    before = np.ascontiguousarray(states[:, frames - 2])
    from t8b._lib import State
    sim2.upload_states((State * fights).from_buffer_copy(before.tobytes()))
    sim2.step_engine(inputs[:, frames - 1])
    ref_states = before.copy()
    ref_events = ref_roster.engine_step(p1, p2, ref_states, inputs[:, frames - 1])
    assert np.array_equal(sim2.download_state_bytes(), ref_states)
    got_events = np.frombuffer(bytes(sim2.download_events()), np.uint8).reshape(fights, 208)
    assert np.array_equal(got_events, ref_events)


def env_config(**kw):
    from t8b.sim import env_config as make
    base = dict(max_round_frames=900, hold_frames=8, draw_penalty=0.5, throw_break_penalty=0.03,
                time_penalty_per_second=0.01, perception_delay=12, live_noise=1, screen_view=1)
    base.update(kw)
    return make(**base)


def gpu_read(sim):
    return {
        "learner_obs": sim.learner_observations().cpu().numpy(),
        "opponent_obs": sim.opponent_observations().cpu().numpy(),
        "learner_masks": sim.learner_masks().cpu().numpy(),
        "opponent_masks": sim.opponent_masks().cpu().numpy(),
        "rewards": sim.rewards().cpu().numpy(),
        "terminated": sim.terminated().cpu().numpy(),
        "outcomes": sim.outcomes().cpu().numpy(),
        "states": sim.download_state_bytes(),
    }


def test_env_matches_golden_digests(cuda, roster):
    import torch
    from t8b._lib import EnvConfig
    from t8b.sim import GpuFullMoveSimulator
    g = np.load(GOLDEN / "env_trace.npz")
    n, steps, seed = int(g["n"]), int(g["steps"]), int(g["seed"])
    config = EnvConfig.from_buffer_copy(g["config"].tobytes())
    sim = GpuFullMoveSimulator(roster, n, config)
    sim.set_matchups(g["p1"], g["p2"])
    sim.set_learner_sides(g["learner_is_p1"])
    sim.set_pending_opponents(g["opponents"], g["aggression"], g["scenarios"])
    sim.reset_all(seed, 0)
    rng = np.random.default_rng(7)
    d = make_golden.digest
    for step in range(1, steps + 1):
        out = gpu_read(sim)
        act = np.zeros(n, np.int64)
        for e in range(n):
            legal = np.nonzero(out["learner_masks"][e])[0]
            act[e] = legal[rng.integers(len(legal))] if len(legal) else 0
        assert np.array_equal(act, g["actions"][step - 1]), f"step {step}"
        pre = [d(out["learner_obs"]), d(out["opponent_obs"]), d(out["learner_masks"]), d(out["opponent_masks"])]
        sim.step(torch.as_tensor(act, device="cuda"), None, seed, step)
        post = gpu_read(sim)
        row = pre + [d(post["rewards"]), d(post["terminated"]), d(post["outcomes"]), d(post["states"])]
        got = np.frombuffer(b"".join(row), np.uint8).reshape(8, 8)
        assert np.array_equal(got, g["digests"][step - 1]), f"step {step}"
        sim.reset_done(seed, step)


@pytest.mark.parametrize("noise,screen,self_play,memory", [(1, 1, False, 0), (0, 0, False, 0), (1, 0, True, 0),
                                                             (1, 0, False, 1), (0, 0, True, 1)])
def test_env_matches_reference_contract(cuda, roster, ref_roster, noise, screen, self_play, memory):
    """Step for step against the reference contract on the host, all outputs compared (with
    --memory the observation carries each fighter's move history and habit traces)."""
    import torch
    from oracle import ref
    from t8b.sim import GpuFullMoveSimulator
    n, steps, seed = 256, 150, 31
    config = env_config(live_noise=noise, screen_view=screen, perception_delay=12 if noise else 0, memory=memory,
                        damage_dealt_weight=0.8, damage_taken_weight=1.2, distance_penalty_per_second=0.002)
    p1, p2, sides, opponents, aggression, scenarios = make_golden.env_case(n)
    sim = GpuFullMoveSimulator(roster, n, config)
    sim.set_matchups(p1, p2)
    sim.set_learner_sides(sides)
    sim.set_pending_opponents(opponents, aggression, scenarios)
    cpu = ref.RefEnv(ref_roster, n, config, threads=16)
    cpu.setup(p1=p1, p2=p2, learner_is_p1=sides, opponents=opponents, aggression=aggression, scenarios=scenarios,
              learners=np.full(n, -1))
    sim.reset_all(seed, 0)
    cpu.reset_all(seed, 0)
    assert sim.observation_size() == cpu.width == 148 + 90 * memory + 3 * noise
    rng = np.random.default_rng(3)
    terminations = 0
    for step in range(1, steps + 1):
        a, b = gpu_read(sim), cpu.read()
        for key in ("learner_obs", "opponent_obs", "learner_masks", "opponent_masks", "states"):
            assert np.array_equal(a[key].view(np.uint8), b[key].view(np.uint8)), (key, step, first_mismatch(a[key], b[key]))
        if noise:
            got = np.frombuffer(bytes(sim.download_noise_levels()), np.uint8).reshape(n, 16)
            assert np.array_equal(got, b["noise"]), step
        assert np.array_equal(sim.learner_feature_tables().cpu().numpy(), np.where(sides == 1, b["p1"], b["p2"]))
        act = np.array([np.nonzero(m)[0][rng.integers(m.sum())] for m in a["learner_masks"]], np.int64)
        opp = None
        if self_play:
            opp = np.array([np.nonzero(m)[0][rng.integers(m.sum())] for m in a["opponent_masks"]], np.int64)
        sim.step(torch.as_tensor(act, device="cuda"), None if opp is None else torch.as_tensor(opp, device="cuda"),
                 seed, step)
        cpu.step(act, opp, seed, step)
        a, b = gpu_read(sim), cpu.read()
        for key in ("rewards", "terminated", "outcomes", "states", "learner_obs", "learner_masks"):
            assert np.array_equal(a[key].view(np.uint8), b[key].view(np.uint8)), (key, step, first_mismatch(a[key], b[key]))
        terminations += int(a["terminated"].sum())
        sim.reset_done(seed, step)
        cpu.reset_done(seed, step)
    assert terminations > 20
    assert sim.frames_simulated() == cpu.read()["frames"]


@pytest.mark.parametrize("noise,screen,self_play,memory", [(1, 1, False, 0), (1, 0, True, 1)])
def test_step_and_reset_equals_step_then_reset_done(cuda, roster, ref_roster, noise, screen, self_play, memory):
    """t8b_sim_step_and_reset against t8b_sim_step + t8b_sim_reset_done on a second simulator and
    against the reference contract's step + reset_done: after every call the states, matchups,
    noise levels, rewards, terminations, outcomes, both sides' observations and masks, and at
    the end the tallies and frame counts are identical. Short rounds and pending learners make
    the in-step reset run on many fights."""
    import torch
    from oracle import ref
    from t8b.sim import GpuFullMoveSimulator
    n, steps, seed = 256, 120, 17
    config = env_config(live_noise=noise, screen_view=screen, perception_delay=12 if noise else 0, memory=memory,
                        max_round_frames=300)
    p1, p2, sides, opponents, aggression, scenarios = make_golden.env_case(n)
    learners = np.where(np.arange(n) % 3 == 0, (np.arange(n) * 7) % 41, -1).astype(np.int32)
    sims = []
    for _ in range(2):
        sim = GpuFullMoveSimulator(roster, n, config)
        sim.set_matchups(p1, p2)
        sim.set_learner_sides(sides)
        sim.set_pending_opponents(opponents, aggression, scenarios)
        sim.set_pending_learners(learners)
        sim.reset_all(seed, 0)
        sims.append(sim)
    fused, split = sims
    cpu = ref.RefEnv(ref_roster, n, config, threads=16)
    cpu.setup(p1=p1, p2=p2, learner_is_p1=sides, opponents=opponents, aggression=aggression, scenarios=scenarios,
              learners=learners)
    cpu.reset_all(seed, 0)
    rng = np.random.default_rng(8)
    terminations = 0
    for step in range(1, steps + 1):
        a = gpu_read(fused)
        act = np.array([np.nonzero(m)[0][rng.integers(m.sum())] for m in a["learner_masks"]], np.int64)
        opp = None
        if self_play:
            opp = np.array([np.nonzero(m)[0][rng.integers(m.sum())] for m in a["opponent_masks"]], np.int64)
        la = torch.as_tensor(act, device="cuda")
        oa = None if opp is None else torch.as_tensor(opp, device="cuda")
        fused.step_and_reset(la, oa, seed, step)
        split.step(la, oa, seed, step)
        split.reset_done(seed, step)
        cpu.step(act, opp, seed, step)
        cpu.reset_done(seed, step)
        a, b, c = gpu_read(fused), gpu_read(split), cpu.read()
        for key in ("rewards", "terminated", "outcomes", "states", "learner_obs", "opponent_obs", "learner_masks",
                    "opponent_masks"):
            assert np.array_equal(a[key].view(np.uint8), b[key].view(np.uint8)), (key, step, first_mismatch(a[key], b[key]))
            assert np.array_equal(a[key].view(np.uint8), c[key].view(np.uint8)), (key, step, first_mismatch(a[key], c[key]))
        if noise:
            assert bytes(fused.download_noise_levels()) == bytes(split.download_noise_levels())
        assert np.array_equal(fused.learner_feature_tables().cpu().numpy(), split.learner_feature_tables().cpu().numpy())
        terminations += int(a["terminated"].sum())
    assert terminations > 100
    assert fused.frames_simulated() == split.frames_simulated() == cpu.read()["frames"]
    for x, y in zip(fused.download_and_clear_tally(), split.download_and_clear_tally()):
        assert np.array_equal(x, y)


def test_engine_legal_mask_and_tallies(cuda, roster, ref_roster):
    import torch
    from t8b.sim import GpuFullMoveSimulator
    n = 64
    p1, p2, sides, opponents, aggression, scenarios = make_golden.env_case(n)
    sim = GpuFullMoveSimulator(roster, n, env_config(max_round_frames=300))
    sim.set_matchups(p1, p2)
    sim.set_learner_sides(sides)
    sim.set_pending_opponents(opponents, aggression, scenarios)
    sim.reset_all(5, 0)
    finished = 0
    for step in range(1, 40):
        masks = sim.learner_masks().cpu().numpy()
        act = torch.as_tensor(np.argmax(masks[:, ::-1] > 0, axis=1).astype(np.int64) * 0, device="cuda")
        sim.step(act, None, 5, step)
        finished += int(sim.terminated().cpu().numpy().sum())
        sim.reset_done(5, step)
    tally, scenario, learner, bot = sim.download_and_clear_tally()
    assert tally.sum() == finished == scenario.sum() == learner.sum()
    again = sim.download_and_clear_tally()
    assert all(t.sum() == 0 for t in again)
    for player in (0, 1):
        got = sim.download_legal_mask(player)
        states = sim.download_state_bytes()
        chars = p1 if player == 0 else p2
        for e in range(0, n, 7):
            count = roster.characters[chars[e]].candidate_count
            assert got[e, count:].sum() == 0


def test_snapshot_restore_round_trip(cuda, roster):
    import torch
    from t8b.sim import GpuFullMoveSimulator
    import ctypes as C
    from t8b._lib import State
    n = 32
    p1, p2, sides, opponents, aggression, scenarios = make_golden.env_case(n)
    sim = GpuFullMoveSimulator(roster, n, env_config())
    sim.set_matchups(p1, p2)
    sim.set_learner_sides(sides)
    sim.set_pending_opponents(opponents, aggression, scenarios)
    sim.reset_all(9, 0)
    for step in range(1, 6):
        sim.step(torch.zeros(n, dtype=torch.int64, device="cuda"), None, 9, step)
        sim.reset_done(9, step)
    arrays = [(State * n)(), np.zeros(n, np.int32), np.zeros(n, np.int32), np.zeros(n, np.uint8),
              np.zeros(n, np.float32), np.zeros(n, np.int32), np.zeros(n, np.float32), np.zeros(n, np.uint8),
              np.zeros(n, np.int32), np.zeros(n, np.int32), np.zeros(n, np.int32)]
    ptrs = [arrays[0]] + [a.ctypes.data_as(C.c_void_p) for a in arrays[1:]]
    from t8b._lib import call
    call("t8b_sim_snapshot", sim.handle, *ptrs)
    other = GpuFullMoveSimulator(roster, n, env_config())
    call("t8b_sim_restore", other.handle, *ptrs)
    assert np.array_equal(other.download_state_bytes(), sim.download_state_bytes())
    # observations are recomputed from the restored state (noise levels are redrawn, as the reference)
    assert other.learner_observations().shape == (n, 151)
    assert np.array_equal(other.learner_masks().cpu().numpy(), sim.learner_masks().cpu().numpy())


def test_self_play_iteration_with_a_checkpoint_opponent(cuda, roster, tmp_path):
    """Mirror self-play: a frozen policy loaded from a .t8ppo file plays the other side from the
    opponent observations on its own stream; an iteration runs and is reproducible."""
    import torch
    from t8b.policy import GpuActorCritic, actor_config
    from t8b.train import SelfPlayTrainer
    frozen = GpuActorCritic(1024, actor_config(), 41)
    frozen.save_checkpoint(tmp_path / "frozen.t8ppo")
    results = []
    for _ in range(2):
        trainer = SelfPlayTrainer(roster, environments=1024, horizon=8, epochs=1, minibatches=2, seed=5,
                                  opponent=tmp_path / "frozen.t8ppo")
        metrics = trainer.iterate()
        torch.cuda.synchronize()
        assert all(np.isfinite(v) for v in metrics.values())
        results.append((trainer.policy.parameters(), trainer.sim.download_state_bytes()))
    assert np.array_equal(results[0][0], results[1][0])
    assert np.array_equal(results[0][1], results[1][1])


@pytest.mark.parametrize("self_play, envs", [(False, 1024), (True, 1024), (False, 8192)])
def test_native_rollout_loop_equals_the_python_loop(cuda, roster, tmp_path, self_play, envs):
    """t8b_collect_rollout issues the same calls as the trainer's Python loop: one iteration
    from the same seeds gives bit-identical weights, simulator states and advantages. At 8,192
    fights against scripted opponents the native loop also runs with the two halves of the
    fights on two streams (T8B_ROLLOUT_GROUPS=2), which must not change a bit."""
    import os
    import torch
    from t8b.policy import GpuActorCritic, actor_config
    from t8b.train import SelfPlayTrainer
    opponent = None
    if self_play:
        GpuActorCritic(1024, actor_config(), 8).save_checkpoint(tmp_path / "frozen.t8ppo")
        opponent = tmp_path / "frozen.t8ppo"
    results = []
    grouped = envs >= 8192 and not self_play
    for native in (True, False):
        trainer = SelfPlayTrainer(roster, environments=envs, horizon=8, epochs=1, minibatches=2, seed=11,
                                  opponent=opponent)
        if native and grouped:
            os.environ["T8B_ROLLOUT_GROUPS"] = "2"
        try:
            trainer.iterate(native=native)
        finally:
            os.environ.pop("T8B_ROLLOUT_GROUPS", None)
        torch.cuda.synchronize()
        results.append((trainer.policy.parameters(), trainer.sim.download_state_bytes(),
                        trainer.rollout.tensor("advantages").cpu().numpy().copy()))
    for a, b in zip(*results):
        assert np.array_equal(a, b)
