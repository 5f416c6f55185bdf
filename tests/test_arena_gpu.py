"""Evaluation (src/full_move_train.cpp:921-1044): the device-side first-outcome recording of
t8b/arena.py against the reference's own bookkeeping (terminated flags and outcomes downloaded
after every step) on the same schedule, seeds and policies."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def host_tracked(sim, step_fn, max_steps, seed):
    """The reference's loop: download terminated and outcomes after every step."""
    n = sim.environment_count()
    finished = np.zeros(n, bool)
    result = np.zeros(n, np.int8)
    for step in range(1, max_steps + 1):
        step_fn(step)
        terminated = sim.terminated().cpu().numpy().astype(bool)
        outcomes = sim.outcomes().cpu().numpy()
        new = terminated & ~finished
        result[new] = outcomes[new]
        finished |= new
        sim.reset_done(seed, step)
        if finished.all():
            break
    return finished, result


def test_evaluate_matches_per_step_host_bookkeeping(cuda, roster):
    import torch
    from t8b.arena import evaluate
    from t8b.policy import GpuActorCritic, actor_config
    from t8b.sim import GpuFullMoveSimulator
    from t8b.train import config4_env
    n, seed = 1024, 9
    learners, opponents = list(range(0, 41, 3)), list(range(41))
    policy = GpuActorCritic(n, actor_config(), 5)
    policy.set_action_feature_tables(roster.feature_tables())
    sim = GpuFullMoveSimulator(roster, n, config4_env())
    got = evaluate(policy, sim, learners, opponents, True, seed, max_steps=3000)
    # the same schedule with the reference's per-step downloads
    sim2 = GpuFullMoveSimulator(roster, n, config4_env())
    pair = np.arange(n) // 2
    ln = np.asarray(learners, np.int32)[pair % len(learners)]
    op = np.asarray(opponents, np.int32)[(pair // len(learners) + pair) % len(opponents)]
    ag = ((pair // len(opponents)) % 5).astype(np.float32) / 4.0
    sides = (np.arange(n) % 2 == 0).astype(np.uint8)
    sim2.set_matchups(np.where(sides == 1, ln, op), np.where(sides == 1, op, ln))
    sim2.set_learner_sides(sides)
    sim2.set_pending_opponents(op, ag)
    sim2.set_pending_learners(ln)
    sim2.reset_all(seed, 0)

    def step(s):
        out = policy.forward(sim2.learner_observations(), sim2.learner_masks(), n, seed + 17, s, True, None,
                             sim2.learner_feature_tables())
        sim2.step(out["actions"], None, seed, s)

    finished, result = host_tracked(sim2, step, 3000, seed)
    assert got.episodes == int(finished.sum()) > 0
    assert abs(got.win_rate - float((result[finished] > 0).mean())) < 1e-12
    assert abs(got.draw_rate - float((result[finished] == 0).mean())) < 1e-12
    for character, row in got.characters.items():
        mask = finished & (op == character)
        assert row[3] == int(mask.sum())
        assert row[0] == int((result[mask] > 0).sum()) and row[1] == int((result[mask] < 0).sum())
    torch.cuda.synchronize()


def test_head_to_head_matches_per_step_host_bookkeeping(cuda, roster):
    from t8b.arena import head_to_head
    from t8b.policy import GpuActorCritic, actor_config
    from t8b.sim import GpuFullMoveSimulator
    from t8b.train import config4_env
    n, seed = 1024, 4
    learners = list(range(0, 41, 5))
    a = GpuActorCritic(n, actor_config(), 1)
    b = GpuActorCritic(n, actor_config(), 2)
    for p in (a, b):
        p.set_action_feature_tables(roster.feature_tables())
    got = head_to_head(a, b, GpuFullMoveSimulator(roster, n, config4_env()), learners, seed, True, max_steps=3000)
    sim2 = GpuFullMoveSimulator(roster, n, config4_env())
    pair = np.arange(n) // 2
    k = len(learners)
    own = np.asarray(learners, np.int32)[pair % k]
    other = np.asarray(learners, np.int32)[(pair // k + pair) % k]
    sides = (np.arange(n) % 2 == 0).astype(np.uint8)
    sim2.set_matchups(np.where(sides == 1, own, other), np.where(sides == 1, other, own))
    sim2.set_learner_sides(sides)
    sim2.set_pending_opponents(other)
    sim2.set_pending_learners(own)
    sim2.reset_all(seed, 0)

    def step(s):
        mine = a.forward(sim2.learner_observations(), sim2.learner_masks(), n, seed, s, True, None,
                         sim2.learner_feature_tables())
        theirs = b.forward(sim2.opponent_observations(), sim2.opponent_masks(), n, seed + 1, s, True, None,
                           sim2.opponent_feature_tables())
        sim2.step(mine["actions"], theirs["actions"], seed, s)

    finished, result = host_tracked(sim2, step, 3000, seed)
    r = result[finished]
    assert got == [int((r > 0).sum()), int((r < 0).sum()), int((r == 0).sum())]
    assert sum(got) == int(finished.sum()) > 0
