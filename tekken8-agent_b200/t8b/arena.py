"""Evaluation of a policy: the reference trainer's `evaluate` (against the scripted opponents)
and `head_to_head` (against a frozen policy), src/full_move_train.cpp:921-1044, with the same
pairings, sides, aggression styles, seeds and step limits. Where the reference downloads the
terminated flags and outcomes after every step, the first finished round of each fight is
recorded on the device (t8b_sim_record_first_outcomes) and the host reads one counter every
`check_every` steps."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import call


@dataclass
class Evaluation:
    episodes: int = 0
    win_rate: float = 0.0
    p1_win_rate: float = 0.0
    p2_win_rate: float = 0.0
    draw_rate: float = 0.0
    worst_character_win_rate: float = 1.0
    worst_character: int = -1
    characters: dict = field(default_factory=dict)  # opponent character -> [wins, losses, draws, episodes]
    learners: dict = field(default_factory=dict)    # learner character -> [wins, losses, draws, episodes]
    styles: list = field(default_factory=lambda: [[0, 0, 0, 0] for _ in range(5)])  # per aggression bucket


class FirstOutcomes:
    """Device buffers for the first finished round of every fight."""

    def __init__(self, sim):
        n = sim.environment_count()
        self.sim = sim
        self.result = torch.zeros(n, dtype=torch.int8, device="cuda")
        self.finished = torch.zeros(n, dtype=torch.uint8, device="cuda")
        self.remaining = torch.full((1,), n, dtype=torch.int32, device="cuda")

    def record(self):
        call("t8b_sim_record_first_outcomes", self.sim.handle, C.c_void_p(self.result.data_ptr()),
             C.c_void_p(self.finished.data_ptr()), C.c_void_p(self.remaining.data_ptr()))

    def left(self) -> int:
        return int(self.remaining.item())


def _schedule(sim, p1, p2, sides, opponents, learners, aggression=None):
    sim.set_matchups(p1, p2)
    sim.set_learner_sides(sides)
    sim.set_pending_opponents(opponents, aggression)
    sim.set_pending_learners(learners)


def evaluate(policy, sim, learner_roster, opponent_roster, deterministic: bool, seed: int, max_steps: int = 20000,
             check_every: int = 64) -> Evaluation:
    """One round per fight against the scripted opponents: learners and opponents over every
    pairing in turn, five aggression styles, half the fights on each side
    (src/full_move_train.cpp:921-1000)."""
    n = sim.environment_count()
    pair = np.arange(n) // 2
    learners = np.asarray(learner_roster, np.int32)[pair % len(learner_roster)]
    opponents = np.asarray(opponent_roster, np.int32)[(pair // len(learner_roster) + pair) % len(opponent_roster)]
    aggression = ((pair // len(opponent_roster)) % 5).astype(np.float32) / 4.0
    sides = (np.arange(n) % 2 == 0).astype(np.uint8)
    p1 = np.where(sides == 1, learners, opponents).astype(np.int32)
    p2 = np.where(sides == 1, opponents, learners).astype(np.int32)
    _schedule(sim, p1, p2, sides, opponents, learners, aggression)
    sim.reset_all(seed, 0)
    first = FirstOutcomes(sim)
    for step in range(1, max_steps + 1):
        out = policy.forward(sim.learner_observations(), None, n, seed + 17, step, deterministic, None,
                             sim.learner_feature_tables(), mask_bits=sim.learner_mask_bits())
        sim.step(out["actions"], None, seed, step)
        first.record()
        # finished fights keep playing new rounds; only their first counts
        sim.reset_done(seed, step)
        if step % check_every == 0 and first.left() == 0:
            break
    finished = first.finished.cpu().numpy().astype(bool)
    result = first.result.cpu().numpy()
    e = Evaluation()
    side_wins, side_episodes, wins, draws = [0, 0], [0, 0], 0, 0
    for env in np.nonzero(finished)[0]:
        e.episodes += 1
        side = 0 if sides[env] else 1
        side_episodes[side] += 1
        column = 0 if result[env] > 0 else (1 if result[env] < 0 else 2)
        for table, key in ((e.characters, int(opponents[env])), (e.learners, int(learners[env]))):
            row = table.setdefault(key, [0, 0, 0, 0])
            row[column] += 1
            row[3] += 1
        style = e.styles[int(round(float(aggression[env]) * 4.0))]
        style[column] += 1
        style[3] += 1
        wins += result[env] > 0
        draws += result[env] == 0
        side_wins[side] += result[env] > 0
    rate = lambda part, whole: 0.0 if whole == 0 else part / whole
    e.win_rate = rate(wins, e.episodes)
    e.draw_rate = rate(draws, e.episodes)
    e.p1_win_rate = rate(side_wins[0], side_episodes[0])
    e.p2_win_rate = rate(side_wins[1], side_episodes[1])
    for key, row in sorted(e.characters.items()):
        r = rate(row[0], row[3])
        if r <= e.worst_character_win_rate:
            e.worst_character_win_rate = r
            e.worst_character = key
    return e


def head_to_head(learner, opponent, sim, learner_roster, seed: int, deterministic: bool = True,
                 max_steps: int = 40000, check_every: int = 64) -> list[int]:
    """The learner against a frozen policy, both on learner characters (every pairing in turn),
    one round per fight, half on each side: [wins, losses, draws]
    (src/full_move_train.cpp:1004-1044)."""
    n = sim.environment_count()
    pair = np.arange(n) // 2
    k = len(learner_roster)
    roster = np.asarray(learner_roster, np.int32)
    own = roster[pair % k]
    other = roster[(pair // k + pair) % k]
    sides = (np.arange(n) % 2 == 0).astype(np.uint8)
    p1 = np.where(sides == 1, own, other).astype(np.int32)
    p2 = np.where(sides == 1, other, own).astype(np.int32)
    _schedule(sim, p1, p2, sides, other, own)
    sim.reset_all(seed, 0)
    first = FirstOutcomes(sim)
    for step in range(1, max_steps + 1):
        mine = learner.forward(sim.learner_observations(), None, n, seed, step, deterministic, None,
                               sim.learner_feature_tables(), mask_bits=sim.learner_mask_bits())
        theirs = opponent.forward(sim.opponent_observations(), None, n, seed + 1, step, deterministic, None,
                                  sim.opponent_feature_tables(), mask_bits=sim.opponent_mask_bits())
        sim.step(mine["actions"], theirs["actions"], seed, step)
        first.record()
        sim.reset_done(seed, step)
        if step % check_every == 0 and first.left() == 0:
            break
    finished = first.finished.cpu().numpy().astype(bool)
    result = first.result.cpu().numpy()[finished]
    return [int((result > 0).sum()), int((result < 0).sum()), int((result == 0).sum())]
