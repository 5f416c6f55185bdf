"""One self-play training iteration, as the reference trainer's hot loop runs it
(src/full_move_train.cpp:1374-1414): a rollout of `horizon` decisions over every fight
(policy forward -> record -> simulator step -> reset of finished rounds), return
normalisation, GAE, then the PPO update.

Two changes of schedule, neither of which changes what is learned:
  * the critic's bootstrap value of a decision's successor state is the value the next
    decision's forward pass computes anyway (the reference runs a second, deterministic forward
    per step for it). For a fight whose round ended the successor value is the reset state's,
    which GAE multiplies by zero (terminated and not truncated; the simulator never truncates),
    so advantages and returns are identical; one forward per decision remains, plus one at the
    end of the rollout for the last bootstrap;
  * masks stay packed (12 words per fight) from the simulator through the rollout to the
    update, and the update's permutations are drawn on a host thread while the rollout runs.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from .policy import GpuActorCritic, GpuRolloutBuffer, actor_config, ppo_config
from ._lib import call
from .sim import GpuFullMoveSimulator, env_config


def config4_env(**overrides):
    """The measured self-play configuration (training.ini): screen-only observation with live noise (sigma 0.28 m,
    detection errors 10 %, latency 2-6 frames), perception delay 12, 8-frame holds, and the
    trainer's anti-stalling terms (src/train_launcher.cpp:106-160)."""
    base = dict(screen_view=1, live_noise=1, noise_position_max=0.28, noise_flip_max=0.10, latency_min=2,
                latency_max=6, perception_delay=12, hold_frames=8, draw_penalty=0.5, throw_break_penalty=0.03,
                time_penalty_per_second=0.01, max_round_frames=3600)
    base.update(overrides)
    return env_config(**base)


class SelfPlayTrainer:
    """With `opponent` (a checkpoint path, or a GpuActorCritic) the fights are mirror self-play:
    the frozen policy plays the other side from the opponent observations, masks and feature
    tables (src/full_move_train.cpp:1333-1358, 1382-1387), on a second stream that overlaps the
    learner's forward; otherwise scripted opponents play."""

    def __init__(self, roster, environments=32768, horizon=128, epochs=4, minibatches=8, seed=3, hidden=512,
                 layers=2, env=None, comm=None, rank=0, target_kl=0.0, scenario_share=0.25, opponent=None):
        self.roster = roster
        self.n = environments
        self.horizon = horizon
        self.epochs = epochs
        self.seed = seed + rank
        self.rank = rank
        self.samples = environments * horizon
        self.minibatch = self.samples // minibatches
        self.sim = GpuFullMoveSimulator(roster, environments, env if env is not None else config4_env())
        self.actor = actor_config(observation_size=self.sim.observation_size(), hidden_size=hidden,
                                  shared_layers=layers)
        self.policy = GpuActorCritic(max(environments, self.minibatch), self.actor, seed)  # identical init on every rank
        self.policy.set_action_feature_tables(roster.feature_tables())
        self.rollout = GpuRolloutBuffer(environments, horizon, self.actor)
        if comm is not None:
            self.policy.set_comm(comm)
            self.rollout.set_comm(comm)
        self.ppo = ppo_config(epochs=epochs, minibatch_size=self.minibatch, learning_rate=5e-4, target_kl=target_kl,
                              entropy_coefficient=0.01)
        self.opponent = None
        if opponent is not None:
            if isinstance(opponent, GpuActorCritic):
                self.opponent = opponent
            else:
                self.opponent = GpuActorCritic(environments, self.actor, seed + 1)
                self.opponent.load_checkpoint(opponent, load_optimizer_state=False)
            self.opponent.set_action_feature_tables(roster.feature_tables())
            self.opponent_stream = torch.cuda.Stream()
        rng = np.random.default_rng(self.seed)
        count = len(roster)
        self.sides = (np.arange(environments) % 2 == 0).astype(np.uint8)
        self.learners = rng.integers(0, count, environments).astype(np.int32)
        self.scenario_share = scenario_share
        self.rng = rng
        opponents, aggression, scenarios = self.schedule()
        p1 = np.where(self.sides == 1, self.learners, opponents).astype(np.int32)
        p2 = np.where(self.sides == 1, opponents, self.learners).astype(np.int32)
        self.sim.set_matchups(p1, p2)
        self.sim.set_learner_sides(self.sides)
        self.sim.set_pending_opponents(opponents, aggression, scenarios)
        self.sim.set_pending_learners(self.learners)
        self.sim.reset_all(self.seed, 0)
        self.update_index = 0
        self.stream = None

    def schedule(self):
        """Uniform opponents over the roster, scripted aggression in [0, 1], a share of scenario
        starts (src/full_move_train.cpp schedule_opponents)."""
        rng = self.rng
        opponents = rng.integers(0, len(self.roster), self.n).astype(np.int32)
        if self.opponent is not None:
            # self-play rounds start neutral, at the fixed aggression the reference gives them
            return opponents, np.full(self.n, 0.5, np.float32), np.zeros(self.n, np.int32)
        aggression = rng.random(self.n).astype(np.float32)
        scenarios = np.where(rng.random(self.n) < self.scenario_share, rng.integers(1, 9, self.n), 0).astype(np.int32)
        return opponents, aggression, scenarios

    def upload_schedule(self):
        """Host -> device: the next rounds' opponents, aggression, scenarios and learners."""
        opponents, aggression, scenarios = self.schedule()
        self.sim.set_pending_opponents(opponents, aggression, scenarios)
        self.sim.set_pending_learners(self.learners)
        return 4 * 4 * self.n

    def iterate(self, native: bool = True):
        """One update: rollout + return normalisation + GAE + PPO. Returns the PPO metrics.

        The rollout loop runs natively (t8b_collect_rollout) unless native is False, which
        runs the same sequence of calls from Python."""
        update = self.update_index = self.update_index + 1
        self.policy.prepare_shuffle(self.samples, self.epochs, self.seed + update)
        sim, policy, rollout = self.sim, self.policy, self.rollout
        started = time.perf_counter()
        if native:
            call("t8b_collect_rollout", sim.handle, policy._handle, rollout._handle,
                 self.opponent._handle if self.opponent is not None else None, self.seed, update, self.horizon, 1.0,
                 None)
        else:
            self.rollout_from_python(update)
        self.rollout_host_ms = 1000.0 * (time.perf_counter() - started)  # time to queue the rollout
        marker = getattr(self, "rollout_event", None)
        if marker is not None:
            marker.record()
        rollout.normalize_rewards(0.99)
        rollout.compute_gae(0.99, 0.95, True)
        return policy.update_ppo(rollout.device_view(packed=True), self.ppo, self.seed + update)

    def rollout_from_python(self, update):
        """The rollout loop of t8b_collect_rollout, call for call, from Python."""
        t, n = self.horizon, self.n
        sim, policy, rollout = self.sim, self.policy, self.rollout
        tables = sim.learner_feature_tables()
        for step in range(t):
            counter = update * t + step
            obs, bits = sim.learner_observations(), sim.learner_mask_bits()
            opponent_actions = self.opponent_launch(counter) if self.opponent is not None else None
            out = policy.forward(obs, None, n, self.seed + 1, counter, False, None, tables, mask_bits=bits)
            if step > 0:
                rollout.record_outcome_device(step - 1, sim.rewards(), sim.terminated(), sim.truncated(), out["values"])
            rollout.record_policy_device(step, obs, None, out["actions"], out["log_probabilities"], out["values"],
                                         None, tables, out["entropies"], mask_bits=bits)
            if opponent_actions is not None:
                torch.cuda.current_stream().wait_stream(self.opponent_stream)
            sim.step(out["actions"], opponent_actions, self.seed, counter + 1)
            if step == t - 1:
                last = policy.forward(sim.learner_observations(), None, n, self.seed + 3, counter, True, None, tables,
                                      mask_bits=sim.learner_mask_bits())
                rollout.record_outcome_device(step, sim.rewards(), sim.terminated(), sim.truncated(), last["values"])
            sim.reset_done(self.seed, counter + 1)

    def opponent_launch(self, counter):
        """Enqueues the frozen policy's forward for this decision on the opponent stream, after
        the simulator's last step; it overlaps the learner's forward, and the caller makes the
        main stream wait for it before stepping the simulator."""
        side = self.opponent_stream
        # the views first: the opponent's masks are computed on the simulator's stream when asked for
        obs, tables, bits = (self.sim.opponent_observations(), self.sim.opponent_feature_tables(),
                             self.sim.opponent_mask_bits())
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            out = self.opponent.forward(obs, None, self.n, self.seed + 2, counter, False, side.cuda_stream, tables,
                                        mask_bits=bits)
        return out["actions"]

    def host_boundary(self):
        """The per-update host traffic of the reference trainer (schedule upload, tally and
        metric download): returns (bytes to device, bytes to host)."""
        up = self.upload_schedule()
        tally, scenario, learner, bot = self.sim.download_and_clear_tally()
        down = tally.nbytes + scenario.nbytes + learner.nbytes + bot.nbytes
        return up, down
