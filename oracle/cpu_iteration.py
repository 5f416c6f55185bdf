"""Test infrastructure (not product code): the CPU timing leg of bench.py. One self-play training
iteration on the host cores: the reference's own CPU environment contract (oracle/_ref, one
thread per core over fights) for the rollout, and a float32 numpy port of the policy forward,
PPO objective, backward and Adam (the arithmetic of oracle/ppo_ref.py, vectorised) for the
decisions and the update. The reference has no CPU trainer; this is the CPU baseline."""
from __future__ import annotations

import os
import time

import numpy as np

from . import ppo_ref as R
from . import ref


class CpuIteration:
    def __init__(self, roster_raw: bytes, features: np.ndarray, env_config, envs: int, horizon: int, epochs: int = 4,
                 minibatches: int = 8, hidden: int = 512, threads: int | None = None, seed: int = 3):
        self.threads = threads or os.cpu_count() or 1
        self.roster = ref.RefRoster(roster_raw)
        self.env = ref.RefEnv(self.roster, envs, env_config, threads=self.threads)
        self.n, self.t = envs, horizon
        self.epochs, self.minibatches = epochs, minibatches
        rng = np.random.default_rng(seed)
        count = features.shape[0]
        sides = (np.arange(envs) % 2 == 0).astype(np.uint8)
        learners = rng.integers(0, count, envs)
        opponents = rng.integers(0, count, envs)
        p1 = np.where(sides == 1, learners, opponents)
        p2 = np.where(sides == 1, opponents, learners)
        self.env.setup(p1=p1, p2=p2, learner_is_p1=sides, opponents=opponents, aggression=rng.random(envs),
                       scenarios=np.zeros(envs), learners=learners)
        self.env.reset_all(seed, 0)
        self.features = features.astype(np.float32)
        self.width = self.env.width
        w = self.width
        self.params = {
            "w1": (rng.normal(size=(hidden, w)) / np.sqrt(w)).astype(np.float32), "b1": np.zeros(hidden, np.float32),
            "w2": (rng.normal(size=(hidden, hidden)) / np.sqrt(hidden)).astype(np.float32),
            "b2": np.zeros(hidden, np.float32),
            "w_out": (rng.normal(size=(33, hidden)) * 0.01).astype(np.float32), "b_out": np.zeros(33, np.float32),
        }
        self.m = {k: np.zeros_like(v) for k, v in self.params.items()}
        self.v = {k: np.zeros_like(v) for k, v in self.params.items()}
        self.step = 0
        self.rng = rng
        self.seed = seed
        self.update_index = 0

    def _forward(self, x):
        p = self.params
        h1 = np.tanh(x @ p["w1"].T + p["b1"])
        h2 = np.tanh(h1 @ p["w2"].T + p["b2"])
        return h1, h2, h2 @ p["w_out"].T + p["b_out"]

    def _scores(self, q, tables):
        return np.einsum("nf,naf->na", q, self.features[tables]) / np.float32(np.sqrt(32.0))

    def iterate(self) -> float:
        """One iteration (rollout + GAE + PPO update); returns its wall seconds."""
        start = time.perf_counter()
        self.update_index += 1
        n, t = self.n, self.t
        obs = np.zeros((t, n, self.width), np.float32)
        masks = np.zeros((t, n, 368), np.uint8)
        actions = np.zeros((t, n), np.int64)
        lps = np.zeros((t, n), np.float32)
        values = np.zeros((t + 1, n), np.float32)
        rewards = np.zeros((t, n), np.float32)
        term = np.zeros((t, n), np.uint8)
        tables = np.zeros((t, n), np.int64)
        for s in range(t):
            state = self.env.read()
            obs[s], masks[s] = state["learner_obs"], state["learner_masks"]
            tables[s] = np.where(np.arange(n) % 2 == 0, state["p1"], state["p2"])
            _, _, out = self._forward(obs[s])
            logits = self._scores(out[:, :32], tables[s])
            lp, p, legal = R.log_softmax_masked(logits.astype(np.float64), masks[s])
            u = self.rng.random(n)
            cdf = np.cumsum(p, axis=1)
            actions[s] = np.minimum((cdf < (u * cdf[:, -1])[:, None]).sum(axis=1), 367)
            lps[s] = lp[np.arange(n), actions[s]]
            values[s] = out[:, 32]
            counter = self.update_index * t + s
            self.env.step(actions[s], None, self.seed, counter + 1)
            after = self.env.read()
            rewards[s], term[s] = after["rewards"], after["terminated"]
            self.env.reset_done(self.seed, counter + 1)
        values[t] = self._forward(self.env.read()["learner_obs"])[2][:, 32]
        adv, ret = R.gae(rewards, values[:t], term, np.zeros_like(term), values[1:], 0.99, 0.95)
        adv = R.normalize_advantages(adv).astype(np.float32)
        samples = n * t
        flat = lambda a: a.reshape(samples, *a.shape[2:])
        o_all, m_all, a_all, lp_all, v_all = flat(obs), flat(masks), flat(actions), flat(lps), flat(values[:t])
        adv_all, ret_all, tab_all = flat(adv), flat(ret.astype(np.float32)), flat(tables)
        mb = samples // self.minibatches
        for _ in range(self.epochs):
            order = self.rng.permutation(samples)
            for k in range(self.minibatches):
                idx = order[k * mb:(k + 1) * mb]
                self._update(o_all[idx], m_all[idx], a_all[idx], lp_all[idx], v_all[idx], adv_all[idx], ret_all[idx],
                             tab_all[idx])
        return time.perf_counter() - start

    def _update(self, x, masks, actions, old_lp, old_v, adv, ret, tables):
        p = self.params
        b = x.shape[0]
        h1, h2, out = self._forward(x)
        logits = self._scores(out[:, :32], tables)
        g, dv, _ = R.objective_gradient(logits.astype(np.float64), masks, actions, old_lp, old_v, adv, ret,
                                        out[:, 32].astype(np.float64), 0.2, 0.2, 0.5, 0.01, b)
        dq = np.einsum("na,naf->nf", g.astype(np.float32), self.features[tables]) / np.float32(np.sqrt(32.0))
        dout = np.concatenate([dq, dv[:, None].astype(np.float32)], axis=1)
        grads = {"w_out": dout.T @ h2, "b_out": dout.sum(0)}
        dz2 = (dout @ p["w_out"]) * (1 - h2 * h2)
        grads["w2"], grads["b2"] = dz2.T @ h1, dz2.sum(0)
        dz1 = (dz2 @ p["w2"]) * (1 - h1 * h1)
        grads["w1"], grads["b1"] = dz1.T @ x, dz1.sum(0)
        self.step += 1
        norm = np.sqrt(sum(float((gv.astype(np.float64) ** 2).sum()) for gv in grads.values()))
        scale = 0.5 / norm if norm > 0.5 else 1.0
        bc1, bc2 = 1 - 0.9 ** self.step, 1 - 0.999 ** self.step
        for k in p:
            gk = grads[k] * scale
            self.m[k] = 0.9 * self.m[k] + 0.1 * gk
            self.v[k] = 0.999 * self.v[k] + 0.001 * gk * gk
            p[k] -= 5e-4 * (self.m[k] / bc1) / (np.sqrt(self.v[k] / bc2) + 1e-5)
