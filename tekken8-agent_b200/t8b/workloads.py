"""Seeded synthetic inputs with the shapes and value distributions of the measured workloads
(no recorded game data exists; every tensor is drawn on the device from a seeded generator).

config2_rollout: the GAE + clipped-loss microbench, a rollout of T = 128 decisions x N = 32,768
fights whose policy scores K = 256 candidate slots, about 30 % of them legal.
  * rewards are 0 except on health-change decisions (one in ten), where they are N(0, 0.1); a
    round's last decision carries +-1;
  * round ends are Bernoulli(1/600) per decision; one in ten of them is a time-limit end, flagged
    truncated as well as terminated (the bootstrap/trace masks of src/ppo.cu:2021-2023);
  * values and bootstrap values are N(0, 1);
  * the acting policy's logits are N(0, 1); actions are drawn from its masked softmax
    (Gumbel-max) and the old log-probability is that softmax's at the action;
  * the current policy's outputs are the acting logits plus N(0, 0.05) and the old value plus
    N(0, 0.1), as after a few minibatch updates, so ratios and values straddle their clips.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class Config2:
    horizon: int
    envs: int
    slots: int
    rewards: torch.Tensor        # [T][N] f32
    values: torch.Tensor         # [T][N] f32
    next_values: torch.Tensor    # [T][N] f32
    terminated: torch.Tensor     # [T][N] u8
    truncated: torch.Tensor      # [T][N] u8
    outputs: torch.Tensor        # [T*N][K + 1] f32: current logits, then the current value
    masks: torch.Tensor          # [T*N][K] u8
    actions: torch.Tensor        # [T*N] i64
    old_log_probabilities: torch.Tensor  # [T*N] f32

    @property
    def samples(self) -> int:
        return self.horizon * self.envs


def config2_rollout(horizon: int = 128, envs: int = 32768, slots: int = 256, seed: int = 1,
                    device: str = "cuda", chunk: int = 524288) -> Config2:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    t, n = horizon, envs
    rnd = lambda *shape: torch.rand(*shape, generator=g, device=device)
    nrm = lambda *shape: torch.randn(*shape, generator=g, device=device)
    health = rnd(t, n) < 0.1
    rewards = torch.where(health, 0.1 * nrm(t, n), torch.zeros(t, n, device=device))
    done = rnd(t, n) < 1.0 / 600.0
    rewards = torch.where(done, torch.where(rnd(t, n) < 0.5, -1.0, 1.0), rewards)
    truncated = done & (rnd(t, n) < 0.1)
    values = nrm(t, n)
    next_values = nrm(t, n)
    s = t * n
    outputs = torch.empty(s, slots + 1, device=device)
    masks = torch.empty(s, slots, dtype=torch.uint8, device=device)
    actions = torch.empty(s, dtype=torch.int64, device=device)
    old_lp = torch.empty(s, device=device)
    flat_values = values.reshape(-1)
    for begin in range(0, s, chunk):
        end = min(s, begin + chunk)
        rows = end - begin
        legal = rnd(rows, slots) < 0.3
        legal[:, 0] |= ~legal.any(dim=1)
        acting = nrm(rows, slots)
        masked = acting.masked_fill(~legal, float("-inf"))
        gumbel = -torch.log(-torch.log(rnd(rows, slots).clamp_min(1e-20)))
        action = torch.argmax(masked + gumbel, dim=1)
        old_lp[begin:end] = torch.log_softmax(masked, dim=1).gather(1, action[:, None])[:, 0]
        actions[begin:end] = action
        masks[begin:end] = legal.to(torch.uint8)
        outputs[begin:end, :slots] = acting + 0.05 * nrm(rows, slots)
        outputs[begin:end, slots] = flat_values[begin:end] + 0.1 * nrm(rows)
    return Config2(t, n, slots, rewards, values, next_values, done.to(torch.uint8), truncated.to(torch.uint8),
                   outputs, masks, actions, old_lp)
