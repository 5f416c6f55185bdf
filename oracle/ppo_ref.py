"""Test infrastructure (not product code): a CPU restatement, in numpy float64, of the policy
and PPO arithmetic of the reference's src/ppo.cu, which has no CPU implementation of its own.
Each function cites the lines it follows. Pinned by tests/test_ppo_oracle.py against the
reference's own known-answer test (tests/ppo_math_tests.cpp) and finite differences."""
from __future__ import annotations

import numpy as np

MASK64 = (1 << 64) - 1


def splitmix64(v: int) -> int:
    v = (v + 0x9E3779B97F4A7C15) & MASK64
    v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & MASK64
    return v ^ (v >> 31)


def uniform01(seed: int, step: int, lane: int) -> np.float32:
    """src/ppo.cu:224-230: the sampler's uniform in float32."""
    bits = splitmix64(seed ^ splitmix64(step) ^ splitmix64(lane))
    return np.float32(np.float32((bits >> 40) + 0.5) * np.float32(1.0 / 16777216.0))


def layout(observation_size: int, hidden: int, layers: int, outputs: int):
    """Canonical parameter order w1, b1, ..., w_out, b_out (src/ppo.cu:974-1000) -> [(name, shape)]."""
    shapes = []
    for l in range(layers):
        shapes.append((f"w{l + 1}", (hidden, observation_size if l == 0 else hidden)))
        shapes.append((f"b{l + 1}", (hidden,)))
    shapes.append(("w_out", (outputs, hidden)))
    shapes.append(("b_out", (outputs,)))
    return shapes


def unflatten(flat: np.ndarray, shapes):
    out, at = {}, 0
    for name, shape in shapes:
        size = int(np.prod(shape))
        out[name] = flat[at: at + size].reshape(shape).astype(np.float64)
        at += size
    return out


def flatten(tensors: dict, shapes) -> np.ndarray:
    return np.concatenate([tensors[name].reshape(-1) for name, _ in shapes])


def normalize_observations(obs, mean, variance, epsilon, clip):
    """normalize_observations_kernel + refresh_inverse_standard_deviation_kernel (src/ppo.cu:132-145, 205-215)."""
    istd = 1.0 / np.sqrt(variance.astype(np.float64) + epsilon)
    return np.clip((obs - mean) * istd, -clip, clip)


def forward(x: np.ndarray, params: dict, layers: int):
    """forward_network (src/ppo.cu:1248-1292): tanh hidden layers, linear output. Returns the
    hidden activations and the output [n, outputs]."""
    hs = []
    h = x
    for l in range(layers):
        h = np.tanh(h @ params[f"w{l + 1}"].T + params[f"b{l + 1}"])
        hs.append(h)
    out = h @ params["w_out"].T + params["b_out"]
    return hs, out


def parametric_scores(query: np.ndarray, features: np.ndarray, tables: np.ndarray):
    """parametric_policy_output_kernel (src/ppo.cu:316-348): q . F[table, a] / sqrt(F)."""
    f = features.shape[-1]
    return np.einsum("nf,naf->na", query, features[tables]) / np.sqrt(f)


def legal_set(mask: np.ndarray) -> np.ndarray:
    """The sampler's legality rule: masked actions, or action 0 when nothing is legal (src/ppo.cu:254-258)."""
    mask = mask.astype(bool)
    any_legal = mask.any(axis=-1, keepdims=True)
    fallback = np.zeros_like(mask)
    fallback[..., 0] = True
    return np.where(any_legal, mask, fallback)


def log_softmax_masked(logits: np.ndarray, mask: np.ndarray):
    """Masked log-softmax as src/ppo.cu:476-489: (log-probabilities over legal actions, probabilities)."""
    legal = legal_set(mask)
    masked = np.where(legal, logits, -np.inf)
    maximum = masked.max(axis=-1, keepdims=True)
    total = np.where(legal, np.exp(logits - maximum), 0.0).sum(axis=-1, keepdims=True)
    log_sum = np.log(np.maximum(total, 1e-20)) + maximum
    lp = logits - log_sum
    p = np.where(legal, np.exp(lp), 0.0)
    return lp, p, legal


def entropy(lp, p):
    return -(p * np.where(p > 0, lp, 0.0)).sum(axis=-1)


def objective(output, mask, action, old_lp, old_v, adv, ret, clip, value_clip, value_coef, entropy_coef):
    """The per-sample PPO objective the reference differentiates (tests/ppo_math_tests.cpp:26-71)."""
    output = np.asarray(output, np.float64)
    logits, value = output[:-1], output[-1]
    lp, p, legal = log_softmax_masked(logits[None], np.asarray(mask)[None])
    lp, p = lp[0], p[0]
    ratio = np.exp(lp[action] - old_lp)
    policy = -min(ratio * adv, np.clip(ratio, 1 - clip, 1 + clip) * adv)
    h = entropy(lp[None], p[None])[0]
    err = value - ret
    vloss = 0.5 * err * err
    if value_clip > 0:
        cv = old_v + np.clip(value - old_v, -value_clip, value_clip)
        vloss = max(vloss, 0.5 * (cv - ret) ** 2)
    return policy + value_coef * vloss - entropy_coef * h


def objective_gradient(logits, mask, actions, old_lp, old_v, adv, ret, value, clip, value_clip, value_coef,
                       entropy_coef, batch):
    """ppo_output_gradient_kernel (src/ppo.cu:453-565), vectorised over samples: the gradient of
    the batch-mean objective w.r.t. the logits and the value, and the per-sample metrics."""
    lp, p, legal = log_softmax_masked(logits, mask)
    any_legal = mask.astype(bool).any(axis=-1)
    selected = np.where(any_legal, actions, 0)
    n = logits.shape[0]
    new_lp = lp[np.arange(n), selected]
    log_ratio = new_lp - old_lp
    ratio = np.exp(log_ratio)
    unclipped = ratio * adv
    clipped = np.clip(ratio, 1 - clip, 1 + clip) * adv
    use_unclipped = unclipped <= clipped
    policy_loss = -np.minimum(unclipped, clipped)
    lp_grad = np.where(use_unclipped, -adv * ratio, 0.0)
    h = entropy(lp, p)
    onehot = np.zeros_like(logits)
    onehot[np.arange(n), selected] = 1.0
    grad = (lp_grad[:, None] * (onehot - p)) / batch
    grad = grad + entropy_coef * p * (np.where(legal, lp, 0.0) + h[:, None]) / batch
    grad = np.where(legal, grad, 0.0)
    err = value - ret
    vgrad = err.copy()
    vloss = 0.5 * err * err
    if value_clip > 0:
        delta = value - old_v
        cv = old_v + np.clip(delta, -value_clip, value_clip)
        cerr = cv - ret
        closs = 0.5 * cerr * cerr
        use = closs > vloss
        vloss = np.where(use, closs, vloss)
        vgrad = np.where(use, np.where(np.abs(delta) <= value_clip, cerr, 0.0), vgrad)
    dvalue = value_coef * vgrad / batch
    legal_count = legal.sum(axis=-1)
    metrics = {
        "policy_loss": policy_loss, "value_loss": vloss, "entropy": h,
        "kl": (ratio - 1) - log_ratio, "clip": (np.abs(ratio - 1) > clip).astype(np.float64),
        "decision": (legal_count > 1).astype(np.float64), "decision_entropy": np.where(legal_count > 1, h, 0.0),
    }
    return grad, dvalue, metrics


def query_gradient(dlogits, features, tables):
    """parametric_policy_gradient_kernel (src/ppo.cu:350-381): dq = sum_a dscore_a F[table, a] / sqrt(F)."""
    f = features.shape[-1]
    return np.einsum("na,naf->nf", dlogits, features[tables]) / np.sqrt(f)


def backward(x, hs, params, dout, layers):
    """backward_network (src/ppo.cu:1296-1337): weight, bias and input gradients of the MLP."""
    grads = {}
    grads["w_out"] = dout.T @ hs[-1]
    grads["b_out"] = dout.sum(axis=0)
    up = dout @ params["w_out"]
    for l in range(layers - 1, -1, -1):
        dz = up * (1.0 - hs[l] ** 2)
        inp = x if l == 0 else hs[l - 1]
        grads[f"w{l + 1}"] = dz.T @ inp
        grads[f"b{l + 1}"] = dz.sum(axis=0)
        if l > 0:
            up = dz @ params[f"w{l + 1}"]
    return grads


def adam(params, grads, m1, m2, step, lr, beta1, beta2, eps, max_norm):
    """gradient_square_sum_kernel + adam_kernel (src/ppo.cu:659-682, 710-736), float32 arithmetic."""
    g = grads.astype(np.float32)
    norm = np.float32(np.sqrt(np.sum(g.astype(np.float64) ** 2)))
    scale = np.float32(max_norm) / np.float32(max(norm, 1e-12)) if norm > max_norm else np.float32(1.0)
    g = g * scale
    b1, b2 = np.float32(beta1), np.float32(beta2)
    m = b1 * m1.astype(np.float32) + (np.float32(1) - b1) * g
    v = b2 * m2.astype(np.float32) + (np.float32(1) - b2) * g * g
    bc1 = np.float32(1) - np.float32(beta1) ** np.float32(step)
    bc2 = np.float32(1) - np.float32(beta2) ** np.float32(step)
    p = params.astype(np.float32) - np.float32(lr) * (m / bc1) / (np.sqrt(v / bc2) + np.float32(eps))
    return p, m, v, float(norm)


def gae(rewards, values, terminated, truncated, next_values, gamma, lam):
    """gae_kernel (src/ppo.cu:2003-2029): [horizon, envs] arrays, reverse sweep per environment."""
    horizon = rewards.shape[0]
    adv = np.zeros_like(rewards, dtype=np.float64)
    nxt = np.zeros(rewards.shape[1], np.float64)
    for t in range(horizon - 1, -1, -1):
        time_limit = truncated[t] != 0
        ended = terminated[t] != 0
        bootstrap = np.where(ended & ~time_limit, 0.0, 1.0)
        trace = np.where(ended | time_limit, 0.0, 1.0)
        delta = rewards[t] + gamma * next_values[t] * bootstrap - values[t]
        nxt = delta + gamma * lam * trace * nxt
        adv[t] = nxt
    return adv, adv + values


def normalize_advantages(adv):
    """advantage stats + normalize_advantages_kernel (src/ppo.cu:2031-2091)."""
    a = adv.astype(np.float64)
    mean = a.mean()
    second = (a * a).mean()
    return (a - mean) / np.sqrt(max(second - mean * mean, 1e-12))


def discounted_returns(rewards, terminated, truncated, running, gamma):
    """discounted_return_kernel (src/ppo.cu:2114-2131)."""
    horizon = rewards.shape[0]
    out = np.zeros_like(rewards, dtype=np.float64)
    r = running.astype(np.float64).copy()
    for t in range(horizon):
        r = r * gamma + rewards[t]
        out[t] = r
        r = np.where((terminated[t] != 0) | (truncated[t] != 0), 0.0, r)
    return out, r


def merge_moments(count, mean, variance, batch):
    """Chan et al. merge of a batch into running (count, mean, variance) (src/ppo.cu:183-203, 2384-2400)."""
    b = np.asarray(batch, np.float64)
    n = b.shape[0]
    bm = b.mean(axis=0)
    bm2 = ((b - bm) ** 2).sum(axis=0)
    total = count + n
    delta = bm - mean
    m2 = variance * count + bm2 + delta * delta * count * n / total
    return total, mean + delta * n / total, m2 / total
