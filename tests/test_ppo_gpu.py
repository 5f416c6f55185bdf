"""Policy, PPO update and rollout buffer against the numpy oracle (oracle/ppo_ref.py).

Tolerances: network outputs and gradients go through bf16 tensor-core products with fp32
accumulation, compared to float64 with a relative (norm) tolerance of 2e-2; the scorer,
sampler, objective, GAE, normalisers and Adam are fp32 arithmetic compared at 1e-4 or tighter;
GAE keeps the reference's own 2e-5 absolute bound (tests/rollout_tests.cpp:75-93)."""
import numpy as np
import pytest

from oracle import ppo_ref as R

pytestmark = pytest.mark.gpu


def make_batch(n, features_tables, rng, width=151):
    obs = rng.random((n, width)).astype(np.float32)
    obs[:, 64:148] = 0.0
    obs[np.arange(n), 64 + rng.integers(0, 41, n)] = 1.0
    obs[np.arange(n), 106 + rng.integers(0, 41, n)] = 1.0
    tables = rng.integers(0, features_tables, n).astype(np.int32)
    masks = (rng.random((n, 368)) < 0.3).astype(np.uint8)
    masks[:, 0] = 1
    return obs, tables, masks


def relative(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def features(roster):
    return roster.feature_tables()


def oracle_params(policy):
    cfg = policy.config
    shapes = R.layout(cfg.observation_size, cfg.hidden_size, cfg.shared_layers, cfg.action_feature_size + 1)
    return shapes, R.unflatten(policy.parameters().astype(np.float64), shapes)


def test_initial_weights_are_orthogonal(cuda):
    from t8b.policy import GpuActorCritic
    policy = GpuActorCritic(256, seed=2027)
    shapes, p = oracle_params(policy)
    w1, w2, wo = p["w1"], p["w2"], p["w_out"]
    assert np.allclose(w1.T @ w1, 2.0 * np.eye(151), atol=1e-4)  # tall: orthonormal columns, gain sqrt(2)
    assert np.allclose(w2 @ w2.T, 2.0 * np.eye(512), atol=1e-4)
    assert np.allclose(wo[32] @ wo[32], 1.0, atol=1e-5)  # value row keeps unit gain
    assert np.allclose(np.abs(wo[:32]).max(), np.abs(wo[:32]).max(), atol=0) and np.abs(wo[:32]).max() < 0.01
    assert all(np.all(p[f"b{i}"] == 0) for i in (1, 2)) and np.all(p["b_out"] == 0)


def test_forward_matches_oracle(cuda, features):
    import torch
    from t8b.policy import GpuActorCritic
    rng = np.random.default_rng(4)
    n = 6000
    policy = GpuActorCritic(8192, seed=7)
    policy.set_action_feature_tables(features)
    # non-trivial weights: scale the output layer up so scores spread
    flat = policy.parameters()
    shapes, p = oracle_params(policy)
    p["w_out"] *= 30.0
    p["b1"] = rng.normal(scale=0.1, size=p["b1"].shape)
    policy.set_parameters(R.flatten(p, shapes).astype(np.float32))
    obs, tables, masks = make_batch(n, features.shape[0], rng)
    d = lambda a: torch.as_tensor(a, device="cuda")
    out = policy.forward(d(obs), d(masks), n, seed=11, step=3, deterministic=True, tables=d(tables), want_logits=True)
    got = policy.outputs(n)
    _, want = R.forward(obs.astype(np.float64), p, 2)
    assert relative(got, want) < 2e-2
    # scorer + sampler against the GPU's own network outputs (fp32 path only)
    q, v = got[:, :32].astype(np.float64), got[:, 32]
    logits = R.parametric_scores(q, features.astype(np.float64), tables)
    assert np.allclose(out["logits"].cpu().numpy(), logits, atol=1e-5, rtol=1e-4)
    lp, prob, legal = R.log_softmax_masked(logits, masks)
    best = np.argmax(np.where(legal, logits, -np.inf), axis=1)
    assert np.array_equal(out["actions"].cpu().numpy(), best)
    assert np.allclose(out["log_probabilities"].cpu().numpy(), lp[np.arange(n), best], atol=1e-4)
    assert np.allclose(out["entropies"].cpu().numpy(), R.entropy(lp, prob), atol=1e-4)
    assert np.array_equal(out["values"].cpu().numpy(), v)
    # stochastic: inverse-CDF with the reference uniform; flips only at a CDF boundary
    out = policy.forward(d(obs), d(masks), n, seed=11, step=3, deterministic=False, tables=d(tables))
    actions = out["actions"].cpu().numpy()
    agree = 0
    for i in range(n):
        u = float(R.uniform01(11, 3, i))
        cdf = np.cumsum(prob[i])
        want_i = int(np.searchsorted(cdf, u * cdf[-1]))
        agree += int(actions[i] == want_i)
    assert agree >= n - 3
    assert np.all(masks[np.arange(n), actions] == 1)


def test_bad_table_gives_nan_and_is_rejected(cuda, features):
    import torch
    from t8b.policy import GpuActorCritic
    rng = np.random.default_rng(5)
    policy = GpuActorCritic(256, seed=3)
    policy.set_action_feature_tables(features)
    obs, tables, masks = make_batch(64, features.shape[0], rng)
    tables[5] = features.shape[0]
    d = lambda a: torch.as_tensor(a, device="cuda")
    out = policy.forward(d(obs), d(masks), 64, tables=d(tables), deterministic=True)
    vals = out["values"].cpu().numpy()
    assert np.isnan(vals[5]) and np.all(np.isfinite(np.delete(vals, 5)))


def test_multi_table_forward_equals_single_table(cuda, features):
    """tests/feature_tables_tests.cpp: a sample scored against its table in a many-table policy
    equals the same sample in a policy holding only that table."""
    import torch
    from t8b.policy import GpuActorCritic
    rng = np.random.default_rng(6)
    obs, tables, masks = make_batch(512, features.shape[0], rng)
    d = lambda a: torch.as_tensor(a, device="cuda")
    many = GpuActorCritic(512, seed=9)
    many.set_action_feature_tables(features)
    a = many.forward(d(obs), d(masks), 512, tables=d(tables), deterministic=True, want_logits=True)
    logits_many = a["logits"].cpu().numpy().copy()
    one = GpuActorCritic(512, seed=9)
    one.set_action_feature_tables(features[7:8])
    b = one.forward(d(obs), d(masks), 512, tables=d(np.zeros(512, np.int32)), deterministic=True, want_logits=True)
    rows = tables == 7
    assert np.array_equal(logits_many[rows], b["logits"].cpu().numpy()[rows])


def rollout_inputs(policy, features, n, rng):
    import torch
    obs, tables, masks = make_batch(n, features.shape[0], rng)
    d = lambda a: torch.as_tensor(a, device="cuda")
    out = policy.forward(d(obs), d(masks), n, seed=1, step=0, tables=d(tables))
    actions = out["actions"].cpu().numpy()
    old_lp = out["log_probabilities"].cpu().numpy() - rng.normal(scale=0.05, size=n).astype(np.float32)
    old_v = out["values"].cpu().numpy()
    adv = rng.normal(size=n).astype(np.float32)
    ret = (old_v + rng.normal(scale=0.5, size=n)).astype(np.float32)
    return obs, tables, masks, actions, old_lp, old_v, adv, ret


def view_of(arrays):
    import torch
    from t8b._lib import RolloutView
    obs, tables, masks, actions, old_lp, old_v, adv, ret = arrays
    keep = [torch.as_tensor(a, device="cuda") for a in (obs, masks, actions.astype(np.int64), old_lp, old_v, adv, ret,
                                                         tables)]
    v = RolloutView()
    v.observations, v.action_masks, v.actions, v.old_log_probabilities, v.old_values, v.advantages, v.returns, \
        v.feature_tables = [t.data_ptr() for t in keep]
    v.sample_count = obs.shape[0]
    v.environment_count = obs.shape[0]
    v.horizon = 1
    return v, keep


def run_update(features, arrays, n, seed=12, scale_out=30.0, lr=1e-3):
    from t8b.policy import GpuActorCritic, ppo_config
    policy = GpuActorCritic(n, seed=seed)
    policy.set_action_feature_tables(features)
    shapes, p = oracle_params(policy)
    p["w_out"] *= scale_out
    policy.set_parameters(R.flatten(p, shapes).astype(np.float32))
    before = policy.parameters()
    if arrays is None:
        arrays = rollout_inputs(policy, features, n, np.random.default_rng(8))
    view, keep = view_of(arrays)
    cfg = ppo_config(epochs=1, minibatch_size=n, learning_rate=lr, target_kl=0.0, entropy_coefficient=0.01)
    metrics = policy.update_ppo(view, cfg, shuffle_seed=5)
    return policy, shapes, before, arrays, metrics


def gathered_order(policy, obs, n):
    """The update's sample order, recovered by matching its bf16 layer-1 rows to the inputs."""
    import torch
    xg = policy.activation(0, 0, n)[:, :obs.shape[1]]
    keyed = {torch.tensor(obs[i]).to(torch.bfloat16).float().numpy().tobytes(): i for i in range(n)}
    return np.array([keyed[xg[j].astype(np.float32).tobytes()] for j in range(n)]), xg.astype(np.float64)


def test_update_stages_match_oracle(cuda, features):
    """Every stage of a minibatch update against float64 recomputed from that stage's own inputs:
    forward activations and backward pre-activation gradients within bf16 rounding (1e-2), the
    fused objective within 1e-2 of float64 on the GPU's network outputs, the weight-gradient GEMMs
    within 1e-5 of their operands (bias gradients, summed from fp32 values before the bf16 rows
    are stored, within 1e-2 of the stored rows' sums), and the metrics equal to the oracle's."""
    n = 8192
    policy, shapes, before, arrays, metrics = run_update(features, None, n)
    obs, tables, masks, actions, old_lp, old_v, adv, ret = arrays
    params = R.unflatten(before.astype(np.float64), shapes)
    got = R.unflatten(policy.gradients().astype(np.float64), shapes)
    order, xg = gathered_order(policy, obs, n)
    a = {key: policy.activation(*key, n).astype(np.float64) for key in ((1, 0), (1, 1), (2, 0), (2, 1))}
    dg = policy.activation(3, 0, n)[:, :33].astype(np.float64)
    o = policy.outputs(n).astype(np.float64)
    assert relative(a[(1, 0)], np.tanh(xg @ params["w1"].T + params["b1"])) < 1e-2
    assert relative(a[(1, 1)], np.tanh(a[(1, 0)] @ params["w2"].T + params["b2"])) < 1e-2
    assert relative(o, np.concatenate([a[(1, 1)] @ params["w_out"].T + params["b_out"]], 1)) < 1e-2
    lg = R.parametric_scores(o[:, :32], features.astype(np.float64), tables[order])
    g, dv, m = R.objective_gradient(lg, masks[order], actions[order], old_lp[order], old_v[order], adv[order],
                                    ret[order], o[:, 32], 0.2, 0.2, 0.5, 0.01, n)
    want_dout = np.concatenate([R.query_gradient(g, features.astype(np.float64), tables[order]), dv[:, None]], 1)
    assert relative(dg, want_dout) < 1e-2
    assert relative(a[(2, 1)], (dg @ params["w_out"]) * (1 - a[(1, 1)] ** 2)) < 1e-2
    assert relative(a[(2, 0)], (a[(2, 1)] @ params["w2"]) * (1 - a[(1, 0)] ** 2)) < 1e-2
    assert relative(got["w_out"], dg.T @ a[(1, 1)]) < 1e-5
    assert relative(got["b_out"], dg.sum(0)) < 1e-2  # fp32 sums before bf16 storage
    assert relative(got["w2"], a[(2, 1)].T @ a[(1, 0)]) < 1e-5
    assert relative(got["b2"], a[(2, 1)].sum(0)) < 1e-2  # fp32 sums before bf16 storage
    assert relative(got["w1"], a[(2, 0)].T @ xg) < 1e-5
    assert relative(got["b1"], a[(2, 0)].sum(0)) < 1e-2  # fp32 sums before bf16 storage
    for key, name in (("policy_loss", "policy_loss"), ("value_loss", "value_loss"), ("entropy", "entropy"),
                      ("approximate_kl", "kl"), ("clip_fraction", "clip"), ("decision_fraction", "decision")):
        assert abs(metrics[key] - m[name].mean()) <= 1e-4 * max(1.0, abs(m[name].mean())), key


def test_update_gradient_and_adam_end_to_end(cuda, features):
    """A well-conditioned minibatch (eight distinct samples, each repeated) so the batch gradient
    does not cancel: the whole update's gradient within 2e-2 of float64 per tensor (north_star's
    bound for bf16 GEMMs), and Adam exact in fp32."""
    import torch
    from t8b.policy import GpuActorCritic
    rng = np.random.default_rng(13)
    n, distinct = 8192, 8
    probe = GpuActorCritic(n, seed=12)
    probe.set_action_feature_tables(features)
    base = rollout_inputs(probe, features, distinct, rng)
    reps = n // distinct
    arrays = [np.repeat(a, reps, axis=0) for a in base]
    arrays[0] = arrays[0] + (np.arange(n) % reps)[:, None].astype(np.float32) * 1e-3 * (np.arange(151) == 7)
    arrays[6] = arrays[6] + 0.3  # returns above the values: a coherent value gradient
    arrays[5] = np.abs(arrays[5]) + 0.5
    policy, shapes, before, arrays, metrics = run_update(features, arrays, n)
    obs, tables, masks, actions, old_lp, old_v, adv, ret = arrays
    params = R.unflatten(before.astype(np.float64), shapes)
    x = obs.astype(np.float64)
    hs, out = R.forward(x, params, 2)
    logits = R.parametric_scores(out[:, :32], features.astype(np.float64), tables)
    g, dv, m = R.objective_gradient(logits, masks, actions, old_lp, old_v, adv, ret, out[:, 32], 0.2, 0.2, 0.5, 0.01, n)
    dout = np.concatenate([R.query_gradient(g, features.astype(np.float64), tables), dv[:, None]], axis=1)
    want = R.backward(x, hs, params, dout, 2)
    grads = policy.gradients()
    got = R.unflatten(grads.astype(np.float64), shapes)
    errors = {name: relative(got[name], want[name]) for name, _ in shapes}
    print(f"end-to-end gradient vs float64: {errors}")
    assert all(e < 2e-2 for e in errors.values()), errors
    after = policy.parameters()
    m1, m2, step = policy.optimizer_state()
    want_p, want_m, want_v, norm = R.adam(before, grads, np.zeros_like(before), np.zeros_like(before), 1, 1e-3, 0.9,
                                          0.999, 1e-5, 0.5)
    assert step == 1
    assert abs(metrics["gradient_norm"] - norm) <= 1e-5 * norm
    assert np.allclose(after, want_p, rtol=1e-5, atol=1e-7)
    assert np.allclose(m1, want_m, rtol=1e-5, atol=1e-9)
    assert np.allclose(m2, want_v, rtol=1e-5, atol=1e-12)


def test_update_is_bit_reproducible(cuda, features):
    from t8b.policy import GpuActorCritic, ppo_config
    rng = np.random.default_rng(9)
    n = 4096
    results = []
    for _ in range(2):
        policy = GpuActorCritic(n, seed=21)
        policy.set_action_feature_tables(features)
        arrays = rollout_inputs(policy, features, n, np.random.default_rng(9))
        view, keep = view_of(arrays)
        cfg = ppo_config(epochs=2, minibatch_size=n // 4, target_kl=0.0)
        policy.update_ppo(view, cfg, shuffle_seed=77)
        results.append(policy.parameters())
    assert np.array_equal(results[0], results[1])


def test_observation_normalizer_merges_like_the_reference(cuda, features):
    from t8b.policy import GpuActorCritic, ppo_config
    rng = np.random.default_rng(10)
    n = 4096
    policy = GpuActorCritic(n, seed=22)
    policy.set_action_feature_tables(features)
    arrays = rollout_inputs(policy, features, n, rng)
    view, keep = view_of(arrays)
    policy.update_ppo(view, ppo_config(epochs=1, minibatch_size=n, target_kl=0.0), shuffle_seed=1)
    mean, var, count = policy.observation_statistics()
    c, mu, v = R.merge_moments(0, np.zeros(151), np.ones(151), arrays[0])
    assert count == n
    assert np.allclose(mean, mu, atol=1e-6) and np.allclose(var, v, rtol=1e-4, atol=1e-7)


def test_gae_and_advantage_normalization_config2(cuda):
    """The GAE microbench shapes: T = 128, N = 32,768."""
    import torch
    from t8b.policy import GpuRolloutBuffer
    rng = np.random.default_rng(1)
    t, n = 128, 32768
    buf = GpuRolloutBuffer(n, t)
    rewards = np.where(rng.random((t, n)) < 0.1, rng.normal(scale=0.1, size=(t, n)), 0.0).astype(np.float32)
    done = rng.random((t, n)) < 1.0 / 600
    rewards[done] = np.sign(rng.normal(size=done.sum()))
    term = done.astype(np.uint8)
    trunc = (done & (rng.random((t, n)) < 0.1)).astype(np.uint8)
    values = rng.normal(size=(t, n)).astype(np.float32)
    nv = rng.normal(size=(t, n)).astype(np.float32)
    d = lambda a: torch.as_tensor(a, device="cuda")
    obs = torch.zeros((n, 151), device="cuda")
    masks = torch.ones((n, 368), dtype=torch.uint8, device="cuda")
    acts = torch.zeros(n, dtype=torch.int64, device="cuda")
    for s in range(t):
        vals = d(values[s])
        buf.record_policy_device(s, obs, masks, acts, vals, vals)
        buf.record_outcome_device(s, d(rewards[s]), d(term[s]), d(trunc[s]), d(nv[s]))
    buf.compute_gae(0.99, 0.95, normalize=False)
    adv = buf.tensor("advantages").cpu().numpy()
    ret = buf.tensor("returns").cpu().numpy()
    want_adv, want_ret = R.gae(rewards, values, term, trunc, nv, 0.99, 0.95)
    assert np.abs(adv - want_adv).max() < 2e-5
    assert np.abs(ret - want_ret).max() < 2e-5
    buf.compute_gae(0.99, 0.95, normalize=True)
    norm = buf.tensor("advantages").cpu().numpy().astype(np.float64)
    assert abs(norm.mean()) < 2e-4 and abs(norm.var() - 1.0) < 2e-3
    assert np.allclose(norm, R.normalize_advantages(want_adv), atol=1e-4)
    # return normaliser against the oracle
    scale = buf.normalize_rewards(0.99)
    samples, running = R.discounted_returns(rewards, term, trunc, np.zeros(n), 0.99)
    _, _, var = R.merge_moments(0, 0.0, 1.0, samples.reshape(-1))
    assert abs(scale - np.sqrt(var + 1e-8)) <= 1e-4 * scale
    count, mean, variance, disc = buf.return_normalizer_state()
    assert count == t * n and np.allclose(disc, running, atol=1e-4)


def objective_against_oracle(outputs, masks, actions, old_lp, old_v, adv, ret, grads, sums, config, batch,
                             chunk=262144):
    """The GPU objective (grads [n][k + 1], metric sums) against the float64 C restatement
    (oracle/objective.c), chunk by chunk: relative norms of the logit and value gradients over the
    samples not within 1e-5 of a gradient discontinuity (the ratio at 1 +- clip, the value delta
    at +-clip), the metric sums, and the count of such samples."""
    from oracle import objective
    n, width = outputs.shape
    diff = np.zeros(2)
    norm = np.zeros(2)
    want_sums = np.zeros(8)
    margins = 0
    host = lambda t: t.cpu().numpy()
    for begin in range(0, n, chunk):
        end = min(n, begin + chunk)
        want, margin, part = objective.objective(
            host(outputs[begin:end]), host(masks[begin:end]), host(actions[begin:end]), host(old_lp[begin:end]),
            host(old_v[begin:end]), host(adv[begin:end]), host(ret[begin:end]), batch, config.clip_range,
            config.value_clip_range, config.value_coefficient, config.entropy_coefficient)
        want_sums += part
        keep = ~margin
        margins += int(margin.sum())
        got = host(grads[begin:end])[keep].astype(np.float64)
        want = want[keep]
        diff += [np.square(got[:, :-1] - want[:, :-1]).sum(), np.square(got[:, -1] - want[:, -1]).sum()]
        norm += [np.square(want[:, :-1]).sum(), np.square(want[:, -1]).sum()]
    rel = np.sqrt(diff / norm)
    got_sums = sums.cpu().numpy()
    return rel, margins, got_sums, want_sums


def test_ppo_output_gradient_small_batch(cuda):
    """The fused objective on raw logits (K = 256 slots, ~30 % legal, the all-masked fallback on 100
    rows) against float64: relative norm <= 1e-5 (north_star's fp32 bound)."""
    import torch
    from t8b.policy import ppo_output_gradient, ppo_config
    rng = np.random.default_rng(3)
    n, k = 65536, 256
    logits = rng.normal(size=(n, k + 1)).astype(np.float32)
    masks = (rng.random((n, k)) < 0.3).astype(np.uint8)
    masks[:100] = 0  # the all-masked fallback
    legal = np.where(masks.any(1, keepdims=True), masks, np.eye(1, k, dtype=np.uint8))
    actions = np.array([rng.choice(np.nonzero(m)[0]) for m in legal], np.int64)
    old_lp = rng.normal(scale=0.1, size=n).astype(np.float32) - 3.0
    old_v = rng.normal(size=n).astype(np.float32)
    adv = rng.normal(size=n).astype(np.float32)
    ret = rng.normal(size=n).astype(np.float32)
    d = lambda a: torch.as_tensor(a, device="cuda")
    cfg = ppo_config(entropy_coefficient=0.017)
    inputs = [d(a) for a in (logits, masks, actions, old_lp, old_v, adv, ret)]
    grads, sums = ppo_output_gradient(*inputs, cfg)
    rel, margins, got, want = objective_against_oracle(*inputs, grads, sums, cfg, n)
    assert rel[0] <= 1e-5 and rel[1] <= 1e-5, (rel, margins)
    assert margins <= 4, margins
    for index in (0, 1, 2, 3, 7):
        assert abs(got[index] - want[index]) <= 1e-5 * abs(want[index]), (index, got[index], want[index])
    assert abs(got[4] - want[4]) <= margins and got[6] == want[6]
    assert np.all(grads.cpu().numpy()[np.arange(100), 1:k] == 0.0)


def test_gae_and_objective_full_config2_rollout(cuda):
    """BASELINE config 2 at full size: T = 128 x N = 32,768 (4,194,304 samples), K = 256 slots,
    seed 1 (t8b.workloads.config2_rollout). GAE against float64 within the reference test's 2e-5
    (tests/rollout_tests.cpp:75-93), its normalisation within 1e-5, then the fp32 objective over all
    4.19 M samples with the normalised advantages against the float64 C restatement: relative norm
    of the logit and of the value gradient <= 1e-5 (north_star's fp32 bound), metric sums within
    1e-5. Samples within 1e-5 of a gradient discontinuity are left out of the norms (a float32 and
    a float64 evaluation may take different branches there); they are fewer than 1 in 10,000."""
    import torch
    from t8b.policy import GpuRolloutBuffer, ppo_config, ppo_output_gradient
    from t8b.workloads import config2_rollout
    w = config2_rollout()
    buf = GpuRolloutBuffer(w.envs, w.horizon)
    for name, src in (("rewards", w.rewards), ("old_values", w.values), ("next_values", w.next_values),
                      ("terminated", w.terminated), ("truncated", w.truncated)):
        buf.tensor(name).copy_(src)
    buf.compute_gae(0.99, 0.95, normalize=False)
    host = lambda t: t.cpu().numpy()
    want_adv, want_ret = R.gae(host(w.rewards), host(w.values), host(w.terminated), host(w.truncated),
                               host(w.next_values), 0.99, 0.95)
    assert np.abs(host(buf.tensor("advantages")) - want_adv).max() < 2e-5
    assert np.abs(host(buf.tensor("returns")) - want_ret).max() < 2e-5
    buf.compute_gae(0.99, 0.95, normalize=True)
    adv = buf.tensor("advantages").reshape(-1)
    ret = buf.tensor("returns").reshape(-1)
    norm_want = R.normalize_advantages(want_adv).reshape(-1)
    assert np.linalg.norm(host(adv) - norm_want) <= 1e-5 * np.linalg.norm(norm_want)
    cfg = ppo_config(entropy_coefficient=0.01)
    inputs = (w.outputs, w.masks, w.actions, w.old_log_probabilities, w.values.reshape(-1), adv, ret)
    grads, sums = ppo_output_gradient(*inputs, cfg)
    torch.cuda.synchronize()
    rel, margins, got, want = objective_against_oracle(*inputs, grads, sums, cfg, w.samples)
    assert rel[0] <= 1e-5 and rel[1] <= 1e-5, (rel, margins)
    assert margins <= 1e-4 * w.samples, margins
    # the policy-loss terms have both signs and their sum cancels: its mean is held to 1e-6
    assert abs(got[0] - want[0]) <= 1e-6 * w.samples, (got[0], want[0])
    for index in (1, 2, 3, 7):
        assert abs(got[index] - want[index]) <= 1e-5 * abs(want[index]), (index, got[index], want[index])
    assert abs(got[4] - want[4]) <= margins and got[6] == want[6]


def test_tensor_core_scorer_with_fewer_candidates(cuda, features):
    """The tensor-core scorer (32 features) at 200 candidates instead of 368: the table image's
    rows past the table are zero and the mask words past the candidates are empty. Forward logits
    and argmax actions against float64, and one update's output-layer gradient rows and metrics
    against the float64 objective on the GPU's own network outputs."""
    import torch
    from t8b.policy import GpuActorCritic, actor_config, ppo_config
    k, n = 200, 4096
    rng = np.random.default_rng(21)
    table = np.ascontiguousarray(features[:, :k, :])
    policy = GpuActorCritic(n, actor_config(action_count=k), seed=13)
    policy.set_action_feature_tables(table)
    shapes, p = oracle_params(policy)
    p["w_out"] *= 30.0
    policy.set_parameters(R.flatten(p, shapes).astype(np.float32))
    obs, tables, _ = make_batch(n, table.shape[0], rng)
    masks = (rng.random((n, k)) < 0.3).astype(np.uint8)
    masks[:, 0] = 1
    d = lambda a: torch.as_tensor(a, device="cuda")
    out = policy.forward(d(obs), d(masks), n, seed=3, step=1, deterministic=True, tables=d(tables), want_logits=True)
    got = policy.outputs(n).astype(np.float64)
    logits = R.parametric_scores(got[:, :32], table.astype(np.float64), tables)
    assert np.allclose(out["logits"].cpu().numpy(), logits, atol=1e-5, rtol=1e-4)
    _, prob, legal = R.log_softmax_masked(logits, masks)
    assert np.array_equal(out["actions"].cpu().numpy(), np.argmax(np.where(legal, logits, -np.inf), axis=1))
    # one update on these samples
    sampled = policy.forward(d(obs), d(masks), n, seed=1, step=0, tables=d(tables))
    actions = sampled["actions"].cpu().numpy()
    old_lp = sampled["log_probabilities"].cpu().numpy() - rng.normal(scale=0.05, size=n).astype(np.float32)
    old_v = sampled["values"].cpu().numpy()
    adv = rng.normal(size=n).astype(np.float32)
    ret = (old_v + rng.normal(scale=0.5, size=n)).astype(np.float32)
    view, keep = view_of((obs, tables, masks, actions, old_lp, old_v, adv, ret))
    cfg = ppo_config(epochs=1, minibatch_size=n, learning_rate=1e-3, target_kl=0.0, entropy_coefficient=0.01)
    metrics = policy.update_ppo(view, cfg, shuffle_seed=5)
    order, _ = gathered_order(policy, obs, n)
    dg = policy.activation(3, 0, n)[:, :33].astype(np.float64)
    o = policy.outputs(n).astype(np.float64)
    lg = R.parametric_scores(o[:, :32], table.astype(np.float64), tables[order])
    g, dv, m = R.objective_gradient(lg, masks[order], actions[order], old_lp[order], old_v[order], adv[order],
                                    ret[order], o[:, 32], 0.2, 0.2, 0.5, 0.01, n)
    want_dout = np.concatenate([R.query_gradient(g, table.astype(np.float64), tables[order]), dv[:, None]], 1)
    assert relative(dg, want_dout) < 1e-2
    for key, name in (("policy_loss", "policy_loss"), ("value_loss", "value_loss"), ("entropy", "entropy"),
                      ("approximate_kl", "kl"), ("decision_fraction", "decision")):
        assert abs(metrics[key] - m[name].mean()) <= 1e-4 * max(1.0, abs(m[name].mean())), key


@pytest.mark.parametrize("n,observation_size,feature_size,normalize",
                         [(1000, 151, 32, True), (32768, 151, 32, False), (300, 128, 48, True), (700, 300, 32, True)])
def test_fused_forward_matches_layer_gemms(cuda, features, n, observation_size, feature_size, normalize):
    """The inference forward as one kernel (k_forward_tc: the normalised bf16 operand, both tanh
    layers and the output layer, the activations kept in shared memory) gives network outputs
    bit-identical to k_prep and the separate layer GEMMs (the path of the update and of
    t8b_policy_debug_network): full-move and config-3 shapes, ragged batches (a partial last tile,
    one or several tiles per CTA), with and without the observation normaliser, and a 300-float
    observation (a 320-column operand: the kernel loads the rows directly instead of staging them)."""
    import ctypes as C
    import torch
    from t8b._lib import call
    from t8b.policy import GpuActorCritic, actor_config
    rng = np.random.default_rng(n + observation_size)
    if feature_size == 32:
        table, config = features, actor_config(observation_size=observation_size)
    else:
        table = rng.normal(size=(8, 256, feature_size)).astype(np.float32)
        config = actor_config(observation_size=observation_size, action_count=256, action_feature_size=feature_size)
    policy = GpuActorCritic(n, config, seed=9)
    policy.set_action_feature_tables(table)
    shapes, p = oracle_params(policy)
    p = {key: value + rng.normal(scale=0.05, size=value.shape) for key, value in p.items()}  # non-zero biases
    policy.set_parameters(R.flatten(p, shapes).astype(np.float32))
    if normalize:
        policy.set_observation_statistics(rng.normal(size=observation_size), rng.random(observation_size) + 0.1, 1000)
    obs = torch.as_tensor(rng.normal(scale=2.0, size=(n, observation_size)).astype(np.float32), device="cuda")
    tables = torch.as_tensor(rng.integers(0, table.shape[0], n).astype(np.int32), device="cuda")
    masks = torch.as_tensor((rng.random((n, table.shape[1])) < 0.3).astype(np.uint8), device="cuda")
    masks[:, 0] = 1
    policy.forward(obs, masks, n, seed=1, step=0, tables=tables)
    fused = policy.outputs(n)
    layered = torch.empty((n, feature_size + 1), device="cuda")
    call("t8b_policy_debug_network", policy._handle, C.c_void_p(obs.data_ptr()), n, None,
         C.c_void_p(layered.data_ptr()), None)
    torch.cuda.synchronize()
    assert np.isfinite(fused).all() and np.abs(fused).max() > 0
    assert np.array_equal(fused, layered.cpu().numpy())


@pytest.mark.parametrize("n", [1000, 300])
def test_network_backward_ragged_rows(cuda, features, n):
    """The layer GEMMs' backward at batch sizes that leave a partial last row tile: the
    tanh-gradient epilogue's TMA stores are clipped at the last row, and skipped for a warp whose
    rows all lie past it. Weight and bias gradients of t8b_policy_debug_network (forward, then
    backward from random output gradients) against float64, within north_star's 2e-2 per tensor
    for bf16 GEMMs."""
    import ctypes as C
    import torch
    from t8b._lib import call
    from t8b.policy import GpuActorCritic
    rng = np.random.default_rng(n)
    policy = GpuActorCritic(n, seed=5)
    policy.set_action_feature_tables(features)
    shapes, p = oracle_params(policy)
    p = {key: value + rng.normal(scale=0.05, size=value.shape) for key, value in p.items()}
    flat = R.flatten(p, shapes).astype(np.float32)
    policy.set_parameters(flat)
    params = R.unflatten(flat.astype(np.float64), shapes)
    obs = rng.normal(size=(n, 151)).astype(np.float32)
    dout = rng.normal(size=(n, 33)).astype(np.float32)
    tobs = torch.as_tensor(obs, device="cuda")
    tdout = torch.as_tensor(dout, device="cuda")
    call("t8b_policy_debug_network", policy._handle, C.c_void_p(tobs.data_ptr()), n, C.c_void_p(tdout.data_ptr()),
         None, None)
    torch.cuda.synchronize()
    got = R.unflatten(policy.gradients().astype(np.float64), shapes)
    x = obs.astype(np.float64)
    hs, _ = R.forward(x, params, 2)
    want = R.backward(x, hs, params, dout.astype(np.float64), 2)
    errors = {name: relative(got[name], want[name]) for name, _ in shapes}
    print(f"backward at {n} rows vs float64: {errors}")
    assert all(e < 2e-2 for e in errors.values()), errors
