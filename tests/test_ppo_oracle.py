"""Pins the numpy PPO oracle (oracle/ppo_ref.py) on the CPU: the reference's own known-answer
test for the objective gradient (tests/ppo_math_tests.cpp:73-128, tolerance 2e-3 against central
finite differences, masked actions exactly zero, the all-masked fallback finite), the scorer
and MLP backward against finite differences, and GAE against the reference test's scalar loop."""
import numpy as np

from oracle import ppo_ref as R

CLIP, VCLIP, VCOEF, ECOEF = 0.2, 0.2, 0.5, 0.017


def reference_case():
    output = np.array([-0.20, 0.12, -0.04, 0.31, 0.08, -0.11, 0.15], np.float32)
    mask = np.array([1, 1, 0, 1, 1, 1], np.uint8)
    selected = 3
    legal = mask.astype(bool)
    maximum = float(np.max(output[:6][legal]))
    total = float(np.sum(np.exp(output[:6][legal].astype(np.float64) - maximum)))
    old_lp = np.float32(output[selected] - (np.log(total) + maximum) - 0.03)
    return output, mask, selected, float(old_lp), 0.10, 0.70, 0.35


def test_objective_gradient_matches_finite_differences_on_the_reference_vector():
    output, mask, sel, old_lp, old_v, adv, ret = reference_case()
    logits = output[None, :6].astype(np.float64)
    g, dv, _ = R.objective_gradient(logits, mask[None], np.array([sel]), np.array([old_lp]), np.array([old_v]),
                                    np.array([adv]), np.array([ret]), np.array([output[6]], np.float64), CLIP, VCLIP,
                                    VCOEF, ECOEF, 1.0)
    grad = np.concatenate([g[0], dv])
    eps = np.float32(1e-3)
    for i in range(7):
        plus, minus = output.copy(), output.copy()
        plus[i] += eps
        minus[i] -= eps
        num = (R.objective(plus, mask, sel, old_lp, old_v, adv, ret, CLIP, VCLIP, VCOEF, ECOEF) -
               R.objective(minus, mask, sel, old_lp, old_v, adv, ret, CLIP, VCLIP, VCOEF, ECOEF)) / (2.0 * float(eps))
        assert abs(grad[i] - num) < 2e-3, (i, grad[i], num)
    assert grad[2] == 0.0


def test_all_masked_fallback_is_finite():
    output, _, _, _, old_v, adv, ret = reference_case()
    g, dv, _ = R.objective_gradient(output[None, :6].astype(np.float64), np.zeros((1, 6), np.uint8), np.array([0]),
                                    np.array([0.0]), np.array([old_v]), np.array([adv]), np.array([ret]),
                                    np.array([output[6]], np.float64), CLIP, VCLIP, VCOEF, ECOEF, 1.0)
    assert np.all(np.isfinite(g)) and np.all(np.isfinite(dv))


def test_query_gradient_matches_finite_differences():
    rng = np.random.default_rng(0)
    features = rng.normal(size=(3, 10, 4))
    tables = np.array([1])
    q = rng.normal(size=(1, 4))
    weights = rng.normal(size=(1, 10))
    f = lambda qq: float((R.parametric_scores(qq, features, tables) * weights).sum())
    analytic = R.query_gradient(weights, features, tables)[0]
    for k in range(4):
        d = np.zeros_like(q)
        d[0, k] = 1e-6
        assert abs((f(q + d) - f(q - d)) / 2e-6 - analytic[k]) < 1e-6


def test_backward_matches_finite_differences():
    rng = np.random.default_rng(1)
    shapes = R.layout(7, 16, 2, 5)
    flat = rng.normal(scale=0.3, size=sum(int(np.prod(s)) for _, s in shapes))
    params = R.unflatten(flat, shapes)
    x = rng.normal(size=(6, 7))
    g_out = rng.normal(size=(6, 5))
    hs, out = R.forward(x, params, 2)
    grads = R.flatten(R.backward(x, hs, params, g_out, 2), shapes)
    f = lambda p: float((R.forward(x, R.unflatten(p, shapes), 2)[1] * g_out).sum())
    for i in rng.choice(flat.size, 40, replace=False):
        d = np.zeros_like(flat)
        d[i] = 1e-6
        num = (f(flat + d) - f(flat - d)) / 2e-6
        assert abs(num - grads[i]) <= 1e-5 * max(1.0, abs(num))


def test_gae_matches_the_reference_scalar_loop():
    rng = np.random.default_rng(2)
    horizon, envs = 64, 48
    rewards = rng.normal(size=(horizon, envs)).astype(np.float32)
    values = rng.normal(size=(horizon, envs)).astype(np.float32)
    nv = rng.normal(size=(horizon, envs)).astype(np.float32)
    term = (rng.random((horizon, envs)) < 0.05).astype(np.uint8)
    trunc = ((rng.random((horizon, envs)) < 0.02) & (term == 1)).astype(np.uint8)
    adv, ret = R.gae(rewards, values, term, trunc, nv, 0.99, 0.95)
    for e in range(envs):
        nxt = np.float32(0)
        for t in range(horizon - 1, -1, -1):
            tl = trunc[t, e] != 0
            bm = np.float32(0 if (term[t, e] and not tl) else 1)
            tm = np.float32(0 if (term[t, e] or tl) else 1)
            delta = rewards[t, e] + np.float32(0.99) * nv[t, e] * bm - values[t, e]
            nxt = delta + np.float32(0.99) * np.float32(0.95) * tm * nxt
            assert abs(adv[t, e] - nxt) < 2e-5
    norm = R.normalize_advantages(adv)
    assert abs(norm.mean()) < 2e-4 and abs(norm.var() - 1) < 2e-3


def test_uniform01_is_the_reference_bit_recipe():
    u = R.uniform01(2028, 7, 3)
    assert 0.0 < u < 1.0 and u.dtype == np.float32


def test_c_objective_equals_the_numpy_restatement():
    """oracle/objective.c (float64, used at full config-2 size) against objective_gradient above on
    a mixed batch: legal sets of every density, the all-masked fallback, clipped and unclipped
    ratios and values."""
    from oracle import objective
    rng = np.random.default_rng(11)
    n, k = 3000, 40
    out = rng.normal(size=(n, k + 1)).astype(np.float32)
    masks = (rng.random((n, k)) < rng.random((n, 1))).astype(np.uint8)
    masks[:20] = 0
    legal = R.legal_set(masks)
    actions = np.array([rng.choice(np.nonzero(m)[0]) for m in legal], np.int64)
    old_lp = (rng.normal(scale=0.3, size=n) - 3.0).astype(np.float32)
    old_v = rng.normal(size=n).astype(np.float32)
    adv = rng.normal(size=n).astype(np.float32)
    ret = rng.normal(size=n).astype(np.float32)
    f32 = lambda v: float(np.float32(v))  # the C oracle takes the float32 config values, as the kernel does
    g, dv, m = R.objective_gradient(out[:, :k].astype(np.float64), masks, actions, old_lp, old_v, adv, ret,
                                    out[:, k].astype(np.float64), f32(CLIP), f32(VCLIP), f32(VCOEF), f32(ECOEF), n)
    got, margin, sums = objective.objective(out, masks, actions, old_lp, old_v, adv, ret, n, CLIP, VCLIP, VCOEF, ECOEF,
                                            threads=3)
    # summation order differs (numpy sums pairwise): equal to float64 rounding of the whole array
    assert np.linalg.norm(got[:, :k] - g) <= 1e-9 * np.linalg.norm(g)
    assert np.linalg.norm(got[:, k] - dv) <= 1e-12 * np.linalg.norm(dv)
    for index, key in enumerate(("policy_loss", "value_loss", "entropy", "kl", "clip")):
        assert abs(sums[index] - m[key].sum()) <= 1e-10 * max(1.0, np.abs(m[key]).sum()), key
    assert sums[6] == m["decision"].sum()
    assert abs(sums[7] - m["decision_entropy"].sum()) <= 1e-10 * m["decision_entropy"].sum()
    assert margin.sum() < n // 100
