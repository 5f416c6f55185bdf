"""The allocation-free PPO objective (t8b_ppo_output_gradient_static) against the allocating
entry point (t8b_ppo_output_gradient), called through the C ABI twice in a row.

It exists for callers that cannot call cudaMalloc: a host whose memory manager owns the whole
GPU, or a step that must not pay cudaMalloc/cudaFree's device synchronisation. Its scratch is a
static device array shared by every call; this file runs last so a failure here never hides the
result of another test."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def batch(n, k, seed):
    import torch
    rng = np.random.default_rng(seed)
    logits = rng.normal(size=(n, k + 1)).astype(np.float32)
    masks = (rng.random((n, k)) < 0.3).astype(np.uint8)
    masks[:, 0] = 1
    actions = np.array([rng.choice(np.nonzero(m)[0]) for m in masks], np.int64)
    arrays = [logits, masks, actions] + [rng.normal(size=n).astype(np.float32) for _ in range(4)]
    return [torch.as_tensor(a, device="cuda") for a in arrays]


def call(name, tensors, k, config, metrics):
    import torch
    from t8b import _lib
    n = tensors[0].shape[0]
    grads = torch.full((n, k + 1), float("nan"), device="cuda")
    sums = torch.full((8,), float("nan"), dtype=torch.float64, device="cuda")
    status = getattr(_lib.lib(), name)(*[t.data_ptr() for t in tensors], n, k, C.byref(config), grads.data_ptr(),
                                        sums.data_ptr() if metrics else None, None)
    assert status == 0, _lib.lib().t8b_last_error()
    torch.cuda.synchronize()
    return grads, sums


def test_static_scratch_objective_matches_allocating_entry_point(cuda):
    import torch
    from t8b.policy import ppo_config
    config = ppo_config(entropy_coefficient=0.02)
    k = 256
    for repeat, n in enumerate((200_000, 65_536)):  # two calls in a row share the static scratch
        tensors = batch(n, k, seed=repeat)
        want_g, want_s = call("t8b_ppo_output_gradient", tensors, k, config, True)
        got_g, got_s = call("t8b_ppo_output_gradient_static", tensors, k, config, True)
        assert torch.allclose(got_g, want_g, rtol=1e-6, atol=0.0)
        assert torch.allclose(got_s, want_s, rtol=1e-12, atol=0.0)
        assert torch.isfinite(got_g).all()


def test_static_entry_point_allocates_nothing(cuda):
    """After a first call (which looks the array up and loads the kernel), further calls leave the
    device's free memory unchanged; without metric sums the gradients are unchanged too."""
    import torch
    from t8b.policy import ppo_config
    config = ppo_config()
    k = 256
    tensors = batch(131_072, k, seed=7)
    want_g, _ = call("t8b_ppo_output_gradient", tensors, k, config, True)
    call("t8b_ppo_output_gradient_static", tensors, k, config, True)
    grads = torch.empty_like(want_g)
    sums = torch.empty(8, dtype=torch.float64, device="cuda")
    from t8b import _lib
    lib = _lib.lib()
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for metrics in (True, False, True):
        status = lib.t8b_ppo_output_gradient_static(*[t.data_ptr() for t in tensors], tensors[0].shape[0], k,
                                                    C.byref(config), grads.data_ptr(),
                                                    sums.data_ptr() if metrics else None, None)
        assert status == 0, lib.t8b_last_error()
        torch.cuda.synchronize()
        assert torch.allclose(grads, want_g, rtol=1e-6, atol=0.0)
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_static_entry_point_rejects_sizes_beyond_its_scratch(cuda):
    import torch
    from t8b import _lib
    from t8b.policy import ppo_config
    n = 524_289
    config = ppo_config()
    dummy = torch.zeros(1, device="cuda")
    status = _lib.lib().t8b_ppo_output_gradient_static(*([dummy.data_ptr()] * 7), n, 256, C.byref(config),
                                                      dummy.data_ptr(), None, None)
    assert status == _lib.T8B_EINVAL
    assert b"524288" in _lib.lib().t8b_last_error()
