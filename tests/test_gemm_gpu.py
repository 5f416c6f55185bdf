"""The tcgen05 GEMM against a plain PyTorch fp32 reference of the same product (bf16 inputs,
fp32 accumulation): every tile width and operand major the policy uses, split-K included.
Tolerance: 1e-3 relative to the largest magnitude (fp32 accumulation order only)."""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu

CASES = [  # (bn, a_mn, b_mn, m, n, k, splits)
    (256, 0, 0, 1024, 512, 192, 1),
    (256, 0, 0, 640, 512, 512, 1),
    (64, 0, 0, 1024, 64, 512, 1),
    (256, 0, 0, 512, 512, 64, 1),
    (192, 0, 0, 512, 192, 1024, 1),
    (256, 1, 1, 512, 512, 4096, 8),
    (192, 1, 1, 512, 192, 4096, 5),
    (64, 1, 1, 512, 64, 4096, 37),
    (256, 1, 0, 256, 512, 1024, 1),
]


@pytest.mark.parametrize("bn,a_mn,b_mn,m,n,k,splits", CASES)
def test_gemm_matches_torch(cuda, bn, a_mn, b_mn, m, n, k, splits):
    import torch
    from t8b import _lib
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    a_store = a.t().contiguous() if a_mn else a
    b_store = b.t().contiguous() if b_mn else b
    c = torch.full((m, n), float("nan"), device="cuda")
    lib = _lib.lib()
    lib.t8b_debug_gemm.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p] + [C.c_int] * 5 + [C.c_void_p]
    status = lib.t8b_debug_gemm(a_store.data_ptr(), a_mn, b_store.data_ptr(), b_mn, c.data_ptr(), m, n, k, bn, splits, None)
    assert status == 0, lib.t8b_last_error()
    torch.cuda.synchronize()
    want = a.float() @ b.float().t()
    err = (c - want).abs().max().item() / want.abs().max().item()
    assert err < 1e-3, err


def test_bounded_wait_gives_up_and_reports(cuda):
    """The mbarrier wait the GEMM uses is bounded: a barrier that nothing arrives at makes the
    wait run out and report it (the kernel returns, the context stays usable); an arrived
    barrier is seen."""
    import ctypes as C
    import torch
    from t8b import _lib
    flag = C.c_int(-1)
    _lib.call("t8b_debug_bounded_wait", 0, 1 << 16, C.byref(flag))
    assert flag.value == 1
    _lib.call("t8b_debug_bounded_wait", 1, 1 << 16, C.byref(flag))
    assert flag.value == 0
    assert torch.ones(4, device="cuda").sum().item() == 4.0
