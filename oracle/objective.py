"""Test infrastructure (not product code): ctypes access to oracle/_ref/libt8oracle.so, the
float64 C restatement of the reference's PPO output-gradient kernel (src/ppo.cu:453-565) in
oracle/objective.c. It needs no reference sources, so it is built wherever the tests run."""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libt8oracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "objective.c").stat().st_mtime:
            build()
        h = C.CDLL(str(LIB))
        vp = C.c_void_p
        h.t8or_objective.argtypes = [vp] * 7 + [C.c_size_t, C.c_int, C.c_double, C.c_float, C.c_float, C.c_float,
                                                C.c_float, C.c_double, vp, vp, vp, C.c_int]
        _lib = h
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def objective(outputs, masks, actions, old_lp, old_v, adv, ret, batch: float, clip=0.2, value_clip=0.2,
              value_coef=0.5, entropy_coef=0.01, tolerance=1e-5, threads: int | None = None):
    """float64 gradient [n][k + 1] of the batch-mean clipped PPO objective w.r.t. raw outputs
    (k logits, then the value), the per-sample branch-margin flags and the metric sums."""
    outputs = np.ascontiguousarray(outputs, np.float32)
    masks = np.ascontiguousarray(masks, np.uint8)
    n, width = outputs.shape
    k = width - 1
    arrays = [np.ascontiguousarray(a, t) for a, t in ((actions, np.int64), (old_lp, np.float32), (old_v, np.float32),
                                                       (adv, np.float32), (ret, np.float32))]
    grads = np.empty((n, width), np.float64)
    margin = np.empty(n, np.uint8)
    sums = np.zeros(8, np.float64)
    status = lib().t8or_objective(_p(outputs), _p(masks), *[_p(a) for a in arrays], n, k, float(batch), clip,
                                  value_clip, value_coef, entropy_coef, tolerance, _p(grads), _p(margin), _p(sums),
                                  threads or os.cpu_count() or 1)
    if status != 0:
        raise RuntimeError("t8or_objective failed")
    return grads, margin.astype(bool), sums
