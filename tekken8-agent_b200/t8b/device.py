"""Zero-copy torch views of device pointers owned by the library (torch is plumbing only)."""
from __future__ import annotations

import torch

_TYPESTR = {torch.float32: "<f4", torch.float64: "<f8", torch.uint8: "|u1", torch.int8: "|i1",
            torch.int32: "<i4", torch.int64: "<i8", torch.uint32: "<u4"}


class _Interface:
    def __init__(self, pointer: int, shape, dtype: torch.dtype):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": _TYPESTR[dtype],
                                         "data": (int(pointer), False), "version": 3, "strides": None}


def view(pointer, shape, dtype: torch.dtype, device: int = 0) -> torch.Tensor:
    """A tensor aliasing `pointer` (valid until the owning object's next mutating call)."""
    if not pointer:
        raise RuntimeError("null device view")
    return torch.as_tensor(_Interface(pointer, shape, dtype), device=f"cuda:{device}")


def ptr(tensor) -> int:
    if tensor is None:
        return 0
    if not tensor.is_cuda or not tensor.is_contiguous():
        raise ValueError("expected a contiguous CUDA tensor")
    return tensor.data_ptr()
