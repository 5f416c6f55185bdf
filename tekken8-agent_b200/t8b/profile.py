"""Launch accounting of the library: how many kernels it launched, and per-kernel device time
from CUDA events around each launch (t8b_launch_count / t8b_profile_enable /
t8b_profile_report in t8b.h)."""
from __future__ import annotations

import ctypes as C

from ._lib import lib


def launch_count() -> int:
    """Kernels the library has launched since it was loaded."""
    return int(lib().t8b_launch_count())


def enable(on: bool = True) -> None:
    """Starts (clearing earlier results) or stops per-launch event timing."""
    lib().t8b_profile_enable(1 if on else 0)


def only(label: str | None) -> None:
    """Brackets only the launches labelled `label` (None: every launch)."""
    lib().t8b_profile_only(None if label is None else label.encode())


def report() -> dict[str, tuple[int, float]]:
    """Synchronises the device and returns {label: (launches, total device ms)}."""
    need = lib().t8b_profile_report(None, 0)
    buf = C.create_string_buffer(need)
    lib().t8b_profile_report(buf, need)
    out = {}
    for line in buf.value.decode().splitlines():
        label, launches, ms = line.rsplit(" ", 2)
        out[label] = (int(launches), float(ms))
    return out
