"""Host side of the B200-native self-play hot path: ctypes mirrors of the reference's
GpuFullMoveSimulator / GpuActorCritic / GpuRolloutBuffer over the C ABI in include/t8b.h."""
from ._lib import lib, call, T8bError  # noqa: F401
from . import roster  # noqa: F401
