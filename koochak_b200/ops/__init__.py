"""Native sm_100a ops (tcgen05 GEMM, attention, norms, fused losses, optimizer kernels)."""

from ._ext import available, check_status, native  # noqa: F401
