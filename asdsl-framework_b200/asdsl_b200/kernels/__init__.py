"""B200 (sm_100a) kernel interfaces, mirroring the reference's ``asdsl.kernels``
public surface for the 4-bit decode path (asdsl/kernels/__init__.py:19-44)."""

KERNEL_TIER = "SM100A"

from asdsl_b200.kernels.gemv_q4 import (  # noqa: E402
    gemv_q4,
    gemv_q4_packed,
    gemv_q4_unpacked,
    gemv_q4km_q8,
    has_native_kernel,
)
from asdsl_b200.kernels.gemv_q2 import gemv_q2_packed, gemv_q2_unpacked  # noqa: E402

__all__ = [
    "KERNEL_TIER",
    "gemv_q4",
    "gemv_q4_packed",
    "gemv_q4_unpacked",
    "gemv_q4km_q8",
    "gemv_q2_packed",
    "gemv_q2_unpacked",
    "has_native_kernel",
]
