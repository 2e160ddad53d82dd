"""Fused 4-bit GEMV, y = dequant(W_q4) @ x, on the B200 kernels.

Mirrors the reference's public API in asdsl/kernels/gemv_q4.py:215-416
(same names, arguments, validation messages and return conventions).  There is
no NumPy fallback: without the CUDA library these raise RuntimeError.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

import numpy as np

from asdsl_b200 import _lib
from asdsl_b200.kernels import _native_gemv as _native

if TYPE_CHECKING:
    from asdsl_b200.quantization.core import QuantizedTensor


def has_native_kernel() -> bool:
    """True when libasdsl_b200.so loads and a CUDA device is present."""
    try:
        _lib.load()
    except (RuntimeError, OSError):
        return False
    import torch

    return torch.cuda.is_available()


def _ndim(a) -> int:
    return a.ndim if hasattr(a, "ndim") else np.asarray(a).ndim


def _shape(a):
    return tuple(a.shape) if hasattr(a, "shape") else np.asarray(a).shape


def gemv_q4_packed(w_packed, x, scales, biases, M: int, K: int, group_size: int, out=None,
                   use_lut: bool = False, use_q8: bool = False, lut_cache=None, bits: int = 4):
    """Fused 4-bit packed GEMV (asdsl/kernels/gemv_q4.py:215-324).

    x is (K,) or (B, K); returns (M,) or (B, M).  ``use_lut`` / ``lut_cache`` /
    ``bits`` select CPU table paths in the reference and do not change the result
    here; ``use_q8`` is accepted for signature compatibility (the reference's Q8
    variant is a different numeric path, asdsl/kernels/gemv_q4.py:270-276).
    """
    del use_lut, lut_cache, bits, use_q8
    if out is not None and (_shape(out)[0] != M or str(getattr(out, "dtype", "")) not in ("float32", "torch.float32")):
        raise ValueError(f"out must be float32 shape ({M},), got {_shape(out)} {getattr(out, 'dtype', None)}")
    nd = _ndim(x)
    if nd == 1:
        if _shape(x)[0] != K:
            raise ValueError(f"x length {_shape(x)[0]} does not match K={K}")
    elif nd == 2:
        if _shape(x)[1] != K:
            raise ValueError(f"x.shape[1]={_shape(x)[1]} does not match K={K}")
    else:
        raise ValueError("x must be 1-D (K,) or 2-D (batch, K)")
    if not has_native_kernel():
        raise RuntimeError("asdsl_b200 CUDA kernels are unavailable (library not built or no GPU)")
    y = _native.gemv_q4_packed(w_packed, x, scales, biases, M, K, group_size)
    if out is not None and nd == 1:
        return _native.gemv_q4_packed_into(w_packed, x, scales, biases, out, M, K, group_size)
    return y


def gemv_q4_unpacked(w, x, scales, biases, M: int, K: int, group_size: int):
    """Fused GEMV on one-code-per-byte weights (asdsl/kernels/gemv_q4.py:327-363)."""
    if not has_native_kernel():
        raise RuntimeError("asdsl_b200 CUDA kernels are unavailable (library not built or no GPU)")
    return _native.gemv_q4_unpacked(w, x, scales, biases, M, K, group_size)


def gemv_q4km_q8(weights_q4km, x, out_features: int, in_features: int):
    """Q4_K super-block GEMV with the kernel's own A8 (asdsl/kernels/gemv_q4.py:366-384)."""
    if not has_native_kernel():
        raise RuntimeError("Native Q4_K_M GEMV is unavailable in this build")
    import torch

    xsz = x.numel() if isinstance(x, torch.Tensor) else np.asarray(x).size
    if xsz != in_features:
        raise ValueError(f"x length {xsz} does not match in_features={in_features}")
    w = weights_q4km.reshape(-1)
    xv = x.reshape(-1)
    if isinstance(x, torch.Tensor) and x.is_cuda:
        y = torch.zeros(out_features, dtype=torch.float32, device=x.device)
    else:
        y = np.zeros(out_features, dtype=np.float32)
    _native.gemv_q4km_q8_avx2(w, xv, y, out_features, in_features)
    return y


def gemv_q4(qtensor: "QuantizedTensor", x):
    """GEMV from a QuantizedTensor (asdsl/kernels/gemv_q4.py:386-416): bias = -zero*scale
    (asymmetric) or -7.5*scale (symmetric)."""
    if qtensor.bits != 4:
        raise ValueError(f"gemv_q4 only supports 4-bit tensors, got {qtensor.bits}-bit")
    M, K = qtensor.shape
    gs = qtensor.group_size
    scales = qtensor.scales.astype(np.float32)
    if qtensor.is_symmetric:
        biases = np.full_like(scales, -7.5) * scales
    else:
        zeros = qtensor.zeros.astype(np.float32)
        biases = -zeros * scales
    return gemv_q4_packed(qtensor.data, x, scales, biases, M, K, gs)
