"""2-bit fp32-activation GEMVs of the QCSD draft bank, mirroring the reference's
``asdsl.kernels.gemv_q2`` (asdsl/kernels/gemv_q2.py:95-171) over ``_native_gemv_q2``
(asdsl/kernels/native/gemv_q2_avx2.cpp:300-372): numpy in, numpy out (CUDA tensors in, a CUDA
tensor out), run by the sm_100a kernels of ``asdsl_b200_gemv_q2_{packed,unpacked}``."""

from __future__ import annotations

import numpy as np

from asdsl_b200 import _device as dv
from asdsl_b200 import _lib


def _numel(a) -> int:
    return a.numel() if hasattr(a, "numel") else np.asarray(a).size


def _q2(packed: bool, w, x, scales, biases, M: int, K: int, group_size: int):
    if M <= 0 or K <= 0 or group_size <= 0:
        raise ValueError("M, K, group_size must be positive")
    if packed and K % 4:
        raise ValueError("K must be divisible by 4 for 2-bit packing")
    if K % group_size:
        raise ValueError("K must be divisible by group_size")
    if _numel(x) != K:
        raise ValueError("x length must equal K")
    if _numel(w) != M * (K // 4 if packed else K):
        raise ValueError("weight buffer size mismatch")
    ng = M * (K // group_size)
    if _numel(scales) != ng or _numel(biases) != ng:
        raise ValueError("scales/biases size mismatch")
    wd, xd = dv.to_device(w, np.uint8), dv.to_device(x, np.float32)
    s, b = dv.to_device(scales, np.float32), dv.to_device(biases, np.float32)
    yd = dv.empty(M, np.float32)
    _lib.call("asdsl_b200_gemv_q2_packed" if packed else "asdsl_b200_gemv_q2_unpacked", wd.data_ptr(),
              xd.data_ptr(), s.data_ptr(), b.data_ptr(), yd.data_ptr(), int(M), int(K), int(group_size),
              dv.stream_ptr())
    return yd if dv.is_cuda_tensor(x) else dv.to_host(yd)


def gemv_q2_unpacked(w, x, scales, biases, M: int, K: int, group_size: int):
    """Fused 2-bit GEMV on one-code-per-byte weights (gemv_q2.py:95-117)."""
    return _q2(False, w, x, scales, biases, M, K, group_size)


def gemv_q2_packed(w_packed, x, scales, biases, M: int, K: int, group_size: int):
    """Fused 2-bit GEMV on packed weights, four codes per byte (gemv_q2.py:120-171)."""
    return _q2(True, w_packed, x, scales, biases, M, K, group_size)
