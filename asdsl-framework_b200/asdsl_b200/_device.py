"""Device-memory plumbing for the Python API (torch is used for HBM buffers and
streams only; all arithmetic runs in libasdsl_b200.so).

Inputs may be numpy arrays (host; copied to the device for the call, results
copied back) or torch CUDA tensors (used in place, work enqueued on torch's
current stream, no synchronization).
"""

from __future__ import annotations

import numpy as np
import torch

_NP2T = {
    np.dtype(np.uint8): torch.uint8,
    np.dtype(np.int8): torch.int8,
    np.dtype(np.float32): torch.float32,
    np.dtype(np.float16): torch.float16,
    np.dtype(np.int32): torch.int32,
    np.dtype(np.uint16): torch.int16,
}


def require_cuda() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("asdsl_b200 needs a CUDA device (sm_100a); none is available")
    return torch.device("cuda", torch.cuda.current_device())


def is_cuda_tensor(a) -> bool:
    return isinstance(a, torch.Tensor) and a.is_cuda


def to_device(a, dtype: np.dtype | None = None) -> torch.Tensor:
    """Return a contiguous, 16-byte aligned CUDA tensor holding `a`'s bytes."""
    if isinstance(a, torch.Tensor):
        t = a
        if dtype is not None and _NP2T[np.dtype(dtype)] != t.dtype:
            t = t.to(_NP2T[np.dtype(dtype)])
        if not t.is_cuda:
            t = t.to(require_cuda())
        if not t.is_contiguous() or (t.data_ptr() & 15):
            t = t.contiguous().clone()
        return t
    arr = np.asarray(a)
    if dtype is not None and arr.dtype != np.dtype(dtype):
        arr = arr.astype(dtype)
    arr = np.ascontiguousarray(arr)
    if arr.dtype == np.uint16:
        arr = arr.view(np.int16)
    return torch.from_numpy(arr).to(require_cuda(), non_blocking=False)


def empty(n, dtype, like=None) -> torch.Tensor:
    return torch.empty(n, dtype=_NP2T[np.dtype(dtype)], device=require_cuda())


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr() -> int | None:
    return torch.cuda.current_stream().cuda_stream or None


def to_host(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()
