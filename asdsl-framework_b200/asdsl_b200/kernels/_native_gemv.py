"""Drop-in counterpart of the reference's ``asdsl.kernels._native_gemv`` module.

Same function names, argument order, defaults, in-place output convention and
exception classes as the reference's pybind bindings
(asdsl/kernels/native/gemv_q4_avx2.cpp:1162-1506), computed by the sm_100a
kernels of libasdsl_b200.so.  Array arguments may be host numpy arrays (copied
to the device for the call; outputs copied back into the caller's array) or
CUDA torch tensors (used in place on torch's current stream).
"""

from __future__ import annotations

import numpy as np
import torch

from asdsl_b200 import _device as dv
from asdsl_b200 import _lib

has_openmp = False
has_q4km_gemv = True


def _writeback(dst, src_t: torch.Tensor) -> None:
    """Copy a device result into the caller's output (numpy or torch)."""
    if isinstance(dst, torch.Tensor):
        if dst.data_ptr() != src_t.data_ptr():
            dst.copy_(src_t.view_as(dst) if dst.numel() == src_t.numel() else src_t)
        return
    np.copyto(dst.reshape(-1), dv.to_host(src_t).reshape(-1)[: dst.size])


def _out(dst, n: int, dtype) -> torch.Tensor:
    """Device buffer for an output: the caller's tensor when it is usable in place."""
    if dv.is_cuda_tensor(dst) and dst.is_contiguous() and (dst.data_ptr() & 15) == 0 and dst.numel() >= n:
        return dst
    if dst is not None and not isinstance(dst, torch.Tensor):
        if np.asarray(dst).size < n:
            raise ValueError("output buffer too small")
    return dv.empty(n, dtype)


def _check_1d(name: str, a) -> None:
    if a is None:
        raise ValueError(f"{name} must not be None")


# ---------------------------------------------------------------------------
# A8 activation quantization (gemv_q4_preq_restored.cpp:505-549)
# ---------------------------------------------------------------------------
def quantize_activation_avx2(x, x_q8, x_scales, in_features: int, group_size: int = 32) -> None:
    xd = dv.to_device(x, np.float32)
    q = _out(x_q8, in_features, np.int8)
    s = _out(x_scales, in_features // group_size, np.float32)
    _lib.call("asdsl_b200_quantize_activation", xd.data_ptr(), q.data_ptr(), s.data_ptr(), None,
              int(in_features), int(group_size), dv.stream_ptr())
    _writeback(x_q8, q)
    _writeback(x_scales, s)


def gemv_preq2_fused_avx2(meta, quant, x_fp32, y, out_features: int, in_features: int, group_size: int = 32) -> None:
    m, q, xd = dv.to_device(meta, np.uint8), dv.to_device(quant, np.uint8), dv.to_device(x_fp32, np.float32)
    yd = _out(y, out_features, np.float32)
    _lib.call("asdsl_b200_gemv_preq2_fused", m.data_ptr(), q.data_ptr(), xd.data_ptr(), yd.data_ptr(),
              int(out_features), int(in_features), int(group_size), dv.stream_ptr())
    _writeback(y, yd)


def gemv_preq2_avx2(meta, quant, x_q8, x_scales, y, out_features: int, in_features: int, group_size: int = 32) -> None:
    m, q = dv.to_device(meta, np.uint8), dv.to_device(quant, np.uint8)
    xq, xs = dv.to_device(x_q8, np.int8), dv.to_device(x_scales, np.float32)
    yd = _out(y, out_features, np.float32)
    _lib.call("asdsl_b200_gemv_preq2", m.data_ptr(), q.data_ptr(), xq.data_ptr(), xs.data_ptr(), yd.data_ptr(),
              int(out_features), int(in_features), int(group_size), dv.stream_ptr())
    _writeback(y, yd)


def gemv_q4_32_preq_avx2(blocks, x_q8, x_scales, y, out_features: int, in_features: int, group_size: int = 32) -> None:
    b = dv.to_device(blocks, np.uint8)
    xq, xs = dv.to_device(x_q8, np.int8), dv.to_device(x_scales, np.float32)
    yd = _out(y, out_features, np.float32)
    _lib.call("asdsl_b200_gemv_q4_32_preq", b.data_ptr(), xq.data_ptr(), xs.data_ptr(), yd.data_ptr(),
              int(out_features), int(in_features), int(group_size), dv.stream_ptr())
    _writeback(y, yd)


def _preq_fp32(blocks, x_fp32, y, out_features, in_features, group_size) -> None:
    b, xd = dv.to_device(blocks, np.uint8), dv.to_device(x_fp32, np.float32)
    yd = _out(y, out_features, np.float32)
    _lib.call("asdsl_b200_gemv_q4_32_preq_fused", b.data_ptr(), xd.data_ptr(), yd.data_ptr(),
              int(out_features), int(in_features), int(group_size), dv.stream_ptr())
    _writeback(y, yd)


# The reference's 4row / 8row / g4fused / fused entries differ only in CPU
# tiling (gemv_q4_preq_restored.cpp:579-669); on the GPU they are one kernel.
def gemv_q4_32_preq_fused_avx2(blocks, x_fp32, y, out_features: int, in_features: int, group_size: int = 32) -> None:
    _preq_fp32(blocks, x_fp32, y, out_features, in_features, group_size)


def gemv_q4_32_preq_4row_avx2(blocks, x_fp32, y, out_features: int, in_features: int, group_size: int = 32) -> None:
    _preq_fp32(blocks, x_fp32, y, out_features, in_features, group_size)


def gemv_q4_32_preq_8row_avx2(blocks, x_fp32, y, out_features: int, in_features: int, group_size: int = 32) -> None:
    _preq_fp32(blocks, x_fp32, y, out_features, in_features, group_size)


def gemv_q4_32_preq_g4fused_4row_avx2(blocks, x_fp32, y, out_features: int, in_features: int,
                                      group_size: int = 32) -> None:
    if group_size == 32 and in_features > 0 and ((in_features // 32) % 4) != 0:
        raise ValueError("gemv_q4_32_preq_g4fused_4row_avx2: n_groups must be <= 640 and divisible by 4")
    _preq_fp32(blocks, x_fp32, y, out_features, in_features, group_size)


def gemv_q4_128_preq_avx2(blocks, x_q8, x_scales, y, out_features: int, in_features: int,
                          group_size: int = 128) -> None:
    b = dv.to_device(blocks, np.uint8)
    xq, xs = dv.to_device(x_q8, np.int8), dv.to_device(x_scales, np.float32)
    yd = _out(y, out_features, np.float32)
    _lib.call("asdsl_b200_gemv_q4_128", b.data_ptr(), xq.data_ptr(), xs.data_ptr(), yd.data_ptr(),
              int(out_features), int(in_features), int(group_size), dv.stream_ptr())
    _writeback(y, yd)


def gemm_q4_128_q8_avx2(blocks, x_batch, y_batch, out_features: int, in_features: int, group_size: int,
                        batch_size: int) -> None:
    """Batched prompt GEMM on fp32 activations (gemm_q4_128_q8_avx2, gemv_q4_128.cpp:262-306):
    y_batch[b][out] = W . x_batch[b] for b < min(batch_size, 64), bit-identical to the reference;
    rows b >= 64 of y_batch keep their values.  group_size != 128 raises ValueError."""
    if group_size != 128:
        raise ValueError("gemm_q4_128_q8_avx2: group_size must be 128")
    b = dv.to_device(blocks, np.uint8)
    xd = dv.to_device(x_batch, np.float32)
    n = int(batch_size) * int(out_features)
    if dv.is_cuda_tensor(y_batch) and y_batch.is_contiguous() and y_batch.numel() >= n:
        yd = y_batch
    else:
        yd = dv.to_device(y_batch, np.float32)  # rows the GEMM leaves alone keep the caller's values
    _lib.call("asdsl_b200_gemm_q4_128_f32", b.data_ptr(), xd.data_ptr(), yd.data_ptr(), int(out_features),
              int(in_features), int(group_size), int(batch_size), dv.stream_ptr())
    _writeback(y_batch, yd)


def gemv_q4_s256_preq_avx2(blocks, x_q8, x_scales, y, out_features: int, in_features: int,
                           group_size: int = 32) -> None:
    b = dv.to_device(blocks, np.uint8)
    xq, xs = dv.to_device(x_q8, np.int8), dv.to_device(x_scales, np.float32)
    yd = _out(y, out_features, np.float32)
    _lib.call("asdsl_b200_gemv_q4_s256", b.data_ptr(), xq.data_ptr(), xs.data_ptr(), yd.data_ptr(),
              int(out_features), int(in_features), int(group_size), dv.stream_ptr())
    _writeback(y, yd)


def gemv_q4km_q8_avx2(weights_q4km, x, y, out_features: int, in_features: int) -> None:
    """Reference checks (gemv_q4_avx2.cpp:1318-1348): sizes must match exactly."""
    w = weights_q4km if isinstance(weights_q4km, torch.Tensor) else np.asarray(weights_q4km)
    nblocks = (in_features // 256) if in_features > 0 else 0
    if in_features > 0 and out_features > 0:
        wsize = w.numel() if isinstance(w, torch.Tensor) else w.size
        if in_features % 256 == 0 and wsize != out_features * nblocks * 144:
            raise ValueError("Q4_K_M weight size mismatch")
        xsize = x.numel() if isinstance(x, torch.Tensor) else np.asarray(x).size
        ysize = y.numel() if isinstance(y, torch.Tensor) else np.asarray(y).size
        if xsize != in_features or ysize != out_features:
            raise ValueError("x/y size mismatch for out_features/in_features")
    wd, xd = dv.to_device(w, np.uint8), dv.to_device(x, np.float32)
    yd = _out(y, max(out_features, 1), np.float32)
    _lib.call("asdsl_b200_gemv_q4km", wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), int(out_features),
              int(in_features), dv.stream_ptr())
    if out_features > 0 and in_features > 0:
        _writeback(y, yd)


def gemv_multi(fmt: int, w0, w1, X, Y, out_features: int, in_features: int) -> None:
    """Multi-token W4A8 GEMV (speculative verification): Y[t] = W . A8(X[t]) for every row t of
    X (n_tokens, in_features); one weight stream serves up to 16 rows.  Row t equals the
    single-token kernel's result (gemv_q4_32_preq_fused_avx2 / gemv_preq2_fused_avx2 /
    gemv_q4km_q8_avx2 on X[t]); fmt is one of _lib.FMT_PREQ, FMT_PREQ2, FMT_Q4_128_BANDED, FMT_Q4K."""
    xt = X if isinstance(X, torch.Tensor) else np.asarray(X)
    if xt.ndim != 2 or int(xt.shape[1]) != in_features:
        raise ValueError("X must be (n_tokens, in_features)")
    n = int(xt.shape[0])
    ysize = Y.numel() if isinstance(Y, torch.Tensor) else np.asarray(Y).size
    if ysize != n * out_features:
        raise ValueError("Y must hold n_tokens * out_features values")
    w0d = dv.to_device(w0, np.uint8)
    w1d = dv.to_device(w1, np.uint8) if w1 is not None else None
    xd = dv.to_device(xt, np.float32)
    yd = _out(Y, n * out_features, np.float32)
    _lib.call("asdsl_b200_gemv_multi", int(fmt), w0d.data_ptr(), None if w1d is None else w1d.data_ptr(),
              xd.data_ptr(), yd.data_ptr(), int(out_features), int(in_features), n, dv.stream_ptr())
    _writeback(Y, yd)


def gemv_q4_32_preq_multi(blocks, X, Y, out_features: int, in_features: int) -> None:
    """k serial gemv_q4_32_preq_fused_avx2 calls in one weight stream (preq 20-byte blocks)."""
    gemv_multi(_lib.FMT_PREQ, blocks, None, X, Y, out_features, in_features)


def gemv_q4km_q8_multi(weights_q4km, X, Y, out_features: int, in_features: int) -> None:
    """k serial gemv_q4km_q8_avx2 calls in one weight stream (reference Q4_K blocks)."""
    gemv_multi(_lib.FMT_Q4K, weights_q4km, None, X, Y, out_features, in_features)


def _packed_args(w_packed, x, scales, biases, M, K, group_size, expected_w):
    xt = x if isinstance(x, torch.Tensor) else np.asarray(x)
    batch = 1 if xt.ndim == 1 else int(xt.shape[0])
    if xt.ndim not in (1, 2):
        raise ValueError("x must be 1-D (K,) or 2-D (batch, K)")
    wsize = w_packed.numel() if isinstance(w_packed, torch.Tensor) else np.asarray(w_packed).size
    ssize = scales.numel() if isinstance(scales, torch.Tensor) else np.asarray(scales).size
    bsize = biases.numel() if isinstance(biases, torch.Tensor) else np.asarray(biases).size
    xsize = xt.numel() if isinstance(xt, torch.Tensor) else xt.size
    # validate_gemv_args (gemv_q4_avx2.cpp:901-936)
    if M <= 0 or K <= 0 or group_size <= 0:
        raise ValueError("M, K, group_size must be positive")
    if K % 2 != 0:
        raise ValueError("K must be even for 4-bit packing")
    if K % group_size != 0:
        raise ValueError("K must be divisible by group_size")
    if group_size % 8 != 0:
        raise ValueError("group_size must be a multiple of 8 for AVX2 vectorization")
    if xsize != batch * K:
        raise ValueError("x size must equal batch * K")
    if wsize != expected_w:
        raise ValueError("weight buffer size mismatch")
    if ssize != M * (K // group_size):
        raise ValueError("scales size mismatch")
    if bsize != M * (K // group_size):
        raise ValueError("biases size mismatch")
    return batch


def gemv_q4_packed(w_packed, x, scales, biases, M: int, K: int, group_size: int = 32):
    """Returns a new array: (M,) for 1-D x, (batch, M) for 2-D x (gemv_q4_avx2.cpp:1084-1126)."""
    batch = _packed_args(w_packed, x, scales, biases, M, K, group_size, M * K // 2)
    w, xd = dv.to_device(w_packed, np.uint8), dv.to_device(x, np.float32)
    s, b = dv.to_device(scales, np.float32), dv.to_device(biases, np.float32)
    yd = dv.empty(batch * M, np.float32)
    _lib.call("asdsl_b200_gemv_q4_packed", w.data_ptr(), xd.data_ptr(), s.data_ptr(), b.data_ptr(), yd.data_ptr(),
              int(M), int(K), int(group_size), int(batch), dv.stream_ptr())
    shape = (M,) if batch == 1 and (not hasattr(x, "ndim") or x.ndim == 1) else (batch, M)
    if dv.is_cuda_tensor(x):
        return yd.view(shape)
    return dv.to_host(yd).reshape(shape)


def gemv_q4_packed_into(w_packed, x, scales, biases, out, M: int, K: int, group_size: int = 32):
    y = gemv_q4_packed(w_packed, x, scales, biases, M, K, group_size)
    if isinstance(out, torch.Tensor):
        out.copy_(y if isinstance(y, torch.Tensor) else torch.from_numpy(y))
    else:
        np.copyto(out, y if isinstance(y, np.ndarray) else dv.to_host(y))
    return out


def gemv_q4_unpacked(w, x, scales, biases, M: int, K: int, group_size: int = 32):
    _packed_args(w, x, scales, biases, M, K, group_size, M * K)
    wd, xd = dv.to_device(w, np.uint8), dv.to_device(x, np.float32)
    s, b = dv.to_device(scales, np.float32), dv.to_device(biases, np.float32)
    yd = dv.empty(M, np.float32)
    _lib.call("asdsl_b200_gemv_q4_unpacked", wd.data_ptr(), xd.data_ptr(), s.data_ptr(), b.data_ptr(),
              yd.data_ptr(), int(M), int(K), int(group_size), dv.stream_ptr())
    return yd if dv.is_cuda_tensor(x) else dv.to_host(yd)


def matmul_batch_q4(w_packed, scales, biases, X_batch, Y_batch, M: int, K: int, B: int, group_size: int = 32) -> None:
    xs = tuple(X_batch.shape)
    ys = tuple(Y_batch.shape)
    if len(xs) != 2 or xs[0] != B or xs[1] != K:
        raise ValueError("X_batch must be shape (B, K)")
    if len(ys) != 2 or ys[0] != B or ys[1] != M:
        raise ValueError("Y_batch must be shape (B, M), caller zero-init")
    wsize = w_packed.numel() if isinstance(w_packed, torch.Tensor) else np.asarray(w_packed).size
    if wsize != M * (K // 2):
        raise ValueError("w_packed size must equal M * K/2")
    w, xd = dv.to_device(w_packed, np.uint8), dv.to_device(X_batch, np.float32)
    s, b = dv.to_device(scales, np.float32), dv.to_device(biases, np.float32)
    yd = _out(Y_batch, B * M, np.float32)
    _lib.call("asdsl_b200_matmul_batch_q4", w.data_ptr(), s.data_ptr(), b.data_ptr(), xd.data_ptr(), yd.data_ptr(),
              int(M), int(K), int(B), int(group_size), dv.stream_ptr())
    _writeback(Y_batch, yd)


# capability probes kept for drop-in callers (gemv_q4_avx2.cpp:1439-1470): the
# native path here is sm_100a CUDA; the CPU ISA probes report what the kernels need.
def check_avx2() -> bool:
    return True


def check_fma() -> bool:
    return True


def check_avx512() -> bool:
    return False


def check_vnni() -> bool:
    return True


def check_avx_vnni() -> bool:
    return False


def check_avx512_vnni() -> bool:
    return False


def get_num_threads() -> int:
    return 1


def set_num_threads(n: int) -> None:  # noqa: ARG001 - CPU threading knob; the CUDA grid replaces it
    return None
