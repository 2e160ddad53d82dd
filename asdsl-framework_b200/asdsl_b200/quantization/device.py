"""Weight preparation on the GPU: the same bytes as asdsl_b200.quantization.core / repack (and as
the reference's NumPy pipeline), computed by libasdsl_b200.so kernels on CUDA tensors.

    quantize_weights_device     quantize_weights (asdsl/quantization/core.py:358-424)
    repack_preq2_device         repack_asymmetric_to_q4_32_blocks + repack_preq_blocks_to_preq2
                                (repack_q4_32.py:63-102, repack_preq2.py:22-46)
    repack_fp32_to_q4_128_device  repack_fp32_to_q4_128_blocks (repack_q4_128.py:72-92)
    requant_q4_128_device       the C0.1 g128 requant (experiments/phi4_cpu_run.py:3432-3517)
    prepare_preq2_device        fp32 weights -> preq2 (meta, quant): the C0 engine format

Inputs and outputs are torch CUDA tensors on the current device; every call is asynchronous on the
current torch stream.  There is no CPU path: without the library or a GPU the calls raise.
"""

from __future__ import annotations

import torch

from asdsl_b200 import _lib
from asdsl_b200.quantization.core import QuantizedTensor


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(t, dtype, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    return t.to(dtype).contiguous()


def quantize_weights_device(weights: torch.Tensor, bits: int = 4, group_size: int = 128, symmetric: bool = True,
                            optimize_clips: bool = False) -> QuantizedTensor:
    """quantize_weights on the device; the QuantizedTensor holds CUDA tensors (data uint8,
    scales / zeros float16)."""
    if bits != 4:
        raise ValueError(f"Unsupported bit-width for this build: {bits}")
    w = _cuda(weights, torch.float32, "weights")
    numel = w.numel()
    if numel == 0:
        raise ValueError("quantize_weights: empty tensor")
    ng = (numel + group_size - 1) // group_size
    packed = torch.empty(ng * group_size // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(ng, dtype=torch.float16, device=w.device)
    zeros = None if symmetric else torch.empty(ng, dtype=torch.float16, device=w.device)
    _lib.call("asdsl_b200_quantize_weights", w.data_ptr(), numel, bits, group_size, 1 if symmetric else 0,
              1 if optimize_clips else 0, packed.data_ptr(), scales.data_ptr(),
              zeros.data_ptr() if zeros is not None else None, _stream(w))
    return QuantizedTensor(data=packed, scales=scales, zeros=zeros, bits=bits, group_size=group_size,
                           shape=tuple(weights.shape), is_symmetric=symmetric)


def repack_preq2_device(qt: QuantizedTensor, rows: int, cols: int) -> tuple[torch.Tensor, torch.Tensor]:
    """gs-32 QuantizedTensor (CUDA) -> preq2 (meta [rows*cols/32*4], quant [ceil(rows/4)*cols/32*64])."""
    if qt.group_size != 32:
        raise ValueError("preq2 repack requires group_size=32")
    dev = qt.data.device
    meta = torch.empty(rows * (cols // 32) * 4, dtype=torch.uint8, device=dev)
    quant = torch.empty(((rows + 3) // 4) * (cols // 32) * 64, dtype=torch.uint8, device=dev)
    _lib.call("asdsl_b200_repack_preq2", qt.data.data_ptr(), qt.scales.data_ptr(),
              qt.zeros.data_ptr() if qt.zeros is not None else None, rows, cols, meta.data_ptr(), quant.data_ptr(),
              _stream(qt.data))
    return meta, quant


def prepare_preq2_device(weights: torch.Tensor, optimize_clips: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 [rows, cols] -> preq2 (meta, quant): the C0 weight format of the engine
    (quantize_weights(gs=32, asymmetric, optimize_clips) -> preq -> preq2)."""
    rows, cols = weights.shape
    qt = quantize_weights_device(weights, 4, 32, symmetric=False, optimize_clips=optimize_clips)
    return repack_preq2_device(qt, rows, cols)


def repack_fp32_to_q4_128_device(weights: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """fp32 [rows, cols] -> Q4_128 blocks uint8 [rows, cols/128, 66]."""
    w = _cuda(weights, torch.float32, "weights")
    if w.numel() != rows * cols:
        raise ValueError("weights must hold rows * cols elements")
    out = torch.empty((rows, cols // 128, 66), dtype=torch.uint8, device=w.device)
    _lib.call("asdsl_b200_repack_q4_128_f32", w.data_ptr(), rows, cols, out.data_ptr(), _stream(w))
    return out


def requant_q4_128_device(qt: QuantizedTensor, rows: int, cols: int) -> torch.Tensor:
    """gs-32 QuantizedTensor (CUDA) -> Q4_128 blocks of its float32 dequantization (C0.1)."""
    if qt.group_size != 32:
        raise ValueError("the C0.1 requant starts from gs-32 weights")
    dev = qt.data.device
    out = torch.empty((rows, cols // 128, 66), dtype=torch.uint8, device=dev)
    _lib.call("asdsl_b200_requant_q4_128", qt.data.data_ptr(), qt.scales.data_ptr(),
              qt.zeros.data_ptr() if qt.zeros is not None else None, rows, cols, out.data_ptr(), _stream(qt.data))
    return out
