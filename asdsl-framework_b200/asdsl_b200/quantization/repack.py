"""Byte-format repackers for the decode GEMVs (offline, host side, vectorized).

Each function produces exactly the bytes of the reference's per-group Python
loop it replaces (those loops take ~28 s per 16384x3072 tensor); the arithmetic
that decides a byte is the reference's, including where it runs in float64:

* repack_asymmetric_to_q4_32_blocks  <- asdsl/quantization/repack_q4_32.py:63-102
  (scale = float(max(s, 1e-8)), zero = -bias/scale in float64, both rounded to fp16)
* repack_preq_blocks_to_preq2        <- asdsl/quantization/repack_preq2.py:22-46
  (pure byte moves: meta [M][ng][4], quant [ceil(M/4)][ng][4 rows x 16 B])
* repack_fp32_to_q4_128_blocks       <- asdsl/quantization/repack_q4_128.py:22-31, :72-92
  (amax in float32, scale = amax/7 in float64 -> fp16, codes from float32 x*fl32(7/amax))
* repack_asymmetric_to_q4_128_blocks <- asdsl/quantization/repack_q4_128.py:34-69
"""

from __future__ import annotations

import numpy as np

from asdsl_b200.quantization.core import unpack_nibbles

PREQ_BLOCK_SIZE = 20
Q4_128_BLOCK_SIZE = 66
PREQ2_META_BYTES = 4
PREQ2_GROUP_QUANT_BYTES = 64
PREQ2_ROW_BAND = 4

_ROW_CHUNK = 8192


def _nibbles_rows(packed: np.ndarray, rows: int, cols: int) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(packed, dtype=np.uint8).reshape(rows, cols // 2))


def repack_asymmetric_to_q4_32_blocks(packed, scales, biases, rows: int, cols: int, group_size: int = 32, *,
                                      bits: int = 4) -> np.ndarray:
    """(rows, cols/32, 20) preq blocks: fp16 scale, fp16 zero, 16 nibble bytes."""
    if group_size != 32:
        raise ValueError("repack_asymmetric_to_q4_32_blocks requires group_size=32")
    del bits
    ng = cols // group_size
    p = _nibbles_rows(packed, rows, cols).reshape(rows, ng, 16)
    sc = np.asarray(scales).astype(np.float32).ravel()[: rows * ng]
    bi = np.asarray(biases).astype(np.float32).ravel()[: rows * ng]
    scale64 = np.maximum(sc.astype(np.float64), 1e-8)
    zero64 = -bi.astype(np.float64) / scale64
    blocks = np.empty((rows, ng, PREQ_BLOCK_SIZE), dtype=np.uint8)
    blocks[:, :, 0:2] = scale64.astype(np.float16).view(np.uint8).reshape(rows, ng, 2)
    blocks[:, :, 2:4] = zero64.astype(np.float16).view(np.uint8).reshape(rows, ng, 2)
    blocks[:, :, 4:] = p
    return blocks


def blocks_to_flat(blocks: np.ndarray) -> np.ndarray:
    r, g, b = blocks.shape
    return np.ascontiguousarray(blocks.reshape(r, g * b))


def repack_preq_blocks_to_preq2(flat_preq, rows: int, cols: int, group_size: int = 32):
    """Split preq blocks into (meta (rows, ng*4), quant (ceil(rows/4), ng, 64))."""
    if group_size != 32:
        raise ValueError("preq2 repack requires group_size=32")
    ng = cols // group_size
    flat = np.ravel(flat_preq)
    if flat.size < rows * ng * PREQ_BLOCK_SIZE:
        raise ValueError("flat_preq too small for shape")
    blk = flat[: rows * ng * PREQ_BLOCK_SIZE].reshape(rows, ng, PREQ_BLOCK_SIZE)
    meta = np.ascontiguousarray(blk[:, :, 0:4]).reshape(rows, ng * 4)
    nb = (rows + 3) // 4
    quant = np.zeros((nb * 4, ng, 16), dtype=np.uint8)
    quant[:rows] = blk[:, :, 4:20]
    quant = np.ascontiguousarray(quant.reshape(nb, 4, ng, 16).transpose(0, 2, 1, 3)).reshape(nb, ng, 64)
    return np.ascontiguousarray(meta), quant


def preq2_flat_sizes(rows: int, cols: int, group_size: int = 32) -> tuple[int, int]:
    ng = cols // group_size
    nb = (rows + 3) // 4
    return rows * ng * PREQ2_META_BYTES, nb * ng * PREQ2_GROUP_QUANT_BYTES


def meta_to_flat(meta: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(meta.reshape(-1))


def quant_to_flat(quant: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(quant.reshape(-1))


def preq2_to_preq(meta, quant, rows: int, cols: int) -> np.ndarray:
    """Inverse byte permutation (preq2 -> flat preq), for tests and caches."""
    ng = cols // 32
    m = np.asarray(meta, dtype=np.uint8).reshape(rows, ng, 4)
    nb = (rows + 3) // 4
    q = np.asarray(quant, dtype=np.uint8).reshape(nb, ng, 4, 16).transpose(0, 2, 1, 3).reshape(nb * 4, ng, 16)
    out = np.empty((rows, ng, 20), dtype=np.uint8)
    out[:, :, 0:4] = m
    out[:, :, 4:] = q[:rows]
    return out.reshape(rows, ng * 20)


def _q4_128_from_f32_rows(w: np.ndarray) -> np.ndarray:
    """Symmetric Q4_128 blocks of a (r, ng, 128) float32 block (repack_q4_128.py:22-31)."""
    r, ng, _ = w.shape
    amax32 = np.abs(w).max(axis=2)
    amax64 = amax32.astype(np.float64)
    zero = amax64 < 1e-12
    safe = np.where(zero, 1.0, amax64)
    scale16 = np.where(zero, 0.0, safe / 7.0).astype(np.float16)
    inv32 = (7.0 / safe).astype(np.float32)
    q = np.clip(np.round(w * inv32[:, :, None]) + np.float32(8.0), 0, 15).astype(np.uint8)
    nib = ((q[:, :, 1::2] << 4) | q[:, :, 0::2]).astype(np.uint8)
    nib[zero] = 0x88
    out = np.empty((r, ng, Q4_128_BLOCK_SIZE), dtype=np.uint8)
    out[:, :, 0:2] = scale16.view(np.uint8).reshape(r, ng, 2)
    out[:, :, 2:] = nib
    return out


def repack_fp32_to_q4_128_blocks(weights, rows: int, cols: int, group_size: int = 128) -> np.ndarray:
    """(rows, cols/128, 66) Q4_128 blocks from fp32 weights (repack_q4_128.py:72-92)."""
    if group_size != 128:
        raise ValueError("repack_fp32_to_q4_128_blocks requires group_size=128")
    ng = cols // 128
    w2d = np.asarray(weights, dtype=np.float32).reshape(rows, cols)
    out = np.empty((rows, ng, Q4_128_BLOCK_SIZE), dtype=np.uint8)
    for r0 in range(0, rows, _ROW_CHUNK):
        blk = w2d[r0 : r0 + _ROW_CHUNK, : ng * 128].reshape(-1, ng, 128)
        out[r0 : r0 + len(blk)] = _q4_128_from_f32_rows(blk)
    return out


def repack_asymmetric_to_q4_128_blocks(packed, scales, biases, rows: int, cols: int, group_size: int = 128, *,
                                       bits: int = 4) -> np.ndarray:
    """Requantize asymmetric packed gs-128 weights to Q4_128 (repack_q4_128.py:34-69):
    zero = -bias/scale in float64; w = (q - zero) * scale evaluated in float32, since
    the reference combines a float32 array with Python floats."""
    if group_size != 128:
        raise ValueError("repack_asymmetric_to_q4_128_blocks requires group_size=128")
    del bits
    ng = cols // 128
    q = unpack_nibbles(packed).reshape(rows, ng, 128).astype(np.float32)
    sc64 = np.maximum(np.asarray(scales).astype(np.float32).ravel()[: rows * ng].astype(np.float64), 1e-8)
    bi64 = np.asarray(biases).astype(np.float32).ravel()[: rows * ng].astype(np.float64)
    zero32 = (-bi64 / sc64).astype(np.float32).reshape(rows, ng, 1)
    w = (q - zero32) * sc64.astype(np.float32).reshape(rows, ng, 1)
    return _q4_128_from_f32_rows(w)


def q4_128_to_banded(blocks, rows: int, cols: int):
    """Host form of the device re-layout of Q4_128 blocks (asdsl_b200_relayout_q4_128):
    quant [ceil(rows/4)][cols/128][4][64] nibble bytes + scales [ceil(rows/4)][cols/128][4] fp16,
    rows past `rows` zero-filled.  Pure byte moves."""
    ng = cols // 128
    nb = (rows + 3) // 4
    b = np.asarray(blocks, dtype=np.uint8).reshape(rows, ng, 66)
    pad = np.zeros((nb * 4, ng, 66), dtype=np.uint8)
    pad[:rows] = b
    pad = pad.reshape(nb, 4, ng, 66).transpose(0, 2, 1, 3)
    quant = np.ascontiguousarray(pad[..., 2:]).reshape(-1)
    scales = np.ascontiguousarray(pad[..., 0:2]).reshape(-1)
    return quant, scales
