"""Seeded synthetic weight generators for formats the reference has no quantizer for.

* Q4_K (reference interpretation, asdsl/kernels/native/gemv_q4_avx2.cpp:110-120,
  :283-329): 144-byte super-block = fp16 d, fp16 dmin, 12 bytes holding sixteen
  6-bit values as a little-endian bitstream (0..7 sub-scales, 8..15 sub-mins),
  then eight 16-byte nibble runs.  The reference ships no Q4_K quantizer; the one
  here is our own (min/max per 32-sub-block, 6-bit scales relative to the block
  maximum), so its *weights* are unpinned -- parity is pinned at the kernel
  boundary (same bytes in, same y out).
* Q4_S256 (gemv_q4_s256.cpp:1-17): 8 fp16 sub-scales then 128 nibble bytes,
  implicit zero 8; our own symmetric quantizer (amax/7 per 32 weights).
* random_preq2 / random_q4k_bytes: fast random byte tensors for engine and
  edge-case tests (any bytes are valid inputs for the kernels).
"""

from __future__ import annotations

import numpy as np

from asdsl_b200.quantization.core import pack_nibbles


def _pack6(vals: np.ndarray) -> np.ndarray:
    """Sixteen 6-bit values per row -> 12 bytes, little-endian bitstream
    (value i occupies bits 6i..6i+5, as get_6bit_packed reads them)."""
    v = np.ascontiguousarray(vals.astype(np.uint8))
    bits = np.unpackbits(v[..., None], axis=-1, bitorder="little")[..., :6]
    bits = bits.reshape(v.shape[:-1] + (96,))
    return np.packbits(bits, axis=-1, bitorder="little")


def quantize_q4k(w: np.ndarray) -> np.ndarray:
    """fp32 [rows, cols] (cols % 256 == 0) -> reference-interpretation Q4_K bytes [rows, cols/256, 144]."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    nb = cols // 256
    sub = w.reshape(rows, nb, 8, 32)
    mn = np.minimum(sub.min(axis=3), 0.0)             # sub-min (<= 0), weights = d*sc*q - dmin*m
    mx = sub.max(axis=3)
    sc_f = np.maximum((mx - mn) / 15.0, 1e-12)        # per sub-block step
    m_f = -mn                                         # per sub-block offset (>= 0)
    d = np.maximum(sc_f.max(axis=2) / 63.0, 1e-12)
    dmin = np.maximum(m_f.max(axis=2) / 63.0, 1e-12)
    d16 = d.astype(np.float16)
    dmin16 = dmin.astype(np.float16)
    d32 = np.maximum(d16.astype(np.float32), 1e-12)
    dmin32 = np.maximum(dmin16.astype(np.float32), 1e-12)
    sc6 = np.clip(np.round(sc_f / d32[:, :, None]), 1, 63).astype(np.uint8)
    m6 = np.clip(np.round(m_f / dmin32[:, :, None]), 0, 63).astype(np.uint8)
    step = d32[:, :, None] * sc6
    off = dmin32[:, :, None] * m6
    q = np.clip(np.round((sub + off[..., None]) / step[..., None]), 0, 15).astype(np.uint8)
    out = np.empty((rows, nb, 144), dtype=np.uint8)
    out[:, :, 0:2] = d16.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:4] = dmin16.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 4:16] = _pack6(np.concatenate([sc6, m6], axis=2))
    nib = pack_nibbles(q.reshape(-1)).reshape(rows, nb, 8, 16)
    out[:, :, 16:] = nib.reshape(rows, nb, 128)
    return out


def quantize_s256(w: np.ndarray) -> np.ndarray:
    """fp32 [rows, cols] (cols % 256 == 0) -> Q4_S256 bytes [rows, cols/256, 144]."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    nb = cols // 256
    sub = w.reshape(rows, nb, 8, 32)
    amax = np.abs(sub).max(axis=3)
    s16 = np.where(amax < 1e-12, 0.0, amax / 7.0).astype(np.float16)
    s32 = s16.astype(np.float32)
    inv = np.where(s32 > 0, 1.0 / np.where(s32 > 0, s32, 1.0), 0.0).astype(np.float32)
    q = np.clip(np.round(sub * inv[..., None]) + 8, 0, 15).astype(np.uint8)
    out = np.empty((rows, nb, 144), dtype=np.uint8)
    out[:, :, 0:16] = s16.view(np.uint8).reshape(rows, nb, 16)
    out[:, :, 16:] = pack_nibbles(q.reshape(-1)).reshape(rows, nb, 128)
    return out


def random_preq2(rng: np.random.Generator, rows: int, cols: int, scale_range=(0.01, 0.05),
                 zero_range=(6.0, 9.0)):
    """Random preq2 (meta, quant) bytes: uniform nibbles, fp16 scales and zeros."""
    ng = cols // 32
    nb = (rows + 3) // 4
    s = rng.uniform(*scale_range, size=(rows, ng)).astype(np.float16)
    z = rng.uniform(*zero_range, size=(rows, ng)).astype(np.float16)
    meta = np.empty((rows, ng, 4), dtype=np.uint8)
    meta[:, :, 0:2] = s.view(np.uint8).reshape(rows, ng, 2)
    meta[:, :, 2:4] = z.view(np.uint8).reshape(rows, ng, 2)
    quant = rng.integers(0, 256, size=(nb, ng, 64), dtype=np.uint8)
    if rows % 4:
        # unused band slots are zero in the reference layout (repack_preq2.py:31-44)
        quant[nb - 1, :, (rows % 4) * 16 :] = 0
    return meta.reshape(rows, ng * 4), quant


def random_q4k_bytes(rng: np.random.Generator, rows: int, cols: int, d: float = 0.002, dmin: float = 0.004):
    """Random Q4_K bytes with fixed fp16 d / dmin and random 6-bit scales and nibbles."""
    nb = cols // 256
    blocks = rng.integers(0, 256, size=(rows, nb, 144), dtype=np.uint8)
    blocks[:, :, 0:2] = np.array([d], dtype=np.float16).view(np.uint8)
    blocks[:, :, 2:4] = np.array([dmin], dtype=np.float16).view(np.uint8)
    return blocks


def random_q4_128(rng: np.random.Generator, rows: int, cols: int, scale_range=(0.006, 0.012)) -> np.ndarray:
    """Random Q4_128 blocks [rows][cols/128][66]: uniform nibbles and fp16 scales in the range the
    symmetric quantizer gives N(0, 0.02) rows (amax / 7); for timing-sized weights whose float
    source would take minutes to quantize on the host."""
    ng = cols // 128
    blocks = rng.integers(0, 256, size=(rows, ng, 66), dtype=np.uint8)
    s = rng.uniform(*scale_range, size=(rows, ng)).astype(np.float16)
    blocks[:, :, 0:2] = s.view(np.uint8).reshape(rows, ng, 2)
    return blocks
