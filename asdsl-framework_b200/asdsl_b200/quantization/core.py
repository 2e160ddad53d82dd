"""Group-wise 4-bit weight quantization (offline, host side).

Produces the same bytes as the reference's quantizer
(asdsl/quantization/core.py:358-424 with the MSE clip search of :291-355 and
the nibble packing of :555-561): the float32 operation sequence below is the
reference's, because the codes, scales and zeros are a bit-exact contract with
every kernel downstream.  The implementation is chunked over groups so a
200k-row lm_head quantizes in bounded memory, and it keeps only the best clip
ratio per group instead of materializing all ratios at once.

This is offline weight preparation (the reference runs it in NumPy too); the
decode hot path never calls it.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np


@dataclass
class QuantizedTensor:
    """Packed 4-bit codes + per-group fp16 scale (and zero when asymmetric)."""

    data: np.ndarray
    scales: np.ndarray
    zeros: np.ndarray | None
    bits: int
    group_size: int
    shape: tuple
    is_symmetric: bool = True

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n

    @property
    def memory_bytes(self) -> int:
        return self.data.nbytes + self.scales.nbytes + (self.zeros.nbytes if self.zeros is not None else 0)


# clip ratios searched per group (asdsl/quantization/core.py:57-60)
CLIP_RATIOS = np.array([0.85, 0.90, 0.93, 0.95, 0.97, 0.98, 0.99, 0.995, 1.0], dtype=np.float32)

_CHUNK_GROUPS = 1 << 18


def clip_ratios() -> np.ndarray:
    """ASDSL_FAST_TEST=1 searches ratio 1.0 only (asdsl/quantization/core.py:97-100)."""
    if os.environ.get("ASDSL_FAST_TEST") == "1":
        return np.array([1.0], dtype=np.float32)
    return CLIP_RATIOS


def _f16_round_trip(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float16).astype(np.float32)


def _asym_candidates(g: np.ndarray, qmax: int, r: np.float32):
    """Scale/zero of one clip ratio for an asymmetric group block (core.py:130-139)."""
    w_min = g.min(axis=1, keepdims=True)
    w_max = g.max(axis=1, keepdims=True)
    w_range = np.maximum(w_max - w_min, 1e-5)
    margin = w_range * (np.float32(1.0) - r) / 2.0
    lo = w_min + margin
    hi = w_max - margin
    span = np.maximum(hi - lo, 1e-5)
    scale = span / qmax
    zero = np.clip(-lo / np.maximum(scale, 1e-5), 0, qmax)
    return scale, zero


def _sym_candidates(g: np.ndarray, qmax: int, r: np.float32):
    """Scale of one clip ratio for a symmetric group block (core.py:124-129)."""
    abs_max = np.maximum(np.abs(g).max(axis=1, keepdims=True), 1e-5)
    return np.maximum(abs_max * r / (qmax / 2.0), 1e-5)


def _search_block(g: np.ndarray, bits: int, symmetric: bool):
    """Per-group MSE-optimal clip ratio over one block of groups (core.py:291-355).

    The first ratio with the smallest float32 MSE wins (np.argmin semantics)."""
    qmax = (1 << bits) - 1
    ratios = clip_ratios()
    best_mse = None
    best_s = best_z = None
    for r in ratios:
        r = np.float32(r)
        if symmetric:
            sc = _sym_candidates(g, qmax, r)
            half = qmax / 2.0
            s16 = np.maximum(_f16_round_trip(sc), 1e-4)
            q = np.clip(np.round(g / s16 + half), 0, qmax)
            deq = (q - half) * s16
            zr = None
        else:
            sc, zr = _asym_candidates(g, qmax, r)
            s16 = np.maximum(_f16_round_trip(sc), 1e-4)
            z16 = _f16_round_trip(zr)
            q = np.clip(np.round(g / s16 + z16), 0, qmax)
            deq = (q - z16) * s16
        mse = np.mean((g - deq) ** 2, axis=1)
        if best_mse is None:
            best_mse, best_s, best_z = mse, sc[:, 0].copy(), (None if zr is None else zr[:, 0].copy())
        else:
            better = mse < best_mse
            best_mse = np.where(better, mse, best_mse)
            best_s = np.where(better, sc[:, 0], best_s)
            if zr is not None:
                best_z = np.where(better, zr[:, 0], best_z)
    return best_s.astype(np.float16), (None if best_z is None else best_z.astype(np.float16))


def _plain_block(g: np.ndarray, bits: int, symmetric: bool):
    """Min/max (asym) or absmax (sym) scale/zero without clip search (core.py:63-94)."""
    qmax = (1 << bits) - 1
    if symmetric:
        abs_max = np.maximum(np.abs(g).max(axis=-1, keepdims=True), 1e-5)
        return (abs_max / (qmax / 2)).astype(np.float16)[:, 0], None
    w_min = g.min(axis=-1, keepdims=True)
    w_max = g.max(axis=-1, keepdims=True)
    w_range = np.maximum(w_max - w_min, 1e-5)
    scales = w_range / qmax
    zeros = -w_min / scales
    return scales.astype(np.float16)[:, 0], zeros.astype(np.float16)[:, 0]


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """Two 4-bit codes per byte, low nibble = even index (core.py:555-561)."""
    c = codes.reshape(-1)
    if c.size % 2:
        c = np.append(c, np.uint8(0))
    return ((c[0::2] & 0x0F) | ((c[1::2] & 0x0F) << 4)).astype(np.uint8)


def unpack_nibbles(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(p.size * 2, dtype=np.uint8)
    out[0::2] = p & 0x0F
    out[1::2] = p >> 4
    return out


def quantize_weights(weights, bits: int = 4, group_size: int = 128, symmetric: bool = True,
                     optimize_clips: bool = False) -> QuantizedTensor:
    """Group-wise quantization with the reference's exact rounding (core.py:358-424)."""
    if bits not in (4, 8):
        raise ValueError(f"Unsupported bit-width for this build: {bits}")
    try:
        import torch

        if isinstance(weights, torch.Tensor):
            weights = weights.detach().cpu().float().numpy()
    except ImportError:  # pragma: no cover
        pass
    w = np.asarray(weights).astype(np.float32)
    shape = w.shape
    flat = w.reshape(-1)
    rem = flat.size % group_size
    if rem:
        flat = np.concatenate([flat, np.zeros(group_size - rem, dtype=np.float32)])
    n_groups = flat.size // group_size
    grouped = flat.reshape(n_groups, group_size)
    qmax = (1 << bits) - 1

    scales = np.empty(n_groups, dtype=np.float16)
    zeros = None if symmetric else np.empty(n_groups, dtype=np.float16)
    codes = np.empty((n_groups, group_size), dtype=np.uint8)
    for g0 in range(0, n_groups, _CHUNK_GROUPS):
        g = grouped[g0 : g0 + _CHUNK_GROUPS]
        if optimize_clips:
            s, z = _search_block(g, bits, symmetric)
        else:
            s, z = _plain_block(g, bits, symmetric)
        scales[g0 : g0 + len(g)] = s
        sf = np.maximum(s.astype(np.float32), 1e-4)[:, None]
        if symmetric:
            q = np.round(g / sf + (qmax / 2))
        else:
            zeros[g0 : g0 + len(g)] = z
            q = np.round(g / sf + z.astype(np.float32)[:, None])
        codes[g0 : g0 + len(g)] = np.clip(q, 0, qmax).astype(np.uint8)

    data = pack_nibbles(codes) if bits == 4 else codes.reshape(-1)
    return QuantizedTensor(data=data, scales=scales, zeros=zeros, bits=bits, group_size=group_size,
                           shape=shape, is_symmetric=symmetric)


def dequantize_weights(qt: QuantizedTensor) -> np.ndarray:
    """(q - zero) * scale, or (q - 7.5) * scale when symmetric (core.py:427-465)."""
    q = unpack_nibbles(qt.data) if qt.bits == 4 else np.asarray(qt.data, dtype=np.uint8)
    numel = qt.numel
    rem = numel % qt.group_size
    padded = numel + (qt.group_size - rem if rem else 0)
    g = q[:padded].reshape(-1, qt.group_size).astype(np.float32)
    s = qt.scales.reshape(-1, 1).astype(np.float32)
    if qt.is_symmetric:
        d = (g - ((1 << qt.bits) - 1) / 2) * s
    else:
        d = (g - qt.zeros.reshape(-1, 1).astype(np.float32)) * s
    return d.reshape(-1)[:numel].reshape(qt.shape)


def scales_biases_f32(qt: QuantizedTensor):
    """fp32 per-group scale and bias = -zero*scale, as the reference's callers build them
    (benchmarks/test_preq_synthetic.py:29-32)."""
    n = qt.numel // qt.group_size
    sc = qt.scales[:n].astype(np.float32)
    if qt.is_symmetric:
        return sc, (np.full_like(sc, -7.5) * sc).astype(np.float32)
    zr = qt.zeros[:n].astype(np.float32)
    return sc, (-zr * sc).astype(np.float32)


def dequant_packed_projection(packed: np.ndarray, sc: np.ndarray, bi: np.ndarray, rows: int, cols: int,
                              gs: int) -> np.ndarray:
    """w = q * scale + bias in float32 (experiments/phi4_cpu_run.py:3432-3448), the
    source of the C0.1 g128 requantization."""
    q = unpack_nibbles(packed).reshape(rows, cols).astype(np.float32)
    ng = cols // gs
    s = np.repeat(sc.reshape(rows, ng), gs, axis=1)
    b = np.repeat(bi.reshape(rows, ng), gs, axis=1)
    return q * s + b
