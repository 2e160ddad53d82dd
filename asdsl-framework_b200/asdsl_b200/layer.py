"""One decoder layer's projection set on the device (the C0.1 byte mix), run as
the dependent chain a decode step runs:

    qkv  = W_qkv  x            preq2 gs 32   (unified_engine.cpp:1411-1413)
    o    = W_o    qkv[:q_dim]  preq2 gs 32   (:1487-1489; the q slice stands in for
                                              the attention output, which config 1 omits)
    h    = silu(W_gate o) * (W_up o)   Q4_128, fused in one kernel (:1532-1538 + :836-857)
    y    = W_down h            Q4_128        (:1592-1598)

Weights live in HBM for the object's lifetime; ``step`` enqueues the four
kernels on torch's current stream (capturable in a CUDA graph), ``forward``
is the host-buffer call a user makes (x in, outputs out, copies included),
one native call (asdsl_b200_layer_forward).
``build_c1_host`` reproduces the reference's C0.1 weight pipeline for the
benchmark: gs-32 asymmetric quantization with the clip search, then
dequantize and requantize to Q4_128 for gate_up/down
(experiments/phi4_cpu_run.py:3482-3517).
"""

from __future__ import annotations

import numpy as np
import torch

from asdsl_b200 import _lib
from asdsl_b200.quantization import core, repack

FMT_PREQ2, FMT_Q4_128, FMT_Q4_128_BANDED = 0, 2, 4


def relayout_q4_128(blocks: torch.Tensor, rows: int, cols: int):
    """Device re-layout of Q4_128 blocks into (quant, scales) bands (asdsl_b200_relayout_q4_128)."""
    nb, ng = (rows + 3) // 4, cols // 128
    q = torch.empty(nb * ng * 256, dtype=torch.uint8, device=blocks.device)
    s = torch.empty(nb * ng * 8, dtype=torch.uint8, device=blocks.device)
    _lib.call("asdsl_b200_relayout_q4_128", blocks.data_ptr(), q.data_ptr(), s.data_ptr(), rows, cols,
              torch.cuda.current_stream().cuda_stream or None)
    return q, s


class LayerProjections:
    def __init__(self, qkv_meta, qkv_quant, o_meta, o_quant, gate_up_q4_128, down_q4_128, hidden: int,
                 qkv_rows: int, q_dim: int, inter: int):
        dev = torch.device("cuda", torch.cuda.current_device())

        def up(a):
            return a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a)).to(dev)

        self.qkv_meta, self.qkv_quant = up(qkv_meta), up(qkv_quant)
        self.o_meta, self.o_quant = up(o_meta), up(o_quant)
        self.H, self.QKV, self.QD, self.I = hidden, qkv_rows, q_dim, inter
        # Q4_128 blocks -> banded device layout (bit-exact byte moves, done once)
        if isinstance(gate_up_q4_128, tuple):
            self.gu_q, self.gu_s = gate_up_q4_128
            self.dn_q, self.dn_s = down_q4_128
        else:
            self.gu_q, self.gu_s = relayout_q4_128(up(gate_up_q4_128), 2 * inter, hidden)
            self.dn_q, self.dn_s = relayout_q4_128(up(down_q4_128), hidden, inter)
        # the three results live side by side in one block, so forward() reads them back in one copy
        n_out = qkv_rows + 2 * hidden
        self._out_cat = torch.empty(n_out, dtype=torch.float32, device=dev)
        self.qkv_out = self._out_cat[:qkv_rows]
        self.o_out = self._out_cat[qkv_rows : qkv_rows + hidden]
        self.y = self._out_cat[qkv_rows + hidden :]
        self.h = torch.empty(inter, dtype=torch.float32, device=dev)
        self._x = torch.empty(hidden, dtype=torch.float32, device=dev)
        self._native = None  # forward(): asdsl_b200_layer handle, created on first use

    @property
    def weight_bytes(self) -> int:
        return sum(t.numel() for t in (self.qkv_meta, self.qkv_quant, self.o_meta, self.o_quant, self.gu_q, self.gu_s,
                                       self.dn_q, self.dn_s))

    @property
    def algorithmic_bytes(self) -> int:
        """Packed weights + fp32 activations in + fp32 results out of each GEMV
        (the reference's GB/s definition without its A8 overhead term,
        benchmarks/kernel_bench_compare.py:46-52)."""
        act = 4 * (self.H + self.QKV) + 4 * (self.QD + self.H) + 4 * (self.H + self.I) + 4 * (self.I + self.H)
        return self.weight_bytes + act

    def step(self, x: torch.Tensor, stream_ptr=None) -> int:
        """Enqueue the 4 kernels; returns the number of launches."""
        s = stream_ptr if stream_ptr is not None else (torch.cuda.current_stream().cuda_stream or None)
        L = _lib.load()
        _lib.check(L.asdsl_b200_gemv_preq2_fused(self.qkv_meta.data_ptr(), self.qkv_quant.data_ptr(), x.data_ptr(),
                                                 self.qkv_out.data_ptr(), self.QKV, self.H, 32, s))
        _lib.check(L.asdsl_b200_gemv_preq2_fused(self.o_meta.data_ptr(), self.o_quant.data_ptr(),
                                                 self.qkv_out.data_ptr(), self.o_out.data_ptr(), self.H, self.QD, 32, s))
        _lib.check(L.asdsl_b200_gateup_silu(FMT_Q4_128_BANDED, self.gu_q.data_ptr(), self.gu_s.data_ptr(),
                                            self.o_out.data_ptr(), self.h.data_ptr(), self.I, self.H, s))
        _lib.check(L.asdsl_b200_gemv_q4_128_banded(self.dn_q.data_ptr(), self.dn_s.data_ptr(), self.h.data_ptr(),
                                                   self.y.data_ptr(), self.H, self.I, s))
        return 4

    def forward(self, x_host: np.ndarray) -> dict:
        """Host buffers in and out: x[hidden] in, {"qkv", "o", "y"} out, synchronous.  One native
        call (asdsl_b200_layer_forward): x into pinned staging, one replay of a CUDA graph holding
        the H2D copy, the four kernels and the D2H copy on the layer's own stream, then the results
        out of pinned staging.  The graph is captured on the first call."""
        import ctypes

        lib = _lib.load()
        if self._native is None:
            h = ctypes.c_void_p()
            ptrs = [t.data_ptr() for t in (self.qkv_meta, self.qkv_quant, self.o_meta, self.o_quant, self.gu_q,
                                           self.gu_s, self.dn_q, self.dn_s, self._x, self.h, self._out_cat)]
            _lib.check(lib.asdsl_b200_layer_create(*ptrs, self.H, self.QKV, self.QD, self.I, ctypes.byref(h)),
                       "layer_create")
            self._native = h
        x = np.ascontiguousarray(x_host, dtype=np.float32)
        if x.size != self.H:
            raise ValueError(f"forward: x has {x.size} elements, the layer takes {self.H}")
        out = np.empty(self.QKV + 2 * self.H, dtype=np.float32)
        _lib.check(lib.asdsl_b200_layer_forward(self._native, x.ctypes.data, out.ctypes.data), "layer_forward")
        n1, n2 = self.QKV, self.QKV + self.H
        return {"qkv": out[:n1], "o": out[n1:n2], "y": out[n2:]}

    def close(self) -> None:
        if self._native is not None:
            _lib.load().asdsl_b200_layer_destroy(self._native)
            self._native = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def clone(self) -> "LayerProjections":
        """Same weights at new device addresses (L2-rotation copies for benchmarking)."""
        return LayerProjections(self.qkv_meta.clone(), self.qkv_quant.clone(), self.o_meta.clone(),
                                self.o_quant.clone(), (self.gu_q.clone(), self.gu_s.clone()),
                                (self.dn_q.clone(), self.dn_s.clone()), self.H, self.QKV, self.QD, self.I)


C1 = dict(hidden=3072, qkv_rows=5120, q_dim=3072, inter=8192)


def build_c1_host(seed: int = 1, cfg: dict = C1) -> dict:
    """Config 1's weights and activation from one seeded generator: W_qkv, W_o, W_gate_up,
    W_down ~ N(0, 0.02) drawn in that order, then x ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    H, QKV, QD, I = cfg["hidden"], cfg["qkv_rows"], cfg["q_dim"], cfg["inter"]
    out = {}
    for name, (rows, cols) in (("qkv", (QKV, H)), ("o", (H, QD))):
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        qt = core.quantize_weights(w, 4, 32, False, True)
        sc, bi = core.scales_biases_f32(qt)
        flat = repack.blocks_to_flat(repack.repack_asymmetric_to_q4_32_blocks(qt.data, sc, bi, rows, cols, 32))
        out[name + "_meta"], out[name + "_quant"] = repack.repack_preq_blocks_to_preq2(flat, rows, cols)
    for name, (rows, cols) in (("gate_up", (2 * I, H)), ("down", (H, I))):
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        qt = core.quantize_weights(w, 4, 32, False, True)
        sc, bi = core.scales_biases_f32(qt)
        wdq = core.dequant_packed_projection(qt.data, sc, bi, rows, cols, 32)
        out[name + "_q4_128"] = repack.repack_fp32_to_q4_128_blocks(wdq, rows, cols)
    out["x"] = rng.standard_normal(H).astype(np.float32)
    out["cfg"] = dict(cfg)
    return out


def build_c1_device(seed: int = 1, cfg: dict = C1) -> dict:
    """build_c1_host's bytes with the quantizer and repackers run on the GPU
    (asdsl_b200.quantization.device): the same seeded float32 draws on the host, then
    quantize / preq2 / C0.1 requant as device kernels; the dict holds host numpy arrays."""
    from asdsl_b200.quantization import device

    rng = np.random.default_rng(seed)
    H, QKV, QD, I = cfg["hidden"], cfg["qkv_rows"], cfg["q_dim"], cfg["inter"]
    out = {}
    for name, (rows, cols) in (("qkv", (QKV, H)), ("o", (H, QD))):
        w = torch.from_numpy((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)).cuda()
        meta, quant = device.prepare_preq2_device(w)
        out[name + "_meta"] = meta.cpu().numpy().reshape(rows, (cols // 32) * 4)
        out[name + "_quant"] = quant.cpu().numpy().reshape((rows + 3) // 4, cols // 32, 64)
    for name, (rows, cols) in (("gate_up", (2 * I, H)), ("down", (H, I))):
        w = torch.from_numpy((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)).cuda()
        qt = device.quantize_weights_device(w, 4, 32, symmetric=False, optimize_clips=True)
        out[name + "_q4_128"] = device.requant_q4_128_device(qt, rows, cols).cpu().numpy()
    out["x"] = rng.standard_normal(H).astype(np.float32)
    out["cfg"] = dict(cfg)
    return out


def from_host(host: dict) -> LayerProjections:
    c = host["cfg"]
    return LayerProjections(host["qkv_meta"], host["qkv_quant"], host["o_meta"], host["o_quant"],
                            host["gate_up_q4_128"], host["down_q4_128"], c["hidden"], c["qkv_rows"], c["q_dim"],
                            c["inter"])


def layer_reference(orc, host: dict) -> dict:
    """The same chain on the CPU oracle (test / bench checker only)."""
    c = host["cfg"]
    H, QKV, QD, I = c["hidden"], c["qkv_rows"], c["q_dim"], c["inter"]
    qkv = orc.gemv_preq2_fused(host["qkv_meta"], host["qkv_quant"], host["x"], QKV, H)
    o = orc.gemv_preq2_fused(host["o_meta"], host["o_quant"], qkv[:QD], H, QD)
    gu = orc.gemv_q4_128_fused(host["gate_up_q4_128"], o, 2 * I, H)
    h = orc.swiglu(gu[:I], gu[I:])
    y = orc.gemv_q4_128_fused(host["down_q4_128"], h, H, I)
    return {"qkv": qkv, "o": o, "y": y}
