"""Seeded random-init Phi-4-mini-shaped decoder weights in the engine's byte formats.

There is no network for checkpoints, so decode benchmarks and trajectory tests
run on random-init weights of the reference's model shape
(experiments/phi4_cpu_run.py:316-334): 32 layers, hidden 3072, 24 Q / 8 KV
heads of 128, MLP 8192, vocab 200064, partial rotary 96, RMSNorm eps 1e-5.

Projection bytes are random preq2 blobs (uniform nibbles, fp16 scales/zeros) --
the kernels consume bytes, and drawing bytes directly is what makes a
3.2-billion-weight model buildable in seconds.  The tied fp16 embedding is the
lm_head source, quantized inside the engine exactly as the reference engine's
constructor does (asdsl/kernels/native/unified_engine.cpp:320-400).
"""

from __future__ import annotations

import hashlib
import math

import numpy as np

from asdsl_b200.quantization.synth import random_preq2

PHI4_MINI = dict(num_layers=32, hidden=3072, n_heads=24, n_kv_heads=8, head_dim=128, inter=8192,
                 vocab=200064, max_seq=2048, rotary_dim=96, eps=1e-5, theta=10000.0)

TINY = dict(num_layers=2, hidden=256, n_heads=2, n_kv_heads=1, head_dim=128, inter=512,
            vocab=512, max_seq=64, rotary_dim=96, eps=1e-5, theta=10000.0)

# long-trajectory parity shape: Phi-4-mini's head geometry (GQA 3:1 would need 3 heads per
# KV head; 6/2 keeps it), small enough for the CPU oracle to run 128+ steps in seconds
SMALL = dict(num_layers=4, hidden=768, n_heads=6, n_kv_heads=2, head_dim=128, inter=2048,
             vocab=8192, max_seq=256, rotary_dim=96, eps=1e-5, theta=10000.0)


def rope_tables(max_seq: int, rotary_dim: int, theta: float = 10000.0):
    """cos/sin [max_seq, rotary_dim/2] float32, angles in float64
    (experiments/phi4_cpu_run.py:3318-3344: freq = 1/theta^(2i/rotary_dim))."""
    half = rotary_dim // 2
    i = np.arange(half, dtype=np.float64)
    freq = 1.0 / (theta ** (2.0 * i / rotary_dim))
    ang = np.arange(max_seq, dtype=np.float64)[:, None] * freq[None, :]
    # math.cos/sin per element as the reference does; numpy's are correctly rounded
    # to the same double values for these arguments, checked in tests.
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope_tables_reference_loop(max_seq: int, rotary_dim: int, theta: float = 10000.0):
    """The reference's scalar loop (for the equality test of rope_tables)."""
    half = rotary_dim // 2
    c = np.zeros((max_seq, half), np.float32)
    s = np.zeros((max_seq, half), np.float32)
    for pos in range(max_seq):
        for i in range(half):
            freq = 1.0 / (theta ** (2.0 * i / rotary_dim))
            c[pos, i] = math.cos(pos * freq)
            s[pos, i] = math.sin(pos * freq)
    return c, s


def build_model(cfg: dict, seed: int, norms_one: bool = True) -> dict:
    """Random-init decoder: dict(config, embed_f16, output_norm, cos, sin, layers=[...]).

    Each layer holds rms_att / rms_ffn (float32) and preq2 meta/quant bytes for
    qkv_proj [(nh+2nkv)*hd, H], o_proj [H, nh*hd], gate_up_proj [2I, H] (gate rows
    first, then up), down_proj [H, I]."""
    rng = np.random.default_rng(seed)
    H, I = cfg["hidden"], cfg["inter"]
    qd = cfg["n_heads"] * cfg["head_dim"]
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]
    layers = []
    for _ in range(cfg["num_layers"]):
        L = {}
        for name, (rows, cols) in (("qkv_proj", (qd + 2 * kvd, H)), ("o_proj", (H, qd)),
                                   ("gate_up_proj", (2 * I, H)), ("down_proj", (H, I))):
            meta, quant = random_preq2(rng, rows, cols, scale_range=(0.004, 0.012), zero_range=(7.0, 8.0))
            L[name + "_meta"] = meta.reshape(-1)
            L[name + "_quant"] = quant.reshape(-1)
        if norms_one:
            L["rms_att"] = np.ones(H, np.float32)
            L["rms_ffn"] = np.ones(H, np.float32)
        else:
            L["rms_att"] = rng.uniform(0.8, 1.2, H).astype(np.float32)
            L["rms_ffn"] = rng.uniform(0.8, 1.2, H).astype(np.float32)
        layers.append(L)
    embed = (rng.standard_normal((cfg["vocab"], H), dtype=np.float32) * 0.02).astype(np.float16)
    cos, sin = rope_tables(cfg["max_seq"], cfg["rotary_dim"], cfg.get("theta", 10000.0))
    return dict(config=dict(cfg), embed_f16=embed, output_norm=np.ones(H, np.float32), cos=cos, sin=sin,
                layers=layers)


def model_digest(model: dict) -> str:
    """sha256 over every byte of a model (detects generator drift against fixtures)."""
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(model["embed_f16"]).tobytes())
    h.update(np.ascontiguousarray(model["output_norm"]).tobytes())
    h.update(np.ascontiguousarray(model["cos"]).tobytes())
    h.update(np.ascontiguousarray(model["sin"]).tobytes())
    for L in model["layers"]:
        for k in sorted(L):
            h.update(np.ascontiguousarray(L[k]).tobytes())
    return h.hexdigest()


def build_model_device(cfg: dict, seed: int, device="cuda", norms_one: bool = True, quantized: bool = False) -> dict:
    """The same kind of random-init model as build_model (preq2 bytes: uniform nibbles, fp16
    scales in [0.004, 0.012) and zeros in [7, 8); fp16 N(0, 0.02) embedding), generated on the
    GPU with torch's CUDA generator: seconds instead of minutes for the full Phi-4-mini shape, for
    timing runs that need no host copy of the weights.  Not byte-identical to build_model.

    quantized=True draws every projection as float32 N(0, 0.02) and runs the reference's C0 weight
    pipeline on it (quantize_weights gs 32 asymmetric with the clip search -> preq -> preq2,
    asdsl_b200.quantization.device): the bytes config 3 prescribes, from the device RNG."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, I = cfg["hidden"], cfg["inter"]
    qd = cfg["n_heads"] * cfg["head_dim"]
    kvd = cfg["n_kv_heads"] * cfg["head_dim"]

    def preq2(rows, cols):
        if quantized:
            from asdsl_b200.quantization.device import prepare_preq2_device

            w = torch.randn((rows, cols), generator=g, device=device) * 0.02
            meta, quant = prepare_preq2_device(w)
            del w
            return meta, quant
        ng = cols // 32
        s = (torch.rand((rows, ng), generator=g, device=device) * 0.008 + 0.004).half()
        z = (torch.rand((rows, ng), generator=g, device=device) + 7.0).half()
        meta = torch.stack([s, z], dim=2).contiguous().view(torch.uint8).reshape(-1)
        nb = (rows + 3) // 4
        quant = torch.randint(0, 256, (nb * ng * 64,), generator=g, device=device, dtype=torch.uint8)
        if rows % 4:
            quant.view(nb, ng, 64)[nb - 1, :, (rows % 4) * 16:] = 0
        return meta, quant

    layers = []
    for _ in range(cfg["num_layers"]):
        L = {}
        for name, (rows, cols) in (("qkv_proj", (qd + 2 * kvd, H)), ("o_proj", (H, qd)),
                                   ("gate_up_proj", (2 * I, H)), ("down_proj", (H, I))):
            L[name + "_meta"], L[name + "_quant"] = preq2(rows, cols)
        ones = torch.ones(H, dtype=torch.float32, device=device)
        L["rms_att"] = ones if norms_one else (torch.rand(H, generator=g, device=device) * 0.4 + 0.8)
        L["rms_ffn"] = ones if norms_one else (torch.rand(H, generator=g, device=device) * 0.4 + 0.8)
        layers.append(L)
    embed = (torch.randn((cfg["vocab"], H), generator=g, device=device) * 0.02).half()
    cos, sin = rope_tables(cfg["max_seq"], cfg["rotary_dim"], cfg.get("theta", 10000.0))
    return dict(config=dict(cfg), embed_f16=embed, output_norm=torch.ones(H, dtype=torch.float32, device=device),
                cos=cos, sin=sin, layers=layers)


def model_to_host(model: dict) -> dict:
    """A copy of a build_model_device model with every tensor as a host numpy array (for the CPU
    oracle engine)."""
    def h(v):
        return v.cpu().numpy() if hasattr(v, "cpu") else v

    return dict(config=dict(model["config"]), embed_f16=h(model["embed_f16"]), output_norm=h(model["output_norm"]),
                cos=model["cos"], sin=model["sin"], layers=[{k: h(v) for k, v in L.items()} for L in model["layers"]])
