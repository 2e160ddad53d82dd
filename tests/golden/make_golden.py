"""Generate tests/golden/*.npz from the reference itself.  Run in a container where
the reference sources are present ($ASDSL_REFERENCE, or a "reference" directory beside the repo)
and oracle/_ref is built
(``make -C oracle ref``):

    python tests/golden/make_golden.py [--ref PATH]

Nothing at test time reads the reference; the fixtures carry its outputs.
Sources of truth per fixture:
  quant_*.npz   asdsl.quantization.core.quantize_weights           (core.py:358-424)
  repack_*.npz  asdsl.quantization.repack_q4_32 / _preq2 / _q4_128 (the repackers)
  kern_*.npz    the reference's compiled AVX2 kernels (oracle/_ref via ref_shim.cpp)
  engine_tiny.npz  the reference's compiled UnifiedEngine (_native_unified in oracle/_ref)
  gemm_q4_128.npz  the reference's compiled gemm_q4_128_q8_avx2 (gemv_q4_128.cpp:262-306, fp32
                   activations, batch rows >= 64 left untouched) via ref_shim.cpp
  engine_long.npz  the same engine: 160 greedy steps on TINY-shaped models with a 256-position
                   cache (seeds 5 and 7), shapes on which the reference and a faithful
                   restatement with another fp32 summation order agree token for token
Inputs are small and stored verbatim, except the tiny engine's weights, which
are regenerated from a seed; their sha256 is stored to catch generator drift.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
OUT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "asdsl-framework_b200"))
sys.path.insert(0, ROOT)


def ref_engine(nu, model, preq_blocks: bool = True):
    """The reference's UnifiedEngine over a synthetic model (preq blocks + preq2 blobs per layer,
    tied fp16 embedding as lm_head source), as unified_bridge.build_unified_engine wires it.
    preq_blocks=False passes one-byte placeholders for the 20-byte preq blocks, which the engine
    binds but never reads when preq2 blobs are present (ASDSL_PREQ2=1, unified_engine.cpp:129-143):
    the full-size model then needs no second copy of its weights."""
    from asdsl_b200.quantization.repack import preq2_to_preq

    c = model["config"]
    cfg = nu.EngineConfig()
    cfg.num_layers, cfg.hidden_size = c["num_layers"], c["hidden"]
    cfg.num_heads, cfg.num_kv_heads, cfg.head_dim = c["n_heads"], c["n_kv_heads"], c["head_dim"]
    cfg.intermediate_size, cfg.vocab_size = c["inter"], c["vocab"]
    cfg.rms_norm_eps, cfg.group_size, cfg.lm_head_group_size = c["eps"], 32, 0
    cfg.max_seq_len, cfg.rotary_dim, cfg.weight_format = c["max_seq"], c["rotary_dim"], 0
    H, I = c["hidden"], c["inter"]
    qkv_rows = (c["n_heads"] + 2 * c["n_kv_heads"]) * c["head_dim"]
    shapes = {"qkv_proj": (qkv_rows, H), "o_proj": (H, c["n_heads"] * c["head_dim"]),
              "gate_up_proj": (2 * I, H), "down_proj": (H, I)}
    layers = {}
    for li, L in enumerate(model["layers"]):
        d = {"rms_att": L["rms_att"], "rms_ffn": L["rms_ffn"]}
        for name, (r, k) in shapes.items():
            d[name] = (preq2_to_preq(L[name + "_meta"], L[name + "_quant"], r, k).reshape(-1) if preq_blocks
                       else np.zeros(1, np.uint8))
            d[name + "_meta"] = L[name + "_meta"]
            d[name + "_quant"] = L[name + "_quant"]
        layers[li] = d
    os.environ["ASDSL_PREQ2"] = "1"
    return nu.UnifiedEngine(cfg, model["embed_f16"], model["output_norm"], model["embed_f16"], model["cos"],
                            model["sin"], layers)


def load_ref_unified():
    from oracle.oracle import ref_lib_path

    spec = importlib.util.spec_from_file_location("_native_unified", ref_lib_path())
    nu = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(nu)
    return nu


def engine_long() -> None:
    """engine_long.npz: the reference engine's greedy trajectories over 160 steps."""
    from asdsl_b200.inference.synthetic import TINY, build_model, model_digest

    nu = load_ref_unified()
    out = {}
    for seed in (5, 7):
        model = build_model(dict(TINY, max_seq=256), seed=seed, norms_one=False)
        eng = ref_engine(nu, model)
        prompt = [3]
        toks = list(prompt)
        logits = np.array(eng.forward_token(prompt[0], 0), copy=True)
        margins = []
        for _ in range(160):
            srt = np.sort(logits)
            margins.append(float(srt[-1] - srt[-2]))
            toks.append(int(np.argmax(logits)))
            logits = np.array(eng.forward_token(toks[-1], len(toks) - 1), copy=True)
        eng.reset_session()
        assert list(eng.generate(prompt, 160)) == toks
        out[f"s{seed}_digest"] = np.array(model_digest(model))
        out[f"s{seed}_tokens"] = np.array(toks, np.int32)
        out[f"s{seed}_margins"] = np.array(margins)
    np.savez_compressed(os.path.join(OUT, "engine_long.npz"), **out)


def gemm_q4_128() -> None:
    """Prompt GEMM fixture: random Q4_128 blocks (scales in the symmetric quantizer's range, one
    all-zero-scale group) and N(0, 1) activations; batches of 5 and 66 rows (the reference leaves
    y rows 64 and 65 as it found them: the fixture pre-fills them with -1)."""
    from asdsl_b200.quantization.synth import random_q4_128
    from oracle.oracle import RefKernels

    rk = RefKernels()
    rng = np.random.default_rng(20261202)
    M, K = 70, 512
    blocks = random_q4_128(rng, M, K)
    blocks[3, 1, 0:2] = 0  # scale 0.0
    x5 = rng.standard_normal((5, K)).astype(np.float32)
    x66 = rng.standard_normal((66, K)).astype(np.float32)
    y5 = rk.gemm_q4_128_f32(blocks, x5, M, K)
    y66 = rk.gemm_q4_128_f32(blocks, x66, M, K, y=np.full((66, M), -1.0, np.float32))
    np.savez_compressed(os.path.join(OUT, "gemm_q4_128.npz"), blocks=blocks, x5=x5, y5=y5, x66=x66, y66=y66)


def main() -> None:
    ap = argparse.ArgumentParser()
    from oracle.oracle import reference_root

    ap.add_argument("--ref", default=reference_root())
    ap.add_argument("--only", choices=["engine_long", "gemm_q4_128"], default=None)
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    if args.only == "engine_long":
        engine_long()
        print("golden fixture engine_long.npz written to", OUT)
        return
    if args.only == "gemm_q4_128":
        gemm_q4_128()
        print("golden fixture gemm_q4_128.npz written to", OUT)
        return
    from asdsl.quantization import core as rcore
    from asdsl.quantization.repack_preq2 import repack_preq_blocks_to_preq2
    from asdsl.quantization.repack_q4_32 import blocks_to_flat, repack_asymmetric_to_q4_32_blocks
    from asdsl.quantization.repack_q4_128 import (
        repack_asymmetric_to_q4_128_blocks,
        repack_fp32_to_q4_128_blocks,
    )

    from oracle.oracle import RefKernels, ref_lib_path

    rk = RefKernels()
    rng = np.random.default_rng(20261201)

    # ---------------- quantizer ----------------
    w = (rng.standard_normal((32, 256)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0           # degenerate group
    w[5, 32:64] = 1e-7        # tiny constant group
    w[7, 64:96] *= 40.0       # outlier group
    out = {"w": w}
    for tag, sym, opt in (("asym_opt", False, True), ("asym_plain", False, False), ("sym_opt", True, True)):
        qt = rcore.quantize_weights(w, bits=4, group_size=32, symmetric=sym, optimize_clips=opt)
        out[f"{tag}_data"] = qt.data
        out[f"{tag}_scales"] = qt.scales.view(np.uint16)
        if qt.zeros is not None:
            out[f"{tag}_zeros"] = qt.zeros.view(np.uint16)
    np.savez_compressed(os.path.join(OUT, "quant_w32x256.npz"), **out)

    # ---------------- repackers ----------------
    rows, cols = 29, 256
    qt = rcore.quantize_weights(w[:rows], bits=4, group_size=32, symmetric=False, optimize_clips=True)
    sc = qt.scales.astype(np.float32)
    zr = qt.zeros.astype(np.float32)
    bi = (-zr * sc).astype(np.float32)
    preq = repack_asymmetric_to_q4_32_blocks(qt.data, sc, bi, rows, cols, 32)
    flat = blocks_to_flat(preq)
    meta, quant = repack_preq_blocks_to_preq2(flat, rows, cols, 32)
    wf = w[:rows].copy()
    wf[2, 128:256] = 0.0
    b128 = repack_fp32_to_q4_128_blocks(wf, rows, cols, 128)
    qt128 = rcore.quantize_weights(w[:rows], bits=4, group_size=128, symmetric=False, optimize_clips=False)
    sc128 = qt128.scales.astype(np.float32)
    bi128 = (-qt128.zeros.astype(np.float32) * sc128).astype(np.float32)
    a128 = repack_asymmetric_to_q4_128_blocks(qt128.data, sc128, bi128, rows, cols, 128)
    np.savez_compressed(os.path.join(OUT, "repack_29x256.npz"), packed=qt.data, scales=sc, biases=bi,
                        preq=preq, meta=meta, quant=quant, w_f32=wf, q4_128=b128, packed128=qt128.data,
                        scales128=sc128, biases128=bi128, q4_128_asym=a128)

    # ---------------- kernels (compiled reference) ----------------
    K = 512
    x = rng.standard_normal(K).astype(np.float32)
    x[0:32] = 0.0
    x[32:64] = 1e-11
    x[64:96] *= 1e4
    xq32, xs32 = rk.quantize_activation(x, 32)
    xq128, xs128 = rk.quantize_activation(x, 128)
    kern = {"x": x, "xq32": xq32, "xs32": xs32, "xq128": xq128, "xs128": xs128}
    # preq / preq2 from the reference pipeline, ragged rows
    M = 61
    wm = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    q = rcore.quantize_weights(wm, bits=4, group_size=32, symmetric=False, optimize_clips=True)
    s_, z_ = q.scales.astype(np.float32), q.zeros.astype(np.float32)
    b_ = (-z_ * s_).astype(np.float32)
    pq = blocks_to_flat(repack_asymmetric_to_q4_32_blocks(q.data, s_, b_, M, K, 32))
    m2, q2 = repack_preq_blocks_to_preq2(pq, M, K, 32)
    kern.update(preq=pq, meta=m2, quant=q2, packed=q.data, pk_scales=s_, pk_biases=b_)
    kern["y_preq2_fused"] = rk.gemv_preq2_fused(m2, q2, x, M, K)
    kern["y_preq_fused"] = rk.gemv_preq_fused(pq, x, M, K)
    kern["y_preq_q8"] = rk.gemv_preq_q8(pq, xq32, xs32, M, K)
    kern["y_packed"] = rk.gemv_q4_packed(q.data, x, s_, b_, M, K, 32)
    M128 = 37
    w128 = (rng.standard_normal((M128, K)) * 0.02).astype(np.float32)
    blk128 = repack_fp32_to_q4_128_blocks(w128, M128, K, 128)
    kern["q4_128"] = blk128
    kern["y_q4_128"] = rk.gemv_q4_128_q8(blk128, xq128, xs128, M128, K)
    from asdsl_b200.quantization.synth import quantize_s256, random_q4k_bytes

    s256 = quantize_s256((rng.standard_normal((19, K)) * 0.02).astype(np.float32))
    kern["s256"] = s256
    kern["y_s256"] = rk.gemv_s256_q8(s256, xq32, xs32, 19, K)
    q4k = random_q4k_bytes(rng, 23, K)
    kern["q4k"] = q4k
    kern["y_q4k"] = rk.gemv_q4km(q4k, x, 23, K)
    np.savez_compressed(os.path.join(OUT, "kern_small.npz"), **kern)

    # ---------------- tiny engine (compiled reference UnifiedEngine) ----------------
    from asdsl_b200.inference.synthetic import TINY, build_model, model_digest

    nu = load_ref_unified()
    model = build_model(TINY, seed=5, norms_one=False)
    eng = ref_engine(nu, model)
    lm_meta, lm_quant = eng.export_lm_head_preq2()
    prompt = [7]
    steps = 40
    logits0 = np.array(eng.forward_token(prompt[0], 0), copy=True)
    toks = list(prompt)
    logits = logits0
    margins = []
    for t in range(steps):
        srt = np.sort(logits)
        margins.append(float(srt[-1] - srt[-2]))
        nxt = int(np.argmax(logits))
        toks.append(nxt)
        logits = np.array(eng.forward_token(nxt, len(toks) - 1), copy=True)
    eng.reset_session()
    gen = eng.generate(prompt, steps)
    np.savez_compressed(os.path.join(OUT, "engine_tiny.npz"), digest=np.array(model_digest(model)),
                        seed=np.array(5), prompt=np.array(prompt, np.int32), tokens=np.array(toks, np.int32),
                        generate=np.array(gen, np.int32), logits0=logits0, margins=np.array(margins),
                        lm_meta=lm_meta, lm_quant=lm_quant)
    engine_long()
    gemm_q4_128()
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
