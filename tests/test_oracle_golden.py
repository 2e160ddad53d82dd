"""Pins the CPU oracle (oracle/asdsl_oracle.c) against outputs of the reference itself
(tests/golden/*.npz, written by tests/golden/make_golden.py from the reference's
compiled kernels and UnifiedEngine).  CPU only."""

import numpy as np
import pytest

from oracle.oracle import OracleEngine, RefKernels, ref_lib_path, rel_err

TOL = 1e-3  # max|d|/max|y| (north-star GEMV tolerance); observed ~1e-7


def test_a8_bit_exact_vs_reference(oracle, golden):
    g = golden("kern_small.npz")
    xq, xs, xsum = oracle.quantize_activation(g["x"], 32)
    assert np.array_equal(xq, g["xq32"])
    assert np.array_equal(xs.view(np.uint32), g["xs32"].view(np.uint32))
    assert np.array_equal(xsum, g["xq32"].reshape(-1, 32).astype(np.int32).sum(1))
    xq, xs, _ = oracle.quantize_activation(g["x"], 128)
    assert np.array_equal(xq, g["xq128"])
    assert np.array_equal(xs.view(np.uint32), g["xs128"].view(np.uint32))
    # degenerate groups: all-zero and sub-1e-9 groups -> codes 0, scale 1.0
    assert (g["xs32"][:2] == 1.0).all() and not g["xq32"][:64].any()


def test_gemv_formats_vs_reference(oracle, golden):
    g = golden("kern_small.npz")
    K = g["x"].size
    M = g["y_preq2_fused"].size
    # the engine's GEMV: restated in the compiled order, bit-exact
    assert np.array_equal(oracle.gemv_preq2_fused(g["meta"], g["quant"], g["x"], M, K).view(np.uint32),
                          g["y_preq2_fused"].view(np.uint32))
    assert rel_err(oracle.gemv_preq_fused(g["preq"], g["x"], M, K), g["y_preq_fused"]) < 1e-5
    assert rel_err(oracle.gemv_preq_q8(g["preq"], g["xq32"], g["xs32"], M, K), g["y_preq_q8"]) < 1e-5
    assert rel_err(oracle.gemv_q4_packed(g["packed"], g["x"], g["pk_scales"], g["pk_biases"], M, K, 32),
                   g["y_packed"]) < 1e-5
    m = g["y_q4_128"].size
    assert rel_err(oracle.gemv_q4_128_q8(g["q4_128"], g["xq128"], g["xs128"], m, K), g["y_q4_128"]) < 1e-5
    m = g["y_s256"].size
    assert rel_err(oracle.gemv_s256_q8(g["s256"], g["xq32"], g["xs32"], m, K), g["y_s256"]) < 1e-5
    m = g["y_q4k"].size
    assert rel_err(oracle.gemv_q4km(g["q4k"], g["x"], m, K), g["y_q4k"]) < 1e-5


def test_gemm_q4_128_f32_vs_reference(oracle, golden):
    """The prompt GEMM restatement (gemm_q4_128_q8_avx2, gemv_q4_128.cpp:262-306) reproduces the
    reference's outputs bit for bit, rows >= 64 of a 66-row batch untouched, gs != 128 rejected."""
    g = golden("gemm_q4_128.npz")
    M, K = 70, 512
    assert np.array_equal(oracle.gemm_q4_128_f32(g["blocks"], g["x5"], M, K), g["y5"])
    y66 = oracle.gemm_q4_128_f32(g["blocks"], g["x66"], M, K, y=np.full((66, M), -1.0, np.float32))
    assert np.array_equal(y66, g["y66"]) and (y66[64:] == -1.0).all()
    with pytest.raises(ValueError):
        oracle.gemm_q4_128_f32(g["blocks"], g["x5"], M, K, gs=32)


def test_engine_tiny_vs_reference_engine(oracle, golden):
    from asdsl_b200.inference.synthetic import TINY, build_model, model_digest

    g = golden("engine_tiny.npz")
    model = build_model(TINY, seed=int(g["seed"]), norms_one=False)
    assert model_digest(model) == str(g["digest"]), "synthetic model generator drifted from the fixture"
    c = model["config"]
    meta, quant = oracle.lmhead_quant_preq2(model["embed_f16"], c["vocab"], c["hidden"])
    assert np.array_equal(meta, g["lm_meta"]) and np.array_equal(quant, g["lm_quant"])
    model["lm_meta"], model["lm_quant"] = meta, quant
    eng = OracleEngine(model, oracle)
    try:
        # bit-exact: the oracle engine restates the reference's compiled operation order
        assert np.array_equal(eng.forward_token(int(g["prompt"][0]), 0).view(np.uint32), g["logits0"].view(np.uint32))
    finally:
        eng.close()
    eng = OracleEngine(model, oracle)
    try:
        toks, _ = eng.generate(list(g["prompt"]), len(g["tokens"]) - len(g["prompt"]))
    finally:
        eng.close()
    assert list(toks) == list(g["tokens"])
    assert list(g["tokens"]) == list(g["generate"])  # reference: forward_token loop == generate()


@pytest.mark.skipif(ref_lib_path() is None, reason="oracle/_ref not built (reference sources absent)")
def test_oracle_vs_live_reference_random(oracle):
    """Same check on fresh random shapes, against the reference compiled in oracle/_ref."""
    from asdsl_b200.quantization.synth import random_preq2, random_q4k_bytes
    from asdsl_b200.quantization.repack import preq2_to_preq

    rk = RefKernels()
    rng = np.random.default_rng(3)
    for M, K in ((5, 64), (33, 1024), (129, 3072)):
        x = rng.standard_normal(K).astype(np.float32)
        meta, quant = random_preq2(rng, M, K)
        assert np.array_equal(oracle.gemv_preq2_fused(meta, quant, x, M, K).view(np.uint32),
                              rk.gemv_preq2_fused(meta, quant, x, M, K).view(np.uint32))
        flat = preq2_to_preq(meta, quant, M, K)
        assert rel_err(oracle.gemv_preq_fused(flat, x, M, K), rk.gemv_preq_fused(flat, x, M, K)) < TOL
        xq, xs = rk.quantize_activation(x, 32)
        oq, os_, _ = oracle.quantize_activation(x, 32)
        assert np.array_equal(xq, oq) and np.array_equal(xs, os_)
        if K % 256 == 0:
            w = random_q4k_bytes(rng, M, K)
            assert rel_err(oracle.gemv_q4km(w, x, M, K), rk.gemv_q4km(w, x, M, K)) < TOL
        if K % 128 == 0:
            from asdsl_b200.quantization.synth import random_q4_128

            blk = random_q4_128(rng, M, K)
            X = rng.standard_normal((3, K)).astype(np.float32)
            assert np.array_equal(oracle.gemm_q4_128_f32(blk, X, M, K), rk.gemm_q4_128_f32(blk, X, M, K))


def test_oracle_engine_long_trajectories_vs_reference(oracle, golden):
    """160 greedy steps of the oracle engine equal the reference engine's (engine_long.npz)."""
    from asdsl_b200.inference.synthetic import TINY, build_model, model_digest

    g = golden("engine_long.npz")
    for seed in (5, 7):
        model = build_model(dict(TINY, max_seq=256), seed=seed, norms_one=False)
        assert model_digest(model) == str(g[f"s{seed}_digest"])
        c = model["config"]
        model["lm_meta"], model["lm_quant"] = oracle.lmhead_quant_preq2(model["embed_f16"], c["vocab"], c["hidden"])
        eng = OracleEngine(model, oracle)
        try:
            toks, _ = eng.generate([3], 160)
        finally:
            eng.close()
        assert toks == [int(t) for t in g[f"s{seed}_tokens"]]
