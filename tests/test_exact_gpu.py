"""GPU parity of the reference-exact numerics mode: bit-identical to the reference's compiled code.

The reference-exact mode runs every op of the decode step in the operation order of the
reference's g++ -O3 -ffast-math build (asdsl/kernels/native/unified_engine.cpp:1339-1688,
gemv_preq2_avx2.cpp:216-253), with the host CPU's RSQRTSS / RCPPS estimates and the C library's
expf captured as tables.  Bar: bitwise equality of every output -- GEMV rows, RMSNorm+GEMV,
gate_up+SiLU, expf, logits -- against the CPU oracle (oracle/asdsl_oracle.c, itself bitwise equal
to the reference engine: tests/test_oracle_exact.py) and, where oracle/_ref is present, against
the reference's own compiled kernels and engine; greedy trajectories identical for >= 64 steps on
the full 32-layer random-init Phi-4-mini model of config 3."""

import ctypes

import numpy as np
import pytest

from oracle.oracle import OracleEngine, RefKernels, ref_lib_path

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _assert_bitwise(got, want, what):
    g, w = _bits(got), _bits(want)
    if not np.array_equal(g, w):
        bad = np.nonzero(g != w)[0]
        raise AssertionError(f"{what}: {bad.size} of {g.size} differ, first {bad[:5]}: "
                             f"{np.asarray(got)[bad[:3]]} vs {np.asarray(want)[bad[:3]]}")


# row counts chosen to cover every unit width (1, 2, 4 and 8 bands; partial last units)
@pytest.mark.parametrize("M,K", [(6, 64), (33, 1024), (5120, 3072), (3072, 3072), (8190, 3072), (16384, 3072),
                                 (3072, 8192), (30001, 512), (200064, 3072)])
def test_gemv_preq2_exact_bitwise(native, oracle, M, K):
    import torch

    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(M * 7 + K)
    meta, quant = random_preq2(rng, M, K)
    x = (rng.standard_normal(K) * 3).astype(np.float32)
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    md, qd, xd = _dev(meta), _dev(quant), _dev(x)
    native.call("asdsl_b200_gemv_preq2_fused_exact", md.data_ptr(), qd.data_ptr(), xd.data_ptr(), None,
                ctypes.c_float(0.0), y.data_ptr(), M, K, None)
    got = y.cpu().numpy()
    _assert_bitwise(got, oracle.gemv_preq2_fused(meta, quant, x, M, K), "exact GEMV vs oracle")
    if ref_lib_path():
        _assert_bitwise(got, RefKernels().gemv_preq2_fused(meta, quant, x, M, K), "exact GEMV vs reference kernel")
    assert native.device_status(clear=True) == 0


@pytest.mark.parametrize("M,K", [(5120, 3072), (200, 8192)])
def test_rmsnorm_gemv_exact_bitwise(native, oracle, M, K):
    import torch

    from asdsl_b200.quantization.synth import random_preq2
    from oracle.oracle import _I, _p

    rng = np.random.default_rng(K + 1)
    meta, quant = random_preq2(rng, M, K)
    x = (rng.standard_normal(K) * 40).astype(np.float32)
    w = rng.uniform(0.8, 1.2, K).astype(np.float32)
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    md, qd, xd, wd = _dev(meta), _dev(quant), _dev(x), _dev(w)
    native.call("asdsl_b200_gemv_preq2_fused_exact", md.data_ptr(), qd.data_ptr(), xd.data_ptr(), wd.data_ptr(),
                ctypes.c_float(1e-5), y.data_ptr(), M, K, None)
    h = np.zeros(K, np.float32)
    oracle.lib.or_rmsnorm(_p(h), _p(x), _p(w), _I(K), ctypes.c_float(1e-5))
    _assert_bitwise(y.cpu().numpy(), oracle.gemv_preq2_fused(meta, quant, h, M, K), "RMSNorm + GEMV")
    assert native.device_status(clear=True) == 0


@pytest.mark.parametrize("I,K,norm", [(8192, 3072, True), (512, 1024, False)])
def test_gateup_silu_exact_bitwise(native, oracle, I, K, norm):
    import torch

    from asdsl_b200.quantization.synth import random_preq2
    from oracle.oracle import _I, _p

    rng = np.random.default_rng(I + K)
    meta, quant = random_preq2(rng, 2 * I, K)
    x = (rng.standard_normal(K) * 20).astype(np.float32)
    w = rng.uniform(0.8, 1.2, K).astype(np.float32)
    h = torch.empty(I, dtype=torch.float32, device="cuda")
    md, qd, xd, wd = _dev(meta), _dev(quant), _dev(x), _dev(w)
    native.call("asdsl_b200_gateup_silu_exact", md.data_ptr(), qd.data_ptr(), xd.data_ptr(),
                wd.data_ptr() if norm else None, ctypes.c_float(1e-5), h.data_ptr(), I, K, None)
    xin = x
    if norm:
        xin = np.zeros(K, np.float32)
        oracle.lib.or_rmsnorm(_p(xin), _p(x), _p(w), _I(K), ctypes.c_float(1e-5))
    gu = oracle.gemv_preq2_fused(meta, quant, xin, 2 * I, K)
    _assert_bitwise(h.cpu().numpy(), oracle.swiglu(gu[:I], gu[I:]), "gate_up + SiLU")
    assert native.device_status(clear=True) == 0


def test_exact_expf_matches_c_library(native, oracle):
    """The attention's expf on 64M inputs: every listed exception, a dense sweep near 0 (where the
    C library's misrounded inputs cluster) and uniform inputs down to full underflow."""
    import torch

    n_exc = ctypes.c_int(0)
    native.call("asdsl_b200_exact_numerics_init", ctypes.byref(n_exc))
    exc = np.zeros(2 * n_exc.value, np.uint32)
    native.call("asdsl_b200_exact_host_tables", None, None, exc.ctypes.data, n_exc.value, ctypes.byref(n_exc))
    rng = np.random.default_rng(9)
    parts = [exc[0::2].view(np.float32),
             np.arange(0x80000000, 0x80000000 + (1 << 25), dtype=np.uint64).astype(np.uint32).view(np.float32)[::-1],
             (-rng.uniform(0, 0.05, 1 << 24)).astype(np.float32),
             (-rng.uniform(0, 110, 1 << 24)).astype(np.float32)]
    x = np.ascontiguousarray(np.concatenate(parts))
    want = oracle.expf_array(x)
    xd = _dev(x)
    y = torch.empty_like(xd)
    native.call("asdsl_b200_exact_expf", xd.data_ptr(), y.data_ptr(), ctypes.c_longlong(x.size), None)
    _assert_bitwise(y.cpu().numpy(), want, "device expf vs the C library's expf")


def _engine(model, **kw):
    from asdsl_b200.kernels._native_unified import engine_from_model

    return engine_from_model(model, numerics="reference_exact", **kw)


def test_engine_exact_tiny_fixture_bitwise(native, oracle, golden):
    from asdsl_b200.inference.synthetic import TINY, build_model

    g = golden("engine_tiny.npz")
    model = build_model(TINY, seed=int(g["seed"]), norms_one=False)
    eng = _engine(model)
    try:
        _assert_bitwise(eng.forward_token(int(g["prompt"][0]), 0), g["logits0"], "TINY logits vs reference engine")
        eng.reset_session()
        n_new = len(g["tokens"]) - len(g["prompt"])
        assert eng.generate([int(t) for t in g["prompt"]], n_new) == [int(t) for t in g["tokens"]]
    finally:
        eng.close()
    g = golden("engine_long.npz")
    for seed in (5, 7):
        model = build_model(dict(TINY, max_seq=256), seed=seed, norms_one=False)
        eng = _engine(model)
        try:
            assert eng.generate([3], 160) == [int(t) for t in g[f"s{seed}_tokens"]]
        finally:
            eng.close()
    assert native.device_status(clear=True) == 0


def test_engine_exact_small_logits_bitwise_and_batch_paths(native, oracle):
    """SMALL (4 layers, GQA 6/2): 40 free-running steps bitwise equal to the oracle engine's
    logits (hence argmax); forward_batch / verify in this mode give the same rows."""
    from asdsl_b200.inference.synthetic import SMALL, build_model

    model = build_model(SMALL, seed=11, norms_one=False)
    c = model["config"]
    model["lm_meta"], model["lm_quant"] = oracle.lmhead_quant_preq2(model["embed_f16"], c["vocab"], c["hidden"])
    ref = OracleEngine(model, oracle)
    eng = _engine(model)
    try:
        toks = [3]
        rows = []
        for pos in range(40):
            lo = ref.forward_token(toks[-1], pos)
            la = eng.forward_token(toks[-1], pos).copy()
            _assert_bitwise(la, lo, f"SMALL logits at step {pos}")
            rows.append(la)
            toks.append(int(np.argmax(lo)))
        eng.reset_session()
        allr = np.asarray(eng.forward_batch_all_logits(toks[:8], 0)).reshape(8, -1)
        for i in range(8):
            _assert_bitwise(allr[i], rows[i], f"forward_batch_all_logits row {i}")
    finally:
        ref.close()
        eng.close()
    assert native.device_status(clear=True) == 0


def test_engine_exact_config3_greedy_trajectory(native, oracle):
    """Config 3: the full 32-layer random-init Phi-4-mini model (seed 3; every projection N(0, 0.02)
    through the reference's C0 weight pipeline on the device; tied fp16 embedding quantized by
    the engine), one prompt token, 72 greedy steps.  The tokens equal the reference UnifiedEngine's
    (oracle/_ref, on the host cores; the oracle engine when the reference is not built), and the
    first step's logits are bitwise equal."""
    from asdsl_b200.inference.synthetic import PHI4_MINI, build_model_device, model_to_host

    steps = 72
    cfg = dict(PHI4_MINI, max_seq=256)
    dmodel = build_model_device(cfg, seed=3, norms_one=True, quantized=True)
    hmodel = model_to_host(dmodel)
    eng = _engine(dmodel)
    try:
        logits0 = eng.forward_token(3, 0).copy()
        eng.reset_session()
        got = eng.generate([3], steps)
    finally:
        eng.close()
        del dmodel
    c = hmodel["config"]
    if ref_lib_path():
        from tests.golden.make_golden import load_ref_unified, ref_engine

        ref = ref_engine(load_ref_unified(), hmodel, preq_blocks=False)
        want_logits0 = np.array(ref.forward_token(3, 0), copy=True)
        ref.reset_session()
        want = [int(t) for t in ref.generate([3], steps)]
    else:
        hmodel["lm_meta"], hmodel["lm_quant"] = oracle.lmhead_quant_preq2(hmodel["embed_f16"], c["vocab"], c["hidden"])
        ref = OracleEngine(hmodel, oracle)
        want_logits0 = ref.forward_token(3, 0)
        ref.close()
        ref = OracleEngine(hmodel, oracle)
        want, _ = ref.generate([3], steps)
        ref.close()
    _assert_bitwise(logits0, want_logits0, "config-3 first-step logits")
    first_diff = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), None)
    assert got == want, f"config-3 greedy tokens differ from step {first_diff}"
    assert native.device_status(clear=True) == 0


def test_engine_exact_generate_across_long_cache_boundary(native, oracle):
    """generate() across position 256, where the engine switches from the single-CTA attention
    graph to the split (head x 128-position chunk) one: 300 greedy tokens on a TINY-shaped model
    with a 512-position cache equal the oracle engine's, and so do the logits at positions 255,
    256 and 299 (teacher-forced on those tokens)."""
    from asdsl_b200.inference.synthetic import TINY, build_model

    model = build_model(dict(TINY, max_seq=512), seed=21, norms_one=False)
    c = model["config"]
    model["lm_meta"], model["lm_quant"] = oracle.lmhead_quant_preq2(model["embed_f16"], c["vocab"], c["hidden"])
    ref = OracleEngine(model, oracle)
    want, _ = ref.generate([5], 300)
    ref.close()
    eng = _engine(model)
    try:
        got = eng.generate([5], 300)
        assert got == [int(t) for t in want]
        eng.reset_session()
        ref = OracleEngine(model, oracle)
        for pos in range(300):
            lo = ref.forward_token(int(want[pos]), pos)
            la = eng.forward_token(int(want[pos]), pos)
            if pos in (255, 256, 299):
                _assert_bitwise(la, lo, f"logits at position {pos}")
        ref.close()
    finally:
        eng.close()
    assert native.device_status(clear=True) == 0
