"""GPU parity of every GEMV entry point of the C ABI against the CPU oracle
(oracle/asdsl_oracle.c, itself pinned to the reference in test_oracle_golden.py).

Bars: A8 codes/scales and all byte unpacking bit-exact; GEMV outputs within
max|d|/max|y| <= 1e-3 (written here as TOL); argmax index
exact whenever the top-2 margin exceeds the measured logit error."""

import numpy as np
import pytest
import torch

from oracle.oracle import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _status_clean(native):
    assert native.device_status(clear=True) == 0


@pytest.fixture(scope="module")
def ng(native):
    from asdsl_b200.kernels import _native_gemv

    return _native_gemv


def _x(rng, K, special=True):
    x = rng.standard_normal(K).astype(np.float32)
    if special and K >= 128:
        x[0:32] = 0.0          # all-zero group -> scale 1.0
        x[32:64] = 1e-11       # below the 1e-9 floor
        x[64:96] *= 1e3
    return x


def test_a8_bit_exact(native, oracle, golden):
    g = golden("kern_small.npz")
    rng = np.random.default_rng(0)
    for x in (g["x"], _x(rng, 3072), _x(rng, 8192), rng.standard_normal(96).astype(np.float32)):
        for gs in (32, 128):
            if x.size % gs:
                continue
            xd = _dev(x)
            q = torch.empty(x.size, dtype=torch.int8, device="cuda")
            s = torch.empty(x.size // gs, dtype=torch.float32, device="cuda")
            sm = torch.empty(x.size // gs, dtype=torch.int32, device="cuda")
            native.call("asdsl_b200_quantize_activation", xd.data_ptr(), q.data_ptr(), s.data_ptr(), sm.data_ptr(),
                        x.size, gs, None)
            oq, os_, osum = oracle.quantize_activation(x, gs)
            assert np.array_equal(q.cpu().numpy(), oq)
            assert np.array_equal(s.cpu().numpy().view(np.uint32), os_.view(np.uint32))
            assert np.array_equal(sm.cpu().numpy(), osum)
    assert np.array_equal(oracle.quantize_activation(g["x"], 32)[0], g["xq32"])
    _status_clean(native)


def test_a8_numpy_api(ng, oracle):
    rng = np.random.default_rng(1)
    x = _x(rng, 3072)
    q = np.zeros(3072, np.int8)
    s = np.zeros(96, np.float32)
    ng.quantize_activation_avx2(x, q, s, 3072, 32)
    oq, os_, _ = oracle.quantize_activation(x, 32)
    assert np.array_equal(q, oq) and np.array_equal(s, os_)


PREQ2_SHAPES = [(1, 64), (3, 96), (5, 256), (61, 512), (512, 3072), (3072, 8192), (4097, 3072), (16384, 3072)]


@pytest.mark.parametrize("M,K", PREQ2_SHAPES)
def test_preq2_fused(ng, oracle, native, M, K):
    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(M * 7 + K)
    meta, quant = random_preq2(rng, M, K)
    x = _x(rng, K)
    y = np.zeros(M, np.float32)
    ng.gemv_preq2_fused_avx2(meta, quant, x, y, M, K, 32)
    ref = oracle.gemv_preq2_fused(meta, quant, x, M, K)
    assert rel_err(y, ref) < TOL
    # pre-quantized entry on the same bytes
    xq, xs, _ = oracle.quantize_activation(x, 32)
    y2 = np.zeros(M, np.float32)
    ng.gemv_preq2_avx2(meta, quant, xq, xs, y2, M, K, 32)
    assert rel_err(y2, ref) < TOL
    _status_clean(native)


def test_preq2_golden_pipeline(ng, golden):
    g = golden("kern_small.npz")
    M, K = g["y_preq2_fused"].size, g["x"].size
    y = np.zeros(M, np.float32)
    ng.gemv_preq2_fused_avx2(g["meta"], g["quant"], g["x"], y, M, K, 32)
    assert rel_err(y, g["y_preq2_fused"]) < TOL
    y = np.zeros(M, np.float32)
    ng.gemv_q4_32_preq_fused_avx2(g["preq"], g["x"], y, M, K, 32)
    assert rel_err(y, g["y_preq_fused"]) < TOL
    y = np.zeros(M, np.float32)
    ng.gemv_q4_32_preq_avx2(g["preq"], g["xq32"], g["xs32"], y, M, K, 32)
    assert rel_err(y, g["y_preq_q8"]) < TOL


@pytest.mark.parametrize("M,K", [(1, 32), (7, 96), (61, 512), (3072, 3072), (5120, 3072), (3072, 8192)])
def test_preq_blocks(ng, oracle, native, M, K):
    from asdsl_b200.quantization.repack import preq2_to_preq
    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(M + K)
    meta, quant = random_preq2(rng, M, K)
    flat = preq2_to_preq(meta, quant, M, K)
    x = _x(rng, K)
    ref = oracle.gemv_preq_fused(flat, x, M, K)
    y = np.zeros(M, np.float32)
    ng.gemv_q4_32_preq_fused_avx2(flat, x, y, M, K, 32)
    assert rel_err(y, ref) < TOL
    for fn in (ng.gemv_q4_32_preq_4row_avx2, ng.gemv_q4_32_preq_8row_avx2):
        y = np.zeros(M, np.float32)
        fn(flat, x, y, M, K, 32)
        assert rel_err(y, ref) < TOL
    xq, xs, _ = oracle.quantize_activation(x, 32)
    y = np.zeros(M, np.float32)
    ng.gemv_q4_32_preq_avx2(flat, xq, xs, y, M, K, 32)
    assert rel_err(y, oracle.gemv_preq_q8(flat, xq, xs, M, K)) < TOL
    _status_clean(native)


@pytest.mark.parametrize("M,K", [(1, 128), (37, 512), (9, 384), (16384, 3072), (3072, 8192)])
def test_q4_128(ng, oracle, native, M, K):
    from asdsl_b200.quantization.repack import repack_fp32_to_q4_128_blocks

    rng = np.random.default_rng(M * 3 + K)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    if M > 2:
        w[1, :128] = 0.0
    blocks = repack_fp32_to_q4_128_blocks(w, M, K)
    x = _x(rng, K)
    xq, xs, _ = oracle.quantize_activation(x, 128)
    ref = oracle.gemv_q4_128_q8(blocks, xq, xs, M, K)
    y = np.zeros(M, np.float32)
    ng.gemv_q4_128_preq_avx2(blocks, xq, xs, y, M, K, 128)
    assert rel_err(y, ref) < TOL
    yt = torch.empty(M, dtype=torch.float32, device="cuda")
    bd, xd = _dev(blocks), _dev(x)  # keep the device copies alive until the kernel has run
    native.call("asdsl_b200_gemv_q4_128_fused", bd.data_ptr(), xd.data_ptr(), yt.data_ptr(), M, K, None)
    assert rel_err(yt.cpu().numpy(), ref) < TOL
    _status_clean(native)


def test_q4_128_golden(ng, golden):
    g = golden("kern_small.npz")
    M, K = g["y_q4_128"].size, g["x"].size
    y = np.zeros(M, np.float32)
    ng.gemv_q4_128_preq_avx2(g["q4_128"], g["xq128"], g["xs128"], y, M, K, 128)
    assert rel_err(y, g["y_q4_128"]) < TOL


def test_gemm_q4_128_f32_golden(ng, golden, native):
    """gemm_q4_128_q8_avx2 (gemv_q4_128.cpp:262-306): bit-identical to the reference's own outputs
    (tests/golden/gemm_q4_128.npz, an all-zero-scale group included), for 5 batch rows and for 66,
    where the reference computes rows 0..63 and leaves rows 64 and 65 as they were (-1 here)."""
    g = golden("gemm_q4_128.npz")
    M, K = 70, 512
    y5 = np.zeros((5, M), np.float32)
    ng.gemm_q4_128_q8_avx2(g["blocks"], g["x5"], y5, M, K, 128, 5)
    assert np.array_equal(y5, g["y5"])
    y66 = np.full((66, M), -1.0, np.float32)
    ng.gemm_q4_128_q8_avx2(g["blocks"], g["x66"], y66, M, K, 128, 66)
    assert np.array_equal(y66, g["y66"])
    with pytest.raises(ValueError, match="group_size must be 128"):
        ng.gemm_q4_128_q8_avx2(g["blocks"], g["x5"], y5, M, K, 32, 5)
    _status_clean(native)


@pytest.mark.parametrize("M,K,B", [(1000, 3072, 37), (3072, 8192, 64), (16384, 3072, 16), (33, 128, 1)])
def test_gemm_q4_128_f32_vs_oracle(oracle, native, M, K, B):
    """The prompt GEMM at the engine's g128 shapes (gate_up 16384x3072, down 3072x8192) and ragged
    ones (rows not a multiple of the 32-row tile, 1 and 37 batch rows), device tensors in place:
    bit-identical to the oracle restatement of the reference's order."""
    from asdsl_b200 import _lib
    from asdsl_b200.quantization.synth import random_q4_128

    rng = np.random.default_rng(M + K + B)
    blocks = random_q4_128(rng, M, K)
    X = rng.standard_normal((B, K)).astype(np.float32)
    Yd = torch.full((B, M), 7.0, dtype=torch.float32, device="cuda")
    bd, xd = _dev(blocks), _dev(X)  # alive until the kernel has run
    _lib.call("asdsl_b200_gemm_q4_128_f32", bd.data_ptr(), xd.data_ptr(), Yd.data_ptr(), M, K, 128, B,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(Yd.cpu().numpy(), oracle.gemm_q4_128_f32(blocks, X, M, K))
    _status_clean(native)


@pytest.mark.parametrize("M,K", [(19, 512), (8192, 3072), (3072, 8192)])
def test_s256(ng, oracle, native, M, K):
    from asdsl_b200.quantization.synth import quantize_s256

    rng = np.random.default_rng(K + M)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    blocks = quantize_s256(w)
    x = _x(rng, K)
    xq, xs, _ = oracle.quantize_activation(x, 32)
    y = np.zeros(M, np.float32)
    ng.gemv_q4_s256_preq_avx2(blocks, xq, xs, y, M, K, 32)
    assert rel_err(y, oracle.gemv_s256_q8(blocks, xq, xs, M, K)) < TOL
    _status_clean(native)


@pytest.mark.parametrize("M,K", [(23, 512), (8192, 3072), (3072, 8192)])
def test_q4k(ng, oracle, native, golden, M, K):
    from asdsl_b200.kernels import gemv_q4km_q8
    from asdsl_b200.quantization.synth import quantize_q4k, random_q4k_bytes

    rng = np.random.default_rng(M * 11 + K)
    x = _x(rng, K)
    for w in (random_q4k_bytes(rng, M, K), quantize_q4k((rng.standard_normal((M, K)) * 0.02).astype(np.float32))):
        y = gemv_q4km_q8(w, x, M, K)
        assert rel_err(y, oracle.gemv_q4km(w, x, M, K)) < TOL
    g = golden("kern_small.npz")
    y = gemv_q4km_q8(g["q4k"], g["x"], g["y_q4k"].size, g["x"].size)
    assert rel_err(y, g["y_q4k"]) < TOL
    _status_clean(native)


@pytest.mark.parametrize("M,K,gs", [(29, 256, 32), (61, 512, 64), (1024, 3072, 32), (100, 3072, 128), (13, 480, 40)])
def test_packed_fp32(oracle, native, M, K, gs):
    from asdsl_b200.kernels import gemv_q4_packed, gemv_q4_unpacked
    from asdsl_b200.kernels import _native_gemv as ngm
    from asdsl_b200.quantization import core

    rng = np.random.default_rng(M + K + gs)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    qt = core.quantize_weights(w, 4, gs, False, False)
    sc, bi = core.scales_biases_f32(qt)
    x = rng.standard_normal(K).astype(np.float32)
    ref = oracle.gemv_q4_packed(qt.data, x, sc, bi, M, K, gs)
    assert rel_err(gemv_q4_packed(qt.data, x, sc, bi, M, K, gs), ref) < TOL
    X = rng.standard_normal((3, K)).astype(np.float32)
    Y = gemv_q4_packed(qt.data, X, sc, bi, M, K, gs)
    assert Y.shape == (3, M)
    for b in range(3):
        assert rel_err(Y[b], oracle.gemv_q4_packed(qt.data, X[b], sc, bi, M, K, gs)) < TOL
    Yb = np.zeros((3, M), np.float32)
    ngm.matmul_batch_q4(qt.data, sc, bi, X, Yb, M, K, 3, gs)
    assert rel_err(Yb, Y) < TOL
    unpacked = core.unpack_nibbles(qt.data)
    assert rel_err(gemv_q4_unpacked(unpacked, x, sc, bi, M, K, gs), ref) < TOL
    _status_clean(native)


@pytest.mark.parametrize("fmt,M,K", [(0, 61, 512), (0, 200064, 3072), (2, 37, 512), (2, 200064, 3072)])
def test_gemv_argmax(oracle, native, fmt, M, K):
    from asdsl_b200.quantization.repack import repack_fp32_to_q4_128_blocks
    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(M + fmt)
    x = _x(rng, K)
    if fmt == 0:
        meta, quant = random_preq2(rng, M, K)
        w0, w1 = _dev(meta), _dev(quant)
        ref = oracle.gemv_preq2_fused(meta, quant, x, M, K)
    else:
        blocks = repack_fp32_to_q4_128_blocks((rng.standard_normal((M, K)) * 0.02).astype(np.float32), M, K)
        w0, w1 = _dev(blocks), None
        ref = oracle.gemv_q4_128_fused(blocks, x, M, K)
    scratch = torch.zeros(native.load().asdsl_b200_argmax_scratch_bytes(), dtype=torch.uint8, device="cuda")
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    ov = torch.empty(1, dtype=torch.float32, device="cuda")
    oi = torch.empty(1, dtype=torch.int32, device="cuda")
    xd = _dev(x)
    for rep in range(2):  # twice: the scratch counter must re-arm itself
        native.call("asdsl_b200_gemv_argmax", fmt, w0.data_ptr(), None if w1 is None else w1.data_ptr(),
                    xd.data_ptr(), y.data_ptr(), ov.data_ptr(), oi.data_ptr(), 1000 * rep,
                    scratch.data_ptr(), scratch.numel(), M, K, None)
        yh = y.cpu().numpy()
        assert rel_err(yh, ref) < TOL
        i = int(oi.item()) - 1000 * rep
        assert i == int(np.argmax(yh))                 # exact first-max on the device logits
        assert float(ov.item()) == float(yh[i])
        srt = np.sort(ref)
        if srt[-1] - srt[-2] > 4 * TOL * np.abs(ref).max():
            assert i == oracle.argmax(ref)
    _status_clean(native)


@pytest.mark.parametrize("fmt,I,K", [(0, 64, 256), (0, 8192, 3072), (2, 40, 512), (2, 8192, 3072)])
def test_gateup_silu(oracle, native, fmt, I, K):
    from asdsl_b200.quantization.repack import repack_fp32_to_q4_128_blocks
    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(I + K + fmt)
    x = _x(rng, K)
    if fmt == 0:
        meta, quant = random_preq2(rng, 2 * I, K)
        gu = oracle.gemv_preq2_fused(meta, quant, x, 2 * I, K)
        w0, w1 = _dev(meta), _dev(quant)
    else:
        blocks = repack_fp32_to_q4_128_blocks((rng.standard_normal((2 * I, K)) * 0.02).astype(np.float32), 2 * I, K)
        gu = oracle.gemv_q4_128_fused(blocks, x, 2 * I, K)
        w0, w1 = _dev(blocks), None
    ref = oracle.swiglu(gu[:I], gu[I:])
    h = torch.empty(I, dtype=torch.float32, device="cuda")
    xd = _dev(x)
    native.call("asdsl_b200_gateup_silu", fmt, w0.data_ptr(), None if w1 is None else w1.data_ptr(),
                xd.data_ptr(), h.data_ptr(), I, K, None)
    assert rel_err(h.cpu().numpy(), ref) < TOL
    _status_clean(native)


def test_config0_reference_pipeline(ng, oracle, native):
    """Config 0 exactly: N(0,0.02) seed 0, reference quantizer (asym gs32, clip search)
    -> preq -> preq2, x ~ N(0,1) drawn after W."""
    from asdsl_b200.quantization import core, repack

    M, K = 16384, 3072
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    qt = core.quantize_weights(w, 4, 32, False, True)
    sc, bi = core.scales_biases_f32(qt)
    flat = repack.blocks_to_flat(repack.repack_asymmetric_to_q4_32_blocks(qt.data, sc, bi, M, K, 32))
    meta, quant = repack.repack_preq_blocks_to_preq2(flat, M, K)
    x = rng.standard_normal(K).astype(np.float32)
    y = np.zeros(M, np.float32)
    ng.gemv_preq2_fused_avx2(meta, quant, x, y, M, K, 32)
    assert rel_err(y, oracle.gemv_preq2_fused(meta, quant, x, M, K)) < TOL
    y2 = np.zeros(M, np.float32)
    ng.gemv_q4_32_preq_fused_avx2(flat, x, y2, M, K, 32)
    assert rel_err(y2, oracle.gemv_preq_fused(flat, x, M, K)) < TOL
    _status_clean(native)


def test_torch_tensor_path_no_copies(native):
    """CUDA tensors are used in place on the current stream."""
    from asdsl_b200.kernels import _native_gemv as ngm
    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(9)
    meta, quant = random_preq2(rng, 256, 1024)
    m, q = _dev(meta), _dev(quant)
    x = torch.randn(1024, device="cuda")
    y = torch.zeros(256, device="cuda")
    ptr = y.data_ptr()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ngm.gemv_preq2_fused_avx2(m, q, x, y, 256, 1024, 32)
    s.synchronize()
    assert y.data_ptr() == ptr and torch.isfinite(y).all() and y.abs().sum() > 0


def test_errors_on_device_path(ng):
    with pytest.raises(ValueError):
        ng.gemv_preq2_fused_avx2(np.zeros(64, np.uint8), np.zeros(64, np.uint8), np.zeros(64, np.float32),
                                 np.zeros(4, np.float32), 4, 64, 64)


@pytest.mark.parametrize("M,K", [(1, 128), (61, 384), (16384, 3072), (3072, 8192)])
def test_q4_128_banded_relayout_and_gemv(oracle, native, M, K):
    """Device re-layout is byte-exact; banded GEMV / argmax / SiLU match the oracle on the raw blocks."""
    from asdsl_b200.layer import relayout_q4_128
    from asdsl_b200.quantization.repack import q4_128_to_banded, repack_fp32_to_q4_128_blocks

    rng = np.random.default_rng(M + 5 * K)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    blocks = repack_fp32_to_q4_128_blocks(w, M, K)
    bd = _dev(blocks)
    q, s = relayout_q4_128(bd, M, K)
    hq, hs = q4_128_to_banded(blocks, M, K)
    assert np.array_equal(q.cpu().numpy(), hq) and np.array_equal(s.cpu().numpy(), hs)
    x = _x(rng, K)
    xd = _dev(x)
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    native.call("asdsl_b200_gemv_q4_128_banded", q.data_ptr(), s.data_ptr(), xd.data_ptr(), y.data_ptr(), M, K, None)
    ref = oracle.gemv_q4_128_fused(blocks, x, M, K)
    assert rel_err(y.cpu().numpy(), ref) < TOL
    scratch = torch.zeros(native.load().asdsl_b200_argmax_scratch_bytes(), dtype=torch.uint8, device="cuda")
    ov = torch.empty(1, dtype=torch.float32, device="cuda")
    oi = torch.empty(1, dtype=torch.int32, device="cuda")
    native.call("asdsl_b200_gemv_argmax", 4, q.data_ptr(), s.data_ptr(), xd.data_ptr(), y.data_ptr(), ov.data_ptr(),
                oi.data_ptr(), 0, scratch.data_ptr(), scratch.numel(), M, K, None)
    yh = y.cpu().numpy()
    assert int(oi.item()) == int(np.argmax(yh)) and rel_err(yh, ref) < TOL
    if M % 8 == 0:
        I = M // 2
        h = torch.empty(I, dtype=torch.float32, device="cuda")
        native.call("asdsl_b200_gateup_silu", 4, q.data_ptr(), s.data_ptr(), xd.data_ptr(), h.data_ptr(), I, K, None)
        assert rel_err(h.cpu().numpy(), oracle.swiglu(ref[:I], ref[I:])) < TOL
    _status_clean(native)


def test_layer_projection_set_matches_oracle(native, oracle):
    """Config-1-shaped layer chain (small seeded weights through the same pipeline) vs the oracle."""
    from asdsl_b200.layer import build_c1_host, from_host, layer_reference

    import torch

    cfg = dict(hidden=512, qkv_rows=768, q_dim=512, inter=1024)
    host = build_c1_host(7, cfg)
    L = from_host(host)
    ref = layer_reference(oracle, host)
    x2 = (np.random.default_rng(3).standard_normal(cfg["hidden"]) * 0.5).astype(np.float32)
    for rep in range(2):  # the native host-buffer call twice (graph captured on the first)
        out = L.forward(host["x"])
        for k in ("qkv", "o", "y"):
            assert rel_err(out[k], ref[k]) < TOL, k
        # another input in between: the staging carries nothing over from call to call
        out2 = L.forward(x2)
        # the same kernels enqueued from Python on torch's stream give the same bits
        L.step(torch.from_numpy(x2).cuda())
        torch.cuda.synchronize()
        for k, t in (("qkv", L.qkv_out), ("o", L.o_out), ("y", L.y)):
            assert np.array_equal(out2[k].view(np.uint32), t.cpu().numpy().view(np.uint32)), k
    with pytest.raises(ValueError):
        L.forward(np.zeros(3, np.float32))
    L.close()
    _status_clean(native)


def test_zero_copy_transfers(native):
    """asdsl_b200_host_to_device / _device_to_host: exact round trips through pinned host memory
    for sizes with and without a 4-float tail, twice in a row; pageable host memory is refused."""
    import torch

    lib = native.load()
    s = torch.cuda.Stream()
    for n in (1, 7, 3072, 11264 + 3):
        src = torch.from_numpy(np.random.default_rng(n).standard_normal(n).astype(np.float32)).pin_memory()
        back = torch.zeros(n, dtype=torch.float32).pin_memory()
        dev = torch.empty(n, dtype=torch.float32, device="cuda")
        for _ in range(2):
            native.check(lib.asdsl_b200_host_to_device(src.data_ptr(), dev.data_ptr(), n, s.cuda_stream), "h2d")
            native.check(lib.asdsl_b200_device_to_host(dev.data_ptr(), back.data_ptr(), n, s.cuda_stream), "d2h")
            s.synchronize()
            assert np.array_equal(back.numpy().view(np.uint32), src.numpy().view(np.uint32)), n
            src.mul_(-1.0)
    pageable = np.zeros(16, np.float32)
    dev = torch.empty(16, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        native.call("asdsl_b200_host_to_device", pageable.ctypes.data, dev.data_ptr(), 16, None)
    # a buffer off the 16-byte grid is refused before any launch (the kernels move float4s)
    pinned = torch.zeros(16, dtype=torch.float32).pin_memory()
    with pytest.raises(ValueError, match="16-byte aligned"):
        native.call("asdsl_b200_host_to_device", pinned.data_ptr(), dev.data_ptr() + 4, 8, None)
    _status_clean(native)
