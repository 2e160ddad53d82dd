"""Device-side weight preparation (asdsl_b200.quantization.device) against the reference's bytes
(tests/golden, made by the reference's own quantizer and repackers) and against the host
restatement (asdsl_b200.quantization.core / repack, pinned by the same goldens) on larger and edge
inputs: all comparisons are byte-exact."""

import numpy as np
import pytest

from asdsl_b200.quantization import core, repack

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev(native):
    import torch

    from asdsl_b200.quantization import device

    assert torch.cuda.is_available()
    return device


def _t(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _np(t):
    return t.cpu().numpy()


def _same_qt(qd, qh):
    assert np.array_equal(_np(qd.data), qh.data)
    assert np.array_equal(_np(qd.scales).view(np.uint16), qh.scales.view(np.uint16))
    if qh.zeros is None:
        assert qd.zeros is None
    else:
        assert np.array_equal(_np(qd.zeros).view(np.uint16), qh.zeros.view(np.uint16))


def test_quantize_weights_device_matches_reference_golden(dev, golden):
    g = golden("quant_w32x256.npz")
    w = _t(g["w"])
    for tag, sym, opt in (("asym_opt", False, True), ("asym_plain", False, False), ("sym_opt", True, True)):
        qt = dev.quantize_weights_device(w, bits=4, group_size=32, symmetric=sym, optimize_clips=opt)
        assert np.array_equal(_np(qt.data), g[f"{tag}_data"]), tag
        assert np.array_equal(_np(qt.scales).view(np.uint16), g[f"{tag}_scales"]), tag
        if not sym:
            assert np.array_equal(_np(qt.zeros).view(np.uint16), g[f"{tag}_zeros"]), tag


def _edge_weights(rng, rows, cols):
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[1] = 0.0                                    # all-zero groups
    w[2] = 0.0123                                 # constant groups
    w[3, 5] = 3.0                                 # an outlier that drives the clip search
    w[4] *= 1e-6                                  # tiny ranges (the 1e-5 / 1e-4 floors)
    w[5] = np.float32(-0.5) + np.arange(cols, dtype=np.float32) * np.float32(1e-3)  # ramps
    return w


@pytest.mark.parametrize("gs", [32, 64, 128])
@pytest.mark.parametrize("sym,opt", [(False, True), (False, False), (True, True), (True, False)])
def test_quantize_weights_device_matches_host(dev, gs, sym, opt):
    rng = np.random.default_rng(100 + gs)
    w = _edge_weights(rng, 24, 1024)
    qh = core.quantize_weights(w, 4, gs, sym, opt)
    qd = dev.quantize_weights_device(_t(w), 4, gs, sym, opt)
    _same_qt(qd, qh)


def test_quantize_weights_device_ragged_numel(dev):
    """numel not a multiple of the group size: the last group is zero-padded like the reference."""
    rng = np.random.default_rng(7)
    w = (rng.standard_normal(1000) * 0.05).astype(np.float32)
    for gs in (32, 128):
        _same_qt(dev.quantize_weights_device(_t(w), 4, gs, False, True), core.quantize_weights(w, 4, gs, False, True))


def _host_preq2(w, rows, cols):
    qt = core.quantize_weights(w, 4, 32, False, True)
    sc, bi = core.scales_biases_f32(qt)
    blocks = repack.repack_asymmetric_to_q4_32_blocks(qt.data, sc, bi, rows, cols, 32)
    meta, quant = repack.repack_preq_blocks_to_preq2(repack.blocks_to_flat(blocks), rows, cols, 32)
    return qt, meta.reshape(-1), quant.reshape(-1)


@pytest.mark.parametrize("rows,cols", [(29, 256), (64, 3072)])
def test_prepare_preq2_device_matches_host_pipeline(dev, rows, cols):
    rng = np.random.default_rng(rows)
    w = _edge_weights(rng, rows, cols)
    qh, mh, nh = _host_preq2(w, rows, cols)
    md, nd = dev.prepare_preq2_device(_t(w))
    assert np.array_equal(_np(md), mh)
    assert np.array_equal(_np(nd), nh)
    # symmetric tensors take bias = -7.5 * scale
    qs = core.quantize_weights(w, 4, 32, True, True)
    sc, bi = core.scales_biases_f32(qs)
    blocks = repack.repack_asymmetric_to_q4_32_blocks(qs.data, sc, bi, rows, cols, 32)
    ms, ns = repack.repack_preq_blocks_to_preq2(repack.blocks_to_flat(blocks), rows, cols, 32)
    md2, nd2 = dev.repack_preq2_device(dev.quantize_weights_device(_t(w), 4, 32, True, True), rows, cols)
    assert np.array_equal(_np(md2), ms.reshape(-1)) and np.array_equal(_np(nd2), ns.reshape(-1))


def test_q4_128_device_matches_reference_golden(dev, golden):
    g = golden("repack_29x256.npz")
    out = dev.repack_fp32_to_q4_128_device(_t(g["w_f32"]), 29, 256)
    assert np.array_equal(_np(out), g["q4_128"])


def test_q4_128_device_matches_host(dev):
    rng = np.random.default_rng(3)
    w = _edge_weights(rng, 40, 3072)
    w[6, 128:256] = 1e-13                         # amax < 1e-12: scale 0, nibbles 0x88
    out = dev.repack_fp32_to_q4_128_device(_t(w), 40, 3072)
    assert np.array_equal(_np(out), repack.repack_fp32_to_q4_128_blocks(w, 40, 3072, 128))


def test_requant_q4_128_device_matches_host(dev):
    """C0.1: gs-32 asymmetric weights dequantized (q*scale + bias, float32) and requantized at g128."""
    rng = np.random.default_rng(11)
    rows, cols = 48, 1024
    w = _edge_weights(rng, rows, cols)
    qh = core.quantize_weights(w, 4, 32, False, True)
    sc, bi = core.scales_biases_f32(qh)
    ref = repack.repack_fp32_to_q4_128_blocks(core.dequant_packed_projection(qh.data, sc, bi, rows, cols, 32),
                                              rows, cols, 128)
    qd = dev.quantize_weights_device(_t(w), 4, 32, False, True)
    assert np.array_equal(_np(dev.requant_q4_128_device(qd, rows, cols)), ref)


def test_weight_prep_device_errors(dev, native):
    import torch

    from asdsl_b200 import _lib

    w = torch.zeros(64, device="cuda")
    with pytest.raises(ValueError):
        dev.quantize_weights_device(w, bits=3)
    with pytest.raises(ValueError):
        dev.quantize_weights_device(w, 4, 48)
    with pytest.raises(ValueError):
        dev.repack_fp32_to_q4_128_device(torch.zeros(2 * 100, device="cuda"), 2, 100)
    with pytest.raises(TypeError):
        dev.quantize_weights_device(np.zeros(64, np.float32))
    assert _lib.device_status(clear=True) == 0


def test_build_c1_device_matches_host(dev):
    """The bench's config-1 weight build on the device gives build_c1_host's bytes (small shape)."""
    from asdsl_b200.layer import build_c1_device, build_c1_host

    cfg = dict(hidden=256, qkv_rows=384, q_dim=256, inter=512)
    h, d = build_c1_host(1, cfg), build_c1_device(1, cfg)
    for k, v in h.items():
        if isinstance(v, np.ndarray):
            assert d[k].shape == v.shape and np.array_equal(d[k], v), k
