"""The host-side weight prep (asdsl_b200.quantization) against bytes produced by
the reference's own quantizer and repackers (tests/golden).  CPU only."""

import numpy as np

from asdsl_b200.quantization import core, repack, synth


def test_quantize_weights_bit_exact(golden):
    g = golden("quant_w32x256.npz")
    for tag, sym, opt in (("asym_opt", False, True), ("asym_plain", False, False), ("sym_opt", True, True)):
        qt = core.quantize_weights(g["w"], bits=4, group_size=32, symmetric=sym, optimize_clips=opt)
        assert np.array_equal(qt.data, g[f"{tag}_data"]), tag
        assert np.array_equal(qt.scales.view(np.uint16), g[f"{tag}_scales"]), tag
        if not sym:
            assert np.array_equal(qt.zeros.view(np.uint16), g[f"{tag}_zeros"]), tag


def test_repackers_bit_exact(golden):
    g = golden("repack_29x256.npz")
    rows, cols = 29, 256
    preq = repack.repack_asymmetric_to_q4_32_blocks(g["packed"], g["scales"], g["biases"], rows, cols, 32)
    assert np.array_equal(preq, g["preq"])
    meta, quant = repack.repack_preq_blocks_to_preq2(repack.blocks_to_flat(preq), rows, cols, 32)
    assert np.array_equal(meta, g["meta"]) and np.array_equal(quant, g["quant"])
    # the inverse permutation restores the preq bytes (ragged last band: 29 = 7*4 + 1)
    assert np.array_equal(repack.preq2_to_preq(meta, quant, rows, cols), repack.blocks_to_flat(preq))
    assert np.array_equal(repack.repack_fp32_to_q4_128_blocks(g["w_f32"], rows, cols, 128), g["q4_128"])
    a128 = repack.repack_asymmetric_to_q4_128_blocks(g["packed128"], g["scales128"], g["biases128"], rows, cols, 128)
    assert np.array_equal(a128, g["q4_128_asym"])


def test_zero_group_rules(golden):
    g = golden("repack_29x256.npz")
    b = g["q4_128"].reshape(29, 2, 66)
    assert b[2, 1, 0] == 0 and b[2, 1, 1] == 0 and (b[2, 1, 2:] == 0x88).all()


def test_q4k_sixbit_packing_roundtrip():
    rng = np.random.default_rng(0)
    vals = rng.integers(0, 64, size=(7, 16), dtype=np.uint8)
    packed = synth._pack6(vals)

    def get6(p, idx):  # gemv_q4_avx2.cpp:110-120
        bit = idx * 6
        byte, off = bit >> 3, bit & 7
        if off <= 2:
            return (int(p[byte]) >> off) & 0x3F
        return ((int(p[byte]) >> off) | (int(p[byte + 1]) << (8 - off))) & 0x3F

    for r in range(7):
        assert [get6(packed[r], i) for i in range(16)] == list(vals[r])


def test_dequant_matches_packed_projection():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((8, 128)) * 0.02).astype(np.float32)
    qt = core.quantize_weights(w, 4, 32, False, True)
    sc, bi = core.scales_biases_f32(qt)
    d1 = core.dequant_packed_projection(qt.data, sc, bi, 8, 128, 32)
    d2 = core.dequantize_weights(qt)
    assert np.max(np.abs(d1 - d2)) < 1e-6
