"""GPU parity of the multi-token W4A8 GEMV (asdsl_b200_gemv_multi, config 4: speculative
verification) against k serial single-token oracle calls.

Config 4 shapes: 8192x3072 and 3072x8192, k in {1, 2, 4, 8, 16}, formats preq gs32 and the
reference-interpretation Q4_K; plus preq2 / banded Q4_128 and ragged row counts.  Bar: every
token row within max|d|/max|y| <= 1e-3 (TOL) of the oracle's single-token GEMV on that row."""

import numpy as np
import pytest
import torch

from oracle.oracle import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _weights(rng, fmt, M, K):
    from asdsl_b200 import _lib
    from asdsl_b200.quantization.repack import preq2_to_preq
    from asdsl_b200.quantization.synth import random_preq2, random_q4k_bytes

    if fmt == _lib.FMT_Q4K:
        return random_q4k_bytes(rng, M, K), None
    meta, quant = random_preq2(rng, M, K, scale_range=(0.004, 0.012), zero_range=(7.0, 8.0))
    if fmt == _lib.FMT_PREQ:
        return preq2_to_preq(meta, quant, M, K).reshape(-1), None
    return meta, quant


def _oracle_row(oracle, fmt, w0, w1, x, M, K):
    from asdsl_b200 import _lib

    if fmt == _lib.FMT_Q4K:
        return oracle.gemv_q4km(w0, x, M, K)
    if fmt == _lib.FMT_PREQ:
        return oracle.gemv_preq_fused(w0, x, M, K)
    return oracle.gemv_preq2_fused(w0, w1, x, M, K)


@pytest.fixture(params=["lane_dot", "tensor_core"])
def multi_path(request, native):
    """both multi-token paths: lane dp4a chains (default) and int8 tensor-core MMAs for >= 5 rows"""
    native.call("asdsl_b200_set_mma_min_tokens", 5 if request.param == "tensor_core" else 0)
    yield request.param
    native.call("asdsl_b200_set_mma_min_tokens", 0)


@pytest.mark.parametrize("fmt_name", ["PREQ", "Q4K"])
@pytest.mark.parametrize("M,K", [(8192, 3072), (3072, 8192)])
def test_gemv_multi_config4(native, oracle, fmt_name, M, K, multi_path):
    from asdsl_b200.kernels._native_gemv import gemv_multi

    fmt = getattr(native, f"FMT_{fmt_name}")
    rng = np.random.default_rng(4)
    w0, w1 = _weights(rng, fmt, M, K)
    w0d = _dev(w0)
    w1d = _dev(w1) if w1 is not None else None
    X = rng.standard_normal((16, K)).astype(np.float32)
    ref = np.stack([_oracle_row(oracle, fmt, w0, w1, X[t], M, K) for t in range(16)])
    for k in (1, 2, 4, 8, 16):
        Y = torch.empty(k * M, dtype=torch.float32, device="cuda")
        gemv_multi(fmt, w0d, w1d, _dev(X[:k]), Y, M, K)
        y = Y.cpu().numpy().reshape(k, M)
        for t in range(k):
            assert rel_err(y[t], ref[t]) < TOL, f"k={k} token {t}: {rel_err(y[t], ref[t])}"
    assert native.device_status(clear=True) == 0


@pytest.mark.parametrize("fmt_name,M,K", [("PREQ", 61, 512), ("Q4K", 23, 512), ("PREQ2", 61, 512),
                                          ("PREQ2", 5120, 3072), ("PREQ", 37, 3072)])
@pytest.mark.parametrize("k", [3, 5, 8, 9, 12, 17])
def test_gemv_multi_ragged(native, oracle, fmt_name, M, K, k, multi_path):
    """odd token counts (partial token groups, a second pass past 16; 8 and more rows run on the
    tensor cores with partial 16-row tiles and partial 8-token groups) and ragged row bands"""
    from asdsl_b200.kernels._native_gemv import gemv_multi

    fmt = getattr(native, f"FMT_{fmt_name}")
    rng = np.random.default_rng(M + k)
    w0, w1 = _weights(rng, fmt, M, K)
    X = rng.standard_normal((k, K)).astype(np.float32)
    X[0, :32] = 0.0  # an all-zero A8 group
    Y = np.zeros(k * M, np.float32)
    gemv_multi(fmt, w0, w1, X, Y, M, K)
    y = Y.reshape(k, M)
    for t in range(k):
        assert rel_err(y[t], _oracle_row(oracle, fmt, w0, w1, X[t], M, K)) < TOL
    assert native.device_status(clear=True) == 0


def test_gemv_multi_banded_q4_128(native, oracle):
    from asdsl_b200.kernels._native_gemv import gemv_multi
    from asdsl_b200.quantization.repack import q4_128_to_banded, repack_fp32_to_q4_128_blocks

    rng = np.random.default_rng(9)
    M, K, k = 1027, 3072, 6
    blocks = repack_fp32_to_q4_128_blocks((rng.standard_normal((M, K)) * 0.02).astype(np.float32), M, K)
    q, s = q4_128_to_banded(blocks, M, K)
    X = rng.standard_normal((k, K)).astype(np.float32)
    Y = np.zeros(k * M, np.float32)
    gemv_multi(native.FMT_Q4_128_BANDED, q, s, X, Y, M, K)
    for t in range(k):
        assert rel_err(Y.reshape(k, M)[t], oracle.gemv_q4_128_fused(blocks, X[t], M, K)) < TOL
    assert native.device_status(clear=True) == 0


def test_gemv_multi_errors(native):
    from asdsl_b200.kernels._native_gemv import gemv_multi

    w = np.zeros(4 * 96 * 20, np.uint8)
    with pytest.raises(ValueError):
        gemv_multi(native.FMT_PREQ, w, None, np.zeros((2, 3000), np.float32), np.zeros(8, np.float32), 4, 3000)
    with pytest.raises(ValueError):
        gemv_multi(99, w, None, np.zeros((2, 3072), np.float32), np.zeros(8, np.float32), 4, 3072)
