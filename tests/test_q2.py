"""2-bit GEMVs of the QCSD draft bank (gemv_q2_packed_impl / gemv_q2_unpacked_impl,
asdsl/kernels/native/gemv_q2_avx2.cpp:128-174, :53-118).

CPU: the oracle's restatement against the reference's compiled kernels (oracle/_ref, when built).
GPU: asdsl_b200_gemv_q2_{packed,unpacked} against the oracle and the reference kernels at the
Phi-4-mini projection shapes, ragged rows and group sizes 32 / 64 / 128.  Bar: max|d|/max|y| <=
1e-3 (TOL; fp32 reassociation only -- the codes, scales and biases are used as given)."""

import numpy as np
import pytest

from oracle.oracle import ref_lib_path, rel_err

TOL = 1e-3


def _case(M, K, gs, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 4, size=(M, K), dtype=np.uint8)
    packed = (codes[:, 0::4] | (codes[:, 1::4] << 2) | (codes[:, 2::4] << 4) | (codes[:, 3::4] << 6)).astype(np.uint8)
    scales = rng.uniform(0.01, 0.03, size=M * (K // gs)).astype(np.float32)
    biases = rng.uniform(-0.05, -0.01, size=M * (K // gs)).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    return codes.reshape(-1), packed.reshape(-1), scales, biases, x


def _dense(codes, scales, biases, x, M, K, gs):
    w = codes.reshape(M, K // gs, gs).astype(np.float64) * scales.reshape(M, K // gs, 1) + biases.reshape(M, K // gs, 1)
    return (w.reshape(M, K) @ x.astype(np.float64)).astype(np.float32)


@pytest.mark.parametrize("M,K,gs", [(37, 256, 32), (64, 512, 64), (16, 384, 128)])
def test_q2_oracle_vs_dense_and_reference(oracle, M, K, gs):
    codes, packed, s, b, x = _case(M, K, gs, M + K)
    dense = _dense(codes, s, b, x, M, K, gs)
    for is_packed, w in ((True, packed), (False, codes)):
        y = oracle.gemv_q2(is_packed, w, x, s, b, M, K, gs)
        assert rel_err(y, dense) < 1e-5
        if ref_lib_path():
            from oracle.oracle import RefKernels

            assert rel_err(y, RefKernels().gemv_q2(is_packed, w, x, s, b, M, K, gs)) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,gs", [(5120, 3072, 32), (3072, 8192, 32), (16384, 3072, 32), (1001, 512, 64),
                                    (37, 384, 128), (3, 32, 32)])
def test_q2_gpu_vs_oracle(native, oracle, M, K, gs):
    from asdsl_b200.kernels import gemv_q2_packed, gemv_q2_unpacked

    codes, packed, s, b, x = _case(M, K, gs, 7 * M + K)
    want = oracle.gemv_q2(True, packed, x, s, b, M, K, gs)
    assert rel_err(gemv_q2_packed(packed, x, s, b, M, K, gs), want) < TOL
    assert rel_err(gemv_q2_unpacked(codes, x, s, b, M, K, gs), oracle.gemv_q2(False, codes, x, s, b, M, K, gs)) < TOL
    if ref_lib_path() and M * K <= 3072 * 3072:
        from oracle.oracle import RefKernels

        assert rel_err(gemv_q2_packed(packed, x, s, b, M, K, gs), RefKernels().gemv_q2(True, packed, x, s, b, M, K, gs)) < TOL
    assert native.device_status(clear=True) == 0


@pytest.mark.gpu
def test_q2_gpu_errors(native):
    from asdsl_b200.kernels import gemv_q2_packed

    codes, packed, s, b, x = _case(8, 64, 32, 1)
    with pytest.raises(ValueError):
        gemv_q2_packed(packed, x, s, b, 8, 66, 32)  # K % 4
    with pytest.raises(ValueError):
        gemv_q2_packed(packed, x, s[:-1], b, 8, 64, 32)  # scales size
    with pytest.raises(ValueError):
        gemv_q2_packed(packed, x, s, b, 8, 64, 48)  # K % group_size
