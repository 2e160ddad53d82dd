"""asdsl_b200_gemv_argmax_static (the allocation-free lm_head argmax entry point) against
asdsl_b200_gemv_argmax with caller scratch, through the C ABI.

Collected last on purpose: it must pass both in a fresh process (first call sets up the
static scratch) and after every other GPU test.  Two calls in a row per case: the
static scratch counter must re-arm itself.  Tolerance: the GEMV bar of the suite,
max|d|/max|y| <= 1e-3 (TOL); index and maximum identical."""

import numpy as np
import pytest
import torch

from oracle.oracle import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("fmt,M,K", [(0, 61, 512), (0, 32064, 3072), (2, 37, 512), (2, 32064, 3072)])
def test_gemv_argmax_static_matches_scratch_entry(native, fmt, M, K):
    from asdsl_b200.quantization.repack import repack_fp32_to_q4_128_blocks
    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(7 * M + fmt)
    x = rng.standard_normal(K).astype(np.float32)
    if fmt == 0:
        meta, quant = random_preq2(rng, M, K)
        w0, w1 = _dev(meta), _dev(quant)
    else:
        blocks = repack_fp32_to_q4_128_blocks((rng.standard_normal((M, K)) * 0.02).astype(np.float32), M, K)
        w0, w1 = _dev(blocks), None
    w1p = None if w1 is None else w1.data_ptr()
    xd = _dev(x)
    lib = native.load()
    scratch = torch.zeros(lib.asdsl_b200_argmax_scratch_bytes(), dtype=torch.uint8, device="cuda")
    y_ref = torch.empty(M, dtype=torch.float32, device="cuda")
    y_st = torch.empty(M, dtype=torch.float32, device="cuda")
    ov = torch.empty(2, dtype=torch.float32, device="cuda")
    oi = torch.empty(2, dtype=torch.int32, device="cuda")
    for rep in range(2):
        base = 500 * rep
        native.call("asdsl_b200_gemv_argmax", fmt, w0.data_ptr(), w1p, xd.data_ptr(), y_ref.data_ptr(),
                    ov[0:1].data_ptr(), oi[0:1].data_ptr(), base, scratch.data_ptr(), scratch.numel(), M, K, None)
        native.call("asdsl_b200_gemv_argmax_static", fmt, w0.data_ptr(), w1p, xd.data_ptr(), y_st.data_ptr(),
                    ov[1:2].data_ptr(), oi[1:2].data_ptr(), base, M, K, None)
        torch.cuda.synchronize()
        yr, ys = y_ref.cpu().numpy(), y_st.cpu().numpy()
        assert rel_err(ys, yr) < TOL
        v, i = ov.cpu().numpy(), oi.cpu().numpy()
        assert int(i[1]) == int(i[0])
        assert float(v[1]) == float(v[0])
        assert int(i[1]) - base == int(np.argmax(ys))
    assert native.device_status(clear=True) == 0


def test_gemv_argmax_static_rejects_bad_args(native):
    with pytest.raises(ValueError):
        native.call("asdsl_b200_gemv_argmax_static", 0, None, None, None, None, None, None, 0, 4, 64, None)
    dummy = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    p = dummy.data_ptr()
    with pytest.raises(ValueError):  # unsupported weight format
        native.call("asdsl_b200_gemv_argmax_static", 99, p, p, p, p, p, p, 0, 4, 64, None)


def test_gemv_argmax_static_first_call_in_fresh_process(native):
    """The first-call path (symbol address resolved, array zeroed on the stream) in a process whose
    CUDA context has never called the static entry: this file's cases run in a child interpreter
    with a fresh context, whatever ran before them in this process."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([os.path.join(root, "asdsl-framework_b200"), root, env.get("PYTHONPATH", "")])
    cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-m", "gpu",
           os.path.join(root, "tests", "test_zz_no_alloc.py"), "-k", "matches_scratch_entry"]
    r = subprocess.run(["timeout", "-k", "10", "600"] + cmd, cwd=root, env=env, capture_output=True, text=True)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert "4 passed" in r.stdout, r.stdout[-2000:]
