"""Failure detection on the GPU without a fault: every device-side wait of the kernels is
bounded (2 s of %globaltimer) and reports through the device status word.  Here a wait that
nothing completes is made to run out -- an mbarrier of the streaming pipeline and a
cross-GPU exchange word -- and the test checks that the host sees TimeoutError, the status
bit, and a context that still runs a GEMV correctly afterwards."""

import numpy as np
import pytest
import torch

from oracle.oracle import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which,bit", [(0, 1), (1, 16)])
def test_bounded_wait_gives_up_and_reports(native, oracle, which, bit):
    assert native.device_status(clear=True) == 0
    with pytest.raises(TimeoutError):
        native.call("asdsl_b200_selftest_bounded_wait", which, None)
    assert native.device_status(clear=True) & bit
    # the context is still usable: a GEMV runs and matches the oracle
    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(1)
    meta, quant = random_preq2(rng, 64, 256)
    x = rng.standard_normal(256).astype(np.float32)
    md, qd, xd = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (meta, quant, x))
    y = torch.empty(64, dtype=torch.float32, device="cuda")
    native.call("asdsl_b200_gemv_preq2_fused", md.data_ptr(), qd.data_ptr(), xd.data_ptr(), y.data_ptr(), 64, 256,
                32, None)
    assert rel_err(y.cpu().numpy(), oracle.gemv_preq2_fused(meta, quant, x, 64, 256)) < 1e-3
    assert native.device_status(clear=True) == 0
