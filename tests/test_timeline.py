"""Host logic of the per-CTA GEMV timeline (asdsl_b200.timeline): grouping records into launch
instances (graph replays reuse launch numbers) and the chain figures.  CPU only; the device side
is exercised by the GPU test below."""

import numpy as np
import pytest

from asdsl_b200.timeline import (END, PROLOGUE, PRODUCED, ROW, START, WAITED, CONSUMED, chain_rows,
                                 group_launches, summarize)


def _recs(launches):
    """launches: [(launch number, t0 ns)] each with 3 CTAs and fixed phase offsets"""
    out = []
    for lid, t0 in launches:
        for b in range(3):
            for ev, dt in ((START, 0), (WAITED, 500), (PROLOGUE, 800), (CONSUMED, 4000 + 10 * b),
                           (END, 4100 + 10 * b), (PRODUCED, 3000)):
                out.append((t0 + dt + b, ev | (0 << 4) | (2 << 8) | (1 << 12) | (1 << 16), lid, b))
    r = np.array(out, dtype=ROW)
    return r[np.random.default_rng(0).permutation(len(r))]  # atomic order is not time order


def test_group_launches_replays_and_chain():
    # a graph of launches 7, 8 replayed twice: four instances
    recs = _recs([(7, 0), (8, 5000), (7, 10000), (8, 15000)])
    ls = group_launches(recs)
    assert [(d["id"], d["instance"]) for d in ls] == [(7, 0), (8, 0), (7, 1), (8, 1)]
    assert all(d["ctas"] == 3 for d in ls)
    assert ls[0]["kernel"] == "k_stream_gemv<0,2,1,1>"
    rows = chain_rows(ls)
    assert rows[0]["span"] == pytest.approx((4100 + 20 + 2) / 1e3)
    assert rows[1]["start_after_prev_end"] == pytest.approx((5000 - 4122) / 1e3)
    assert rows[1]["waited_after_prev_end"] == pytest.approx((5500 - 4122) / 1e3)
    assert rows[0]["prologue"] == pytest.approx(0.3)
    s = summarize(rows)
    assert s["k_stream_gemv<0,2,1,1>"]["launches"] == 4


def test_two_library_builds():
    """The default library is compiled without the timeline records, the profiling one with them;
    both from the same single translation unit, for sm_100a."""
    from asdsl_b200 import build

    d = build._command(build.LIB, False)
    t = build._command(build.LIB_TIMELINE, False)
    assert "-DASDSL_B200_TIMELINE=1" not in d and "-DASDSL_B200_TIMELINE=1" in t
    for cmd, lib in ((d, build.LIB), (t, build.LIB_TIMELINE)):
        assert "arch=compute_100a,code=sm_100a" in cmd and cmd[cmd.index("-o") + 1] == lib + ".tmp"
        assert cmd[-1].endswith("asdsl_b200.cu")


def test_timeline_exports():
    from asdsl_b200 import _lib

    for name in ("asdsl_b200_timeline_set", "asdsl_b200_timeline_bytes"):
        assert name in _lib._SIGS


_CHILD = r"""
import sys
import torch
from asdsl_b200 import _lib
from asdsl_b200.timeline import Timeline

_lib.load(_lib.TIMELINE_LIB_PATH)
M, K = 4096, 3072
meta = torch.randint(0, 256, (M * (K // 32) * 4,), dtype=torch.uint8, device="cuda")
meta.view(torch.float16)[:] = 0.01
quant = torch.randint(0, 256, ((M // 4) * (K // 32) * 64,), dtype=torch.uint8, device="cuda")
x = torch.randn(K, device="cuda")
y = torch.empty(M, device="cuda")
with Timeline(slots=8) as tl:
    for _ in range(3):
        _lib.call("asdsl_b200_gemv_preq2_fused", meta.data_ptr(), quant.data_ptr(), x.data_ptr(), y.data_ptr(),
                  M, K, 32, None)
    torch.cuda.synchronize()
ls = tl.launches()
assert tl.dropped == 0 and len(ls) == 3, (tl.dropped, len(ls))
for d in ls:
    assert d["start_min"] <= d["waited_min"] <= d["prologue_max"] <= d["end_max"]
    assert d["ctas"] == min(torch.cuda.get_device_properties(0).multi_processor_count, M // 4)
# off again: no records
before = tl.buf.clone()
_lib.call("asdsl_b200_gemv_preq2_fused", meta.data_ptr(), quant.data_ptr(), x.data_ptr(), y.data_ptr(), M, K, 32,
          None)
torch.cuda.synchronize()
assert torch.equal(before, tl.buf)
print("timeline ok")
"""


@pytest.mark.gpu
def test_timeline_records_every_cta(native):
    """The timeline build (libasdsl_b200_timeline.so, in a child process: this process has the
    default library loaded) records every CTA of three launches, in phase order."""
    import os
    import subprocess
    import sys

    from asdsl_b200.build import build_library

    build_library(timeline=True)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([os.path.join(root, "asdsl-framework_b200"), root, env.get("PYTHONPATH", "")])
    r = subprocess.run(["timeout", "-k", "10", "300", sys.executable, "-c", _CHILD], cwd=root, env=env,
                       capture_output=True, text=True)
    assert r.returncode == 0 and "timeline ok" in r.stdout, (r.stdout + r.stderr)[-3000:]


@pytest.mark.gpu
def test_default_library_has_no_timeline(native):
    """The default library's kernels carry no timeline hooks: asking it for records is an error."""
    import torch

    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        native.call("asdsl_b200_timeline_set", buf.data_ptr(), 1)
    native.call("asdsl_b200_timeline_set", None, 0)
