"""Multi-GPU parity: the sharded MLP (peer all-reduce of the K-split down projection) and the
sharded lm_head (in-kernel argmax exchange) run as one process per GPU under
torch.distributed.run, world size 2 (and every larger power of two the box has, up to 8), each
rank checking its results against the CPU oracle (tests/sharded_worker.py)."""

import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worlds():
    import torch

    n = torch.cuda.device_count()
    return [w for w in (2, 4, 8) if w <= n]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_ranks_vs_oracle(native, oracle, world):
    if world not in _worlds():
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([os.path.join(ROOT, "asdsl-framework_b200"), ROOT,
                                         env.get("PYTHONPATH", "")])
    env["NCCL_NVLS_ENABLE"] = "0"
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "sharded_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, tail
    assert r.stdout.count(f"/{world} OK") == world, tail
