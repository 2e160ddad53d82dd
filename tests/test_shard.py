"""Sharded lm_head / MLP host logic on the CPU: gloo ranks (world size 2 and 3) with the CPU
oracle as the per-shard backend, against the unsharded oracle.  The same ShardedLMHead /
ShardedMLP code runs the CUDA kernels over NCCL on GPUs (tests/test_shard_gpu.py,
bench.py --gpus N)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle.oracle import rel_err

TOL = 1e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lm_case(seed=2, V=1000, H=512):
    from asdsl_b200.quantization.repack import repack_fp32_to_q4_128_blocks

    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((V, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    return repack_fp32_to_q4_128_blocks(w, V, H), x


def _mlp_case(seed=1, H=256, I=512):
    from asdsl_b200.quantization.synth import random_preq2

    rng = np.random.default_rng(seed)
    gm, gq = random_preq2(rng, 2 * I, H)
    dm, dq = random_preq2(rng, H, I)
    x = rng.standard_normal(H).astype(np.float32)
    return gm, gq, dm, dq, x


def _worker(rank, world, port, kind, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(root, "asdsl-framework_b200"), root):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    from asdsl_b200.shard import ShardedLMHead, ShardedMLP
    from oracle.oracle import Oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        orc = Oracle()
        if kind == "lm":
            blocks, x = _lm_case()
            head = ShardedLMHead(blocks, 1000, 512, local=orc)
            q.put((rank, head.argmax(x), (head.a, head.b)))
        elif kind == "lm_tie":
            blocks, x = _lm_case()
            b = blocks.reshape(1000, -1).copy()
            b[999] = b[3]  # the same row in the last shard as in the first: first index must win
            b[500] = b[3]
            head = ShardedLMHead(b, 1000, 512, local=orc)
            q.put((rank, head.argmax(x), (head.a, head.b)))
        else:
            gm, gq, dm, dq, x = _mlp_case()
            mlp = ShardedMLP(gm, gq, dm, dq, 256, 512, local=orc)
            q.put((rank, mlp.forward(x).numpy().copy(), (mlp.a, mlp.b)))
    finally:
        dist.destroy_process_group()


def _run(kind, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kind, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out, key=lambda t: t[0])


def test_shard_range_partitions():
    from asdsl_b200.shard import shard_range

    for n, align in ((200064, 4), (8192, 32), (8192, 128), (12, 4)):
        for world in (1, 2, 3, 4, 8):
            if n // align < world:
                continue
            spans = [shard_range(n, world, r, align) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a0, b0), (a1, b1) in zip(spans, spans[1:]):
                assert b0 == a1
            sizes = [b - a for a, b in spans]
            assert all(s % align == 0 for s in sizes) and max(sizes) - min(sizes) <= align
    with pytest.raises(ValueError):
        shard_range(10, 2, 0, 4)


def test_combine_argmax_first_max_wins():
    from asdsl_b200.shard import combine_argmax

    vals = np.array([1.5, 2.0, 2.0, -1.0], np.float32)
    pairs = torch.tensor(np.stack([vals.view(np.int32), np.array([7, 100, 200, 300], np.int32)], 1))
    assert combine_argmax(pairs) == (2.0, 100)


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_lm_head_gloo(oracle, world):
    blocks, x = _lm_case()
    y = oracle.gemv_q4_128_fused(blocks, x, 1000, 512)
    out = _run("lm", world)
    for _, (val, idx), _ in out:
        assert idx == oracle.argmax(y) and val == float(y[idx])


def test_sharded_lm_head_gloo_ties(oracle):
    blocks, x = _lm_case()
    b = blocks.reshape(1000, -1).copy()
    b[999] = b[3]
    b[500] = b[3]
    y = oracle.gemv_q4_128_fused(b, x, 1000, 512)
    out = _run("lm_tie", 2)
    for _, (val, idx), _ in out:
        assert idx == oracle.argmax(y)


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_mlp_gloo(oracle, world):
    gm, gq, dm, dq, x = _mlp_case()
    gu = oracle.gemv_preq2_fused(gm, gq, x, 1024, 256)
    h = oracle.swiglu(gu[:512], gu[512:])
    ref = oracle.gemv_preq2_fused(dm, dq, h, 256, 512)
    out = _run("mlp", world)
    for _, y, _ in out:
        assert rel_err(y, ref) < TOL
