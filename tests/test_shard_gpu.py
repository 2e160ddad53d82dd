"""Device path of the sharded lm_head / MLP on one GPU: every shard is computed by the CUDA
kernels (rank emulation), the shards are combined as the collectives would, and the result is
compared with the unsharded oracle.  Config 2 shape: 200064 x 3072 Q4_128, 1/2/4/8 shards."""

import numpy as np
import pytest
import torch

from oracle.oracle import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.fixture(scope="module")
def lm_case():
    from asdsl_b200.quantization.repack import repack_fp32_to_q4_128_blocks

    rng = np.random.default_rng(2)
    V, H = 200064, 3072
    w = (rng.standard_normal((V, H), dtype=np.float32) * 0.02).astype(np.float32)
    x = rng.standard_normal(H).astype(np.float32)
    return repack_fp32_to_q4_128_blocks(w, V, H), x, V, H


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_sharded_lm_head_device(native, oracle, lm_case, world):
    from asdsl_b200.shard import ShardedLMHead, combine_argmax

    blocks, x, V, H = lm_case
    y = oracle.gemv_q4_128_fused(blocks, x, V, H)
    xd = torch.from_numpy(x).cuda()
    pairs, logits = [], []
    for r in range(world):
        head = ShardedLMHead(blocks, V, H, world=world, rank=r)
        pairs.append(head.local_pair(xd).cpu())
        logits.append(head.logits[: head.rows].cpu().numpy())
    val, idx = combine_argmax(torch.stack(pairs))
    full = np.concatenate(logits)
    assert rel_err(full, y) < TOL
    assert idx == int(np.argmax(full)) and val == float(full[idx])
    srt = np.sort(y)
    if srt[-1] - srt[-2] > 4 * TOL * np.abs(y).max():
        assert idx == oracle.argmax(y)
    assert native.device_status(clear=True) == 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_mlp_device(native, oracle, world):
    from asdsl_b200.quantization.synth import random_preq2
    from asdsl_b200.shard import ShardedMLP

    rng = np.random.default_rng(1)
    H, I = 3072, 8192
    gm, gq = random_preq2(rng, 2 * I, H, scale_range=(0.004, 0.012), zero_range=(7.0, 8.0))
    dm, dq = random_preq2(rng, H, I, scale_range=(0.004, 0.012), zero_range=(7.0, 8.0))
    x = rng.standard_normal(H).astype(np.float32)
    gu = oracle.gemv_preq2_fused(gm, gq, x, 2 * I, H)
    ref = oracle.gemv_preq2_fused(dm, dq, oracle.swiglu(gu[:I], gu[I:]), H, I)
    xd = torch.from_numpy(x).cuda()
    acc = np.zeros(H, np.float32)
    for r in range(world):
        mlp = ShardedMLP(gm, gq, dm, dq, H, I, world=world, rank=r)
        acc += mlp.local_partial(xd).cpu().numpy()
    assert rel_err(acc, ref) < TOL
    assert native.device_status(clear=True) == 0


def test_sharded_lm_head_fused_exchange_single_rank(native, oracle, lm_case):
    """The in-kernel exchange path with a world of one (the kernel stores into and waits on
    its own slot buffer); repeated calls advance the device-resident step counter."""
    from asdsl_b200.shard import ShardedLMHead

    blocks, x, V, H = lm_case
    y = oracle.gemv_q4_128_fused(blocks, x, V, H)
    head = ShardedLMHead(blocks, V, H)
    try:
        assert head.xchg is not None
        xd = torch.from_numpy(x).cuda()
        for _ in range(300):  # crosses the 8-bit step wrap
            val, idx = head.argmax(xd)
            assert idx == int(np.argmax(head.logits.cpu().numpy()))
        assert rel_err(head.logits.cpu().numpy(), y) < TOL
    finally:
        head.close()
    assert native.device_status(clear=True) == 0
