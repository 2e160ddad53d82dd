"""Small, self-contained launches of every kernel family, for profiling one kernel at a time
(`ncu -k <kernel> -c <n> python -m asdsl_b200.profile_cases <case>`): each case builds its inputs
on the device (seeded), runs `--reps` launches of its kernels on one stream and exits 0.

Cases (kernels they launch):
  decode_exact / decode_fast   the config-3 decode step (32-layer Phi-4-mini, seed 3, C0 weights
                   quantized on the device), `--reps` graph replays from position 0
  attention        k_attention_split (decode at 1024 cached positions, Phi-4-mini heads; with
                   ASDSL_B200_ATTN_SPLIT=0 the one-CTA-per-head k_attention), and on the way
                   k_attention_rows / k_kv_write_rows / k_quant_tokens / k_stream_gemv<..,NT>
                   (the batched prefill of those positions)
  attention_exact  k_attention_exact (reference-exact mode, positions < 256) and, from position 256,
                   k_attention_exact_scores + k_attention_exact_sums (1024 cached positions)
  attention_exact_short  k_attention_exact at 64 cached positions (the short-cache form)
  multi            k_stream_gemv<preq, .., NT=8> (dp4a lanes) at 3072x8192, 16 tokens
  multi_mma        k_stream_gemv_mma (int8 mma.sync, selected from 5 tokens) at 8192x3072, 16 tokens
  gemm128          k_gemm_q4_128 (prompt GEMM), 16384x3072, 8 rows
  q4k / s256 / packed  the Q4_K, Q4_S256 and fp32-activation packed GEMVs, 8192x3072
  weight_prep      k_quantize_groups, k_pack_preq2, k_q4_128_from_f32 on 8192x3072 fp32
  exact_gemv       k_stream_gemv<preq2 exact> (RMSNorm + A8 prologue), 16384x3072, the gate_up
                   + SiLU form (8192 pairs), then 5120x3072 (qkv) and 3072x3072 (o) without RMSNorm
  q2               k_gemv_q2<packed> (the QCSD draft bank's 2-bit GEMV), 8192x3072
  timeline         per-CTA phase timelines (asdsl_b200.timeline, loads libasdsl_b200_timeline.so) of
                   back-to-back config-0 GEMVs and of the decode graphs in both numerics modes
  xchg1            k_allreduce_peer and the lm_head argmax exchange with a world of one GPU
                   (the peer stores go to this GPU's own buffers)
"""

from __future__ import annotations

import argparse
import ctypes

import numpy as np
import torch

from asdsl_b200 import _lib


def _bytes(n: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda", generator=g)


def _fp16_scales(n: int, lo: float, hi: float, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.rand(n, device="cuda", generator=g) * (hi - lo) + lo).half()


def _preq2(M: int, K: int, seed: int):
    """random preq2 gs32 blobs on the device: meta [M][K/32] (fp16 scale, fp16 zero-term), quant"""
    ng = K // 32
    meta = torch.stack([_fp16_scales(M * ng, 0.004, 0.012, seed), _fp16_scales(M * ng, -0.1, -0.05, seed + 1)], 1)
    meta = meta.contiguous().view(torch.uint8).reshape(-1)
    quant = _bytes(((M + 3) // 4) * ng * 64, seed + 2)
    return meta, quant


def _x(K: int, seed: int, rows: int = 1) -> torch.Tensor:
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(rows * K, device="cuda", generator=g)


def _engine_case(numerics: str, reps: int, cached: int = 1024):
    from asdsl_b200.inference.synthetic import PHI4_MINI, build_model_device
    from asdsl_b200.kernels._native_unified import engine_from_model

    cfg = dict(PHI4_MINI, num_layers=1, vocab=8192, max_seq=2048)
    model = build_model_device(cfg, seed=5, norms_one=False)
    eng = engine_from_model(model, numerics=numerics)
    try:
        prompt = np.random.default_rng(5).integers(0, cfg["vocab"], size=cached).tolist()
        eng.forward_batch(prompt, 0)
        for i in range(reps):
            eng.forward_token_argmax(prompt[i % 7], cached + i)
    finally:
        eng.close()


def case_attention_exact_short(reps):
    _engine_case("reference_exact", reps, cached=64)


def _decode_case(numerics: str, reps: int):
    from asdsl_b200.inference.synthetic import PHI4_MINI, build_model_device
    from asdsl_b200.kernels._native_unified import engine_from_model

    model = build_model_device(PHI4_MINI, seed=3, quantized=True)
    eng = engine_from_model(model, numerics=numerics)
    try:
        eng.set_position(0, 1)
        eng.replay(reps)
    finally:
        eng.close()


def case_decode_exact(reps):
    _decode_case("reference_exact", reps)


def case_decode_fast(reps):
    _decode_case("fast", reps)


def case_attention(reps):
    _engine_case("fast", reps)


def case_attention_exact(reps):
    _engine_case("reference_exact", reps)


def case_multi(reps):
    from asdsl_b200.kernels._native_gemv import gemv_multi

    M, K, k = 3072, 8192, 16
    blocks = _bytes(M * (K // 32) * 20, 1)  # preq gs32 blocks: fp16 scale, fp16 bias, 16 nibble bytes
    blocks.view(torch.float16)[0::10].copy_(_fp16_scales(blocks.numel() // 20, 0.004, 0.012, 2))
    blocks.view(torch.float16)[1::10].copy_(_fp16_scales(blocks.numel() // 20, -0.1, -0.05, 3))
    X = _x(K, 4, k).reshape(k, K)
    Y = torch.empty(k * M, device="cuda")
    for _ in range(reps):
        gemv_multi(_lib.FMT_PREQ, blocks, None, X, Y, M, K)


def case_multi_mma(reps):
    from asdsl_b200.kernels._native_gemv import gemv_multi

    M, K, k = 8192, 3072, 16
    blocks = _bytes(M * (K // 32) * 20, 1)
    blocks.view(torch.float16)[0::10].copy_(_fp16_scales(blocks.numel() // 20, 0.004, 0.012, 2))
    blocks.view(torch.float16)[1::10].copy_(_fp16_scales(blocks.numel() // 20, -0.1, -0.05, 3))
    X = _x(K, 4, k).reshape(k, K)
    Y = torch.empty(k * M, device="cuda")
    _lib.call("asdsl_b200_set_mma_min_tokens", 5)
    try:
        for _ in range(reps):
            gemv_multi(_lib.FMT_PREQ, blocks, None, X, Y, M, K)
    finally:
        _lib.call("asdsl_b200_set_mma_min_tokens", 0)


def case_gemm128(reps):
    M, K, B = 16384, 3072, 8
    blocks = _bytes(M * (K // 128) * 66, 1)
    blocks.view(torch.float16)[0::33].copy_(_fp16_scales(blocks.numel() // 66, 0.006, 0.012, 2))
    X = _x(K, 3, B)
    Y = torch.empty(B * M, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(reps):
        _lib.call("asdsl_b200_gemm_q4_128_f32", blocks.data_ptr(), X.data_ptr(), Y.data_ptr(), M, K, 128, B, s)


def _a8(x: torch.Tensor, K: int, gs: int = 32):
    xq = torch.empty(K, dtype=torch.int8, device="cuda")
    xs = torch.empty(K // gs, device="cuda")
    _lib.call("asdsl_b200_quantize_activation", x.data_ptr(), xq.data_ptr(), xs.data_ptr(), None, K, gs,
              torch.cuda.current_stream().cuda_stream)
    return xq, xs


def case_q4k(reps):
    M, K = 8192, 3072
    w = _bytes(M * (K // 256) * 144, 1)
    w.view(torch.float16).view(-1, 72)[:, 0].copy_(_fp16_scales(M * (K // 256), 0.002, 0.002, 2))
    w.view(torch.float16).view(-1, 72)[:, 1].copy_(_fp16_scales(M * (K // 256), 0.004, 0.004, 3))
    x, y = _x(K, 4), torch.empty(M, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(reps):
        _lib.call("asdsl_b200_gemv_q4km", w.data_ptr(), x.data_ptr(), y.data_ptr(), M, K, s)


def case_s256(reps):
    M, K = 8192, 3072
    w = _bytes(M * (K // 256) * 144, 1)
    w.view(torch.float16).view(-1, 72)[:, 0].copy_(_fp16_scales(M * (K // 256), 0.004, 0.012, 2))
    w.view(torch.float16).view(-1, 72)[:, 1].copy_(_fp16_scales(M * (K // 256), -0.1, -0.05, 3))
    xq, xs = _a8(_x(K, 4), K)
    y = torch.empty(M, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(reps):
        _lib.call("asdsl_b200_gemv_q4_s256", w.data_ptr(), xq.data_ptr(), xs.data_ptr(), y.data_ptr(), M, K, 32, s)


def case_packed(reps):
    M, K, gs = 8192, 3072, 32
    w = _bytes(M * K // 2, 1)
    sc = torch.full((M * K // gs,), 0.01, device="cuda")
    bi = torch.full((M * K // gs,), -0.08, device="cuda")
    x, y = _x(K, 4), torch.empty(M, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(reps):
        _lib.call("asdsl_b200_gemv_q4_packed", w.data_ptr(), x.data_ptr(), sc.data_ptr(), bi.data_ptr(), y.data_ptr(),
                  M, K, gs, 1, s)


def case_q2(reps):
    M, K = 8192, 3072
    w = _bytes(M * K // 4, 1)
    sc = _fp16_scales(M * (K // 32), 0.01, 0.03, 2).float()
    bi = -_fp16_scales(M * (K // 32), 0.01, 0.05, 3).float()
    x, y = _x(K, 4), torch.empty(M, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(reps):
        _lib.call("asdsl_b200_gemv_q2_packed", w.data_ptr(), x.data_ptr(), sc.data_ptr(), bi.data_ptr(), y.data_ptr(),
                  M, K, 32, s)


def case_weight_prep(reps):
    from asdsl_b200.quantization.device import prepare_preq2_device, repack_fp32_to_q4_128_device

    M, K = 8192, 3072
    w = _x(M * K, 1).reshape(M, K) * 0.02
    for _ in range(reps):
        prepare_preq2_device(w)
        repack_fp32_to_q4_128_device(w, M, K)


def case_exact_gemv(reps):
    M, K, I = 16384, 3072, 8192
    meta, quant = _preq2(M, K, 1)
    x = _x(K, 3) * 30
    nw = torch.ones(K, device="cuda")
    y = torch.empty(M, device="cuda")
    h = torch.empty(I, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(reps):
        _lib.call("asdsl_b200_gemv_preq2_fused_exact", meta.data_ptr(), quant.data_ptr(), x.data_ptr(), nw.data_ptr(),
                  ctypes.c_float(1e-5), y.data_ptr(), M, K, s)
    for _ in range(reps):
        _lib.call("asdsl_b200_gateup_silu_exact", meta.data_ptr(), quant.data_ptr(), x.data_ptr(), nw.data_ptr(),
                  ctypes.c_float(1e-5), h.data_ptr(), I, K, s)
    for m2 in (5120, 3072):
        for _ in range(reps):
            _lib.call("asdsl_b200_gemv_preq2_fused_exact", meta.data_ptr(), quant.data_ptr(), x.data_ptr(), None,
                      ctypes.c_float(0.0), y.data_ptr(), m2, K, s)


def case_xchg1(reps):
    from asdsl_b200.quantization.synth import random_q4_128
    from asdsl_b200.shard import ShardedLMHead, _VecExchange

    dev = torch.device("cuda", torch.cuda.current_device())
    vx = _VecExchange(1, 0, 3072, dev)
    part, out = _x(3072, 1), torch.empty(3072, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    try:
        for _ in range(reps):
            vx.allreduce(part, out, 3072, s)
    finally:
        torch.cuda.synchronize()
        vx.close()
    V, H = 32064, 3072
    head = ShardedLMHead(random_q4_128(np.random.default_rng(2), V, H), V, H, world=None, rank=None)
    try:
        xd = _x(H, 5)
        for _ in range(reps):
            head.fused_step(xd)
    finally:
        torch.cuda.synchronize()
        head.close()


def case_timeline(reps):
    """Per-CTA timelines (asdsl_b200.timeline): 16 back-to-back config-0 GEMVs (preq2 gs32
    16384x3072, random bytes, 6 copies rotated past the L2) in a CUDA graph, then `reps` decode
    graph replays of the 32-layer Phi-4-mini shape in both numerics modes; prints the per-kernel
    means of each phase."""
    from asdsl_b200.inference.synthetic import PHI4_MINI, build_model_device
    from asdsl_b200.kernels._native_unified import engine_from_model
    from asdsl_b200.timeline import Timeline, format_chain

    M, K = 16384, 3072
    copies = [_preq2(M, K, 10 + 3 * i) for i in range(6)]
    x, y = _x(K, 3), torch.empty(M, device="cuda")
    st = torch.cuda.Stream()

    def run(c):
        _lib.call("asdsl_b200_gemv_preq2_fused", c[0].data_ptr(), c[1].data_ptr(), x.data_ptr(), y.data_ptr(), M, K,
                  32, st.cuda_stream)

    with torch.cuda.stream(st):
        for c in copies:
            run(c)
    st.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(16):
            run(copies[i % len(copies)])
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    with Timeline() as tl:
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
    print(f"config-0 GEMV, 32 launches in graphs ({len(tl.recs)} records, {tl.dropped} dropped)")
    print(format_chain(tl.launches()))
    # two kernel templates alternating in one graph: the config-0 GEMV and the same weights in the
    # reference-exact form (another function, same shape)
    nw = torch.ones(K, device="cuda")

    def run_x(c):
        _lib.call("asdsl_b200_gemv_preq2_fused_exact", c[0].data_ptr(), c[1].data_ptr(), x.data_ptr(), None,
                  ctypes.c_float(0.0), y.data_ptr(), M, K, st.cuda_stream)

    with torch.cuda.stream(st):
        for c in copies:
            run_x(c)
    st.synchronize()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=st):
        for i in range(16):
            (run if i % 2 == 0 else run_x)(copies[i % len(copies)])
    for _ in range(3):
        g2.replay()
    torch.cuda.synchronize()
    with Timeline() as tl:
        for _ in range(2):
            g2.replay()
        torch.cuda.synchronize()
    print("config-0 GEMV alternating with its reference-exact form, in graphs")
    print(format_chain(tl.launches()))
    # the config-1 layer chain (qkv, o, gate_up + SiLU, down) captured by torch
    from asdsl_b200.layer import build_c1_device, from_host

    host = build_c1_device(1)
    base = from_host(host)
    layers = [base] + [base.clone() for _ in range(5)]
    xl = torch.from_numpy(host["x"]).cuda()
    for L in layers:
        with torch.cuda.stream(st):
            L.step(xl)
    st.synchronize()
    g3 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g3, stream=st):
        for L in layers:
            L.step(xl)
    for _ in range(3):
        g3.replay()
    torch.cuda.synchronize()
    with Timeline() as tl:
        for _ in range(2):
            g3.replay()
        torch.cuda.synchronize()
    print("config-1 layer chain (torch graph); [0..3] = qkv, o, gate_up, down")
    print(format_chain(tl.launches(), period=4))
    del g, g2, g3, copies, layers, base
    torch.cuda.empty_cache()
    for numerics in ("fast", "reference_exact"):
        model = build_model_device(PHI4_MINI, seed=3, quantized=True)
        eng = engine_from_model(model, numerics=numerics)
        try:
            eng.set_position(0, 1)
            eng.replay(3)
            torch.cuda.synchronize()
            with Timeline() as tl:
                eng.replay(max(reps, 1))
                torch.cuda.synchronize()
            tl_long = None
            if numerics == "reference_exact":
                # the same at 200 cached positions (the cache filled by a forward over a prompt)
                prompt = np.random.default_rng(7).integers(0, PHI4_MINI["vocab"], size=200).tolist()
                eng.forward_batch(prompt, 0)
                eng.set_position(200, prompt[-1])
                eng.replay(1)
                torch.cuda.synchronize()
                with Timeline() as tl_long:
                    eng.replay(max(reps, 1))
                    torch.cuda.synchronize()
        finally:
            eng.close()
            del model
            torch.cuda.empty_cache()
        print(f"decode {numerics}, {max(reps, 1)} graph replays from position 3 ({len(tl.recs)} records, "
              f"{tl.dropped} dropped); [0..3] = qkv, o, gate_up, down")
        print(format_chain(tl.launches(), period=4))
        if tl_long is not None:
            print(f"decode {numerics}, {max(reps, 1)} graph replays from position 201")
            print(format_chain(tl_long.launches(), period=4))


CASES = {name[5:]: fn for name, fn in globals().items() if name.startswith("case_")}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=4)
    a = ap.parse_args()
    # the timeline case needs the build with the per-CTA records compiled in
    _lib.load(_lib.TIMELINE_LIB_PATH if a.case == "timeline" else None)
    CASES[a.case](a.reps)
    torch.cuda.synchronize()
    if _lib.device_status(clear=True) != 0:
        raise SystemExit(f"{a.case}: a kernel reported a bounded-wait timeout")
    print(f"ok {a.case}")


if __name__ == "__main__":
    main()
