"""Row-sharded lm_head / gate_up and K-split down projection across the GPUs of one box.

One process per GPU (torch.distributed, NCCL over NVLink); every rank holds a contiguous slice
of the projection's rows (lm_head, gate_up) or of its input columns (down):

* lm_head (BASELINE config 2 / the engine's lm_head, unified_engine.cpp:1628-1662 with
  argmax_f32_avx2 :207-233): rank r owns rows [a_r, b_r), runs the fused GEMV + first-max
  argmax on them with row_base = a_r, and the ranks all-gather one (max, index) pair each
  (8 bytes).  The final pick is the first maximum in rank order; ranks hold ascending row
  ranges, so that is the lowest global index among equal maxima, as the reference's scan.
* gate_up: rank r owns gate rows [a_r, b_r) and the matching up rows [I + a_r, I + b_r), so
  SiLU(gate)*up is local and yields h[a_r:b_r).
* down: rank r owns input columns [a_r, b_r) of down_proj (whole activation groups: the A8
  quantization is per group, so the local A8 of h[a_r:b_r) equals the slice of the global
  one); partial outputs are summed with one all-reduce of hidden_size floats -- on GPUs by
  default one kernel over NVLink peer stores (asdsl_b200_allreduce_peer: each rank pushes its
  partial into every rank's buffer, then sums the world's partials in rank order, so every
  rank holds the same bits), else torch.distributed's all_reduce.  The sum order across ranks
  differs from the reference's single row dot, which the GEMV tolerance covers; with
  numerics="reference_exact" each rank's partial is bitwise the reference kernels' result on
  its shard, and the output is bitwise their rank-ordered float32 sum.

The per-shard compute goes through the C ABI kernels by default; tests running the ranks as
gloo processes on the CPU pass the CPU oracle as `local` backend instead, so the collective
logic is the same code on both.
"""

from __future__ import annotations

import numpy as np
import torch

from asdsl_b200 import _lib


def shard_range(n: int, world: int, rank: int, align: int = 4) -> tuple[int, int]:
    """[a, b) of `n` items for `rank`: contiguous, ascending in rank, boundaries multiples of
    `align` (4-row bands; 32 or 128 columns for whole activation groups), sizes differing by at
    most `align`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("invalid rank / world size")
    if n % align:
        raise ValueError(f"{n} items cannot be split on a {align}-item boundary")
    units = n // align
    a = units * rank // world
    b = units * (rank + 1) // world
    return a * align, b * align


def combine_argmax(pairs: torch.Tensor) -> tuple[float, int]:
    """pairs [world, 2] int32: (max value bits as float32, global index) per rank, in rank
    order.  First maximum wins (ties -> lowest rank = lowest index range)."""
    vals = pairs[:, 0].contiguous().view(torch.float32)
    best = int(torch.nonzero(vals == vals.max())[0].item())
    return float(vals[best].item()), int(pairs[best, 1].item())


def _all_gather_pairs(pair: torch.Tensor, world: int) -> torch.Tensor:
    import torch.distributed as dist

    parts = [torch.empty_like(pair) for _ in range(world)]
    dist.all_gather(parts, pair)
    return torch.stack(parts)


def _group(world=None, rank=None):
    """(world size, rank) of the default process group, or the explicit pair (rank emulation:
    one process computing one shard, with the caller combining the shards)."""
    if world is not None:
        return int(world), int(rank)
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


class _Exchange:
    """Slot buffer of the in-kernel argmax exchange (asdsl_b200_xchg_*): created on every rank,
    its CUDA IPC handle all-gathered in rank order, then the peers' buffers mapped."""

    def __init__(self, world: int, rank: int, device):
        import ctypes

        lib = _lib.load()
        self._lib = lib
        hb = int(lib.asdsl_b200_xchg_handle_bytes())
        h = (ctypes.c_uint8 * hb)()
        self.ptr = ctypes.c_void_p()
        _lib.check(lib.asdsl_b200_xchg_create(world, rank, ctypes.byref(self.ptr), h), "xchg_create")
        mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device=device)
        if world > 1:
            import torch.distributed as dist

            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            allh = np.ascontiguousarray(torch.cat(parts).cpu().numpy())
        else:
            allh = np.ascontiguousarray(mine.cpu().numpy())
        _lib.check(lib.asdsl_b200_xchg_open(self.ptr, allh.ctypes.data), "xchg_open")

    def set_stamps(self, buf=None):
        """record %globaltimer stamps of every exchange step into `buf` (int64 [n, 4] on the
        device, n a power of two); None turns them off"""
        _lib.call("asdsl_b200_xchg_set_stamps", self.ptr, buf.data_ptr() if buf is not None else None,
                  buf.shape[0] if buf is not None else 0)

    def close(self):
        if getattr(self, "ptr", None):
            self._lib.asdsl_b200_xchg_destroy(self.ptr)
            self.ptr = None


class _VecExchange:
    """Buffers of the peer all-reduce (asdsl_b200_vxchg_*): created on every rank with room for
    `n_max` floats per rank and step parity, the CUDA IPC handles all-gathered in rank order,
    then the peers' buffers mapped."""

    def __init__(self, world: int, rank: int, n_max: int, device):
        import ctypes

        lib = _lib.load()
        self._lib = lib
        hb = int(lib.asdsl_b200_vxchg_handle_bytes())
        h = (ctypes.c_uint8 * hb)()
        self.ptr = ctypes.c_void_p()
        _lib.check(lib.asdsl_b200_vxchg_create(world, rank, n_max, ctypes.byref(self.ptr), h), "vxchg_create")
        mine = torch.tensor(list(bytes(h)), dtype=torch.uint8, device=device)
        if world > 1:
            import torch.distributed as dist

            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            allh = np.ascontiguousarray(torch.cat(parts).cpu().numpy())
        else:
            allh = np.ascontiguousarray(mine.cpu().numpy())
        _lib.check(lib.asdsl_b200_vxchg_open(self.ptr, allh.ctypes.data), "vxchg_open")

    def set_stamps(self, buf=None):
        """record %globaltimer stamps of every step into `buf` (int64 [n, 4] on the device, n a
        power of two); None turns them off"""
        _lib.call("asdsl_b200_vxchg_set_stamps", self.ptr, buf.data_ptr() if buf is not None else None,
                  buf.shape[0] if buf is not None else 0)

    def allreduce(self, part, out, n: int, stream, add=None):
        _lib.call("asdsl_b200_allreduce_peer", self.ptr, part.data_ptr(), out.data_ptr(),
                  add.data_ptr() if add is not None else None, n, stream)

    def close(self):
        if getattr(self, "ptr", None):
            self._lib.asdsl_b200_vxchg_destroy(self.ptr)
            self.ptr = None


class ShardedLMHead:
    """This rank's Q4_128 lm_head rows in the banded device layout (or the CPU oracle's raw
    blocks when `local` is given) and the argmax across ranks: with fused=True (GPUs, the
    default) one kernel per step exchanges the (max, index) pairs over NVLink peer stores
    (asdsl_b200_gemv_argmax_xchg); otherwise an all-gather of the pairs through the process
    group follows the local fused GEMV + argmax."""

    def __init__(self, blocks: np.ndarray, vocab: int, hidden: int, local=None, device=None, world=None, rank=None,
                 fused: bool = True):
        self.world, self.rank = _group(world, rank)
        self.V, self.H = vocab, hidden
        self.a, self.b = shard_range(vocab, self.world, self.rank, 4)
        ng = hidden // 128
        rows = np.asarray(blocks, dtype=np.uint8).reshape(vocab, ng * 66)[self.a : self.b]
        self.rows = self.b - self.a
        self.local = local
        if local is None:
            from asdsl_b200.layer import relayout_q4_128

            dev = device or torch.device("cuda", torch.cuda.current_device())
            self.device = dev
            raw = torch.from_numpy(np.ascontiguousarray(rows).reshape(-1)).to(dev)
            self.quant, self.scales = relayout_q4_128(raw, self.rows, hidden)
            del raw
            self.scratch = torch.zeros(_lib.load().asdsl_b200_argmax_scratch_bytes(), dtype=torch.uint8, device=dev)
            self.val = torch.empty(1, dtype=torch.float32, device=dev)
            self.idx = torch.empty(1, dtype=torch.int32, device=dev)
            self.logits = torch.empty(max(self.rows, 1), dtype=torch.float32, device=dev)
            self.xchg = _Exchange(self.world, self.rank, dev) if (fused and world is None) else None
        else:
            self.device = torch.device("cpu")
            self.blocks = np.ascontiguousarray(rows)
            self.xchg = None

    def close(self):
        if getattr(self, "xchg", None) is not None:
            self.xchg.close()
            self.xchg = None

    def fused_step(self, x) -> torch.Tensor:
        """One kernel: local GEMV + argmax + exchange with the peers; returns the global index
        (int32 [1] on this rank's device; self.val holds the maximum)."""
        _lib.call("asdsl_b200_gemv_argmax_xchg", _lib.FMT_Q4_128_BANDED, self.quant.data_ptr(), self.scales.data_ptr(),
                  x.data_ptr(), self.logits.data_ptr(), self.val.data_ptr(), self.idx.data_ptr(), self.a,
                  self.scratch.data_ptr(), self.scratch.numel(), self.rows, self.H, self.xchg.ptr,
                  torch.cuda.current_stream(self.device).cuda_stream)
        return self.idx

    def local_pair(self, x) -> torch.Tensor:
        """(max bits, global index) of this rank's rows, int32 [2] on this rank's device."""
        if self.local is not None:
            y = self.local.gemv_q4_128_fused(self.blocks, np.asarray(x, np.float32), self.rows, self.H)
            i = int(self.local.argmax(y))
            return torch.tensor([np.float32(y[i]).view(np.int32), self.a + i], dtype=torch.int32)
        self.local_argmax(x)
        return torch.cat([self.val.view(torch.int32), self.idx])

    def local_argmax(self, x):
        """one kernel: this rank's GEMV + first-max argmax into self.val / self.idx (global index)"""
        _lib.call("asdsl_b200_gemv_argmax", _lib.FMT_Q4_128_BANDED, self.quant.data_ptr(), self.scales.data_ptr(),
                  x.data_ptr(), self.logits.data_ptr(), self.val.data_ptr(), self.idx.data_ptr(), self.a,
                  self.scratch.data_ptr(), self.scratch.numel(), self.rows, self.H,
                  torch.cuda.current_stream(self.device).cuda_stream)

    def argmax(self, x) -> tuple[float, int]:
        if self.xchg is not None:
            idx = int(self.fused_step(x).item())
            return float(self.val.item()), idx
        pair = self.local_pair(x)
        if self.world == 1:
            return combine_argmax(pair.view(1, 2))
        return combine_argmax(_all_gather_pairs(pair, self.world).cpu())


class ShardedMLP:
    """gate_up rows and down columns of one layer for this rank (preq2 gs32 blobs), with the
    fused gate_up+SiLU on the local rows and an all-reduce of the down partial sums.

    numerics: "fast" (the engine's default kernels) or "reference_exact" (the kernels that are
    bitwise equal to the reference's compiled GEMV and SwiGLU).  fused=True (GPUs, the default)
    sums the partials with the peer all-reduce kernel; fused=False through torch.distributed.
    `exchange`: an open _VecExchange (hidden floats) to share between several layers' MLPs;
    the caller closes it."""

    def __init__(self, gu_meta, gu_quant, dn_meta, dn_quant, hidden: int, inter: int, local=None, device=None,
                 world=None, rank=None, fused: bool = True, numerics: str = "fast", exchange=None):
        if numerics not in ("fast", "reference_exact"):
            raise ValueError(f"unknown numerics mode {numerics!r}")
        self.numerics = numerics
        self.world, self.rank = _group(world, rank)
        self.H, self.I = hidden, inter
        self.a, self.b = shard_range(inter, self.world, self.rank, 32)
        if self.a % 4 or self.b % 4:
            raise ValueError("gate_up shards must start on 4-row bands")
        self.n = self.b - self.a
        H, I = hidden, inter
        ngH, ngI = H // 32, I // 32
        gm = np.asarray(gu_meta, np.uint8).reshape(2 * I, ngH * 4)
        gq = np.asarray(gu_quant, np.uint8).reshape(2 * I // 4, ngH * 64)
        # local gate rows then local up rows, as the paired SiLU layout expects
        self.gu_meta = np.ascontiguousarray(np.concatenate([gm[self.a : self.b], gm[I + self.a : I + self.b]]))
        self.gu_quant = np.ascontiguousarray(
            np.concatenate([gq[self.a // 4 : self.b // 4], gq[(I + self.a) // 4 : (I + self.b) // 4]]))
        g0, g1 = self.a // 32, self.b // 32
        dm = np.asarray(dn_meta, np.uint8).reshape(H, ngI, 4)
        dq = np.asarray(dn_quant, np.uint8).reshape((H + 3) // 4, ngI, 64)
        self.dn_meta = np.ascontiguousarray(dm[:, g0:g1, :]).reshape(-1)
        self.dn_quant = np.ascontiguousarray(dq[:, g0:g1, :]).reshape(-1)
        self.local = local
        self.vx = None
        if local is None:
            dev = device or torch.device("cuda", torch.cuda.current_device())
            self.device = dev
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a).reshape(-1)).to(dev)  # noqa: E731
            self.d_gm, self.d_gq, self.d_dm, self.d_dq = t(self.gu_meta), t(self.gu_quant), t(self.dn_meta), t(self.dn_quant)
            self.h = torch.empty(self.n, dtype=torch.float32, device=dev)
            self.y = torch.empty(H, dtype=torch.float32, device=dev)
            self.out = torch.empty(H, dtype=torch.float32, device=dev)
            self._own_vx = False
            if exchange is not None:
                self.vx = exchange
            elif fused and world is None and self.world > 1:
                self.vx = _VecExchange(self.world, self.rank, H, dev)
                self._own_vx = True
        else:
            self.device = torch.device("cpu")

    def close(self):
        if self.vx is not None and getattr(self, "_own_vx", False):
            self.vx.close()
        self.vx = None

    def local_partial(self, x):
        """down[:, a:b] . A8(silu(gate[a:b] x) * up[a:b] x): this rank's partial output."""
        if self.local is not None:
            o = self.local
            gu = o.gemv_preq2_fused(self.gu_meta, self.gu_quant, np.asarray(x, np.float32), 2 * self.n, self.H)
            h = o.swiglu(gu[: self.n], gu[self.n :])
            return torch.from_numpy(o.gemv_preq2_fused(self.dn_meta, self.dn_quant, h, self.H, self.n))
        s = torch.cuda.current_stream(self.device).cuda_stream
        if self.numerics == "reference_exact":
            import ctypes

            _lib.call("asdsl_b200_gateup_silu_exact", self.d_gm.data_ptr(), self.d_gq.data_ptr(), x.data_ptr(), None,
                      ctypes.c_float(0.0), self.h.data_ptr(), self.n, self.H, s)
            _lib.call("asdsl_b200_gemv_preq2_fused_exact", self.d_dm.data_ptr(), self.d_dq.data_ptr(),
                      self.h.data_ptr(), None, ctypes.c_float(0.0), self.y.data_ptr(), self.H, self.n, s)
            return self.y
        _lib.call("asdsl_b200_gateup_silu", _lib.FMT_PREQ2, self.d_gm.data_ptr(), self.d_gq.data_ptr(), x.data_ptr(),
                  self.h.data_ptr(), self.n, self.H, s)
        _lib.call("asdsl_b200_gemv_preq2_fused", self.d_dm.data_ptr(), self.d_dq.data_ptr(), self.h.data_ptr(),
                  self.y.data_ptr(), self.H, self.n, 32, s)
        return self.y

    def forward(self, x) -> torch.Tensor:
        y = self.local_partial(x)
        if self.vx is not None:
            self.vx.allreduce(y, self.out, self.H, torch.cuda.current_stream(self.device).cuda_stream)
            return self.out
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(y, op=dist.ReduceOp.SUM)
        return y


def _rows(a, ncols: int):
    """a flat weight blob (numpy or torch, host or device) viewed as [rows, ncols] bytes"""
    if hasattr(a, "reshape") and hasattr(a, "is_cuda"):
        return a.reshape(-1, ncols)
    return np.asarray(a, np.uint8).reshape(-1, ncols)


def _cat(parts):
    if hasattr(parts[0], "is_cuda"):
        return torch.cat([p.contiguous() for p in parts]).contiguous()
    return np.ascontiguousarray(np.concatenate(parts))


def shard_mlp_blobs(L: dict, hidden: int, inter: int, a: int, b: int) -> dict:
    """This rank's preq2 (gs 32) MLP blobs of one layer: gate rows [a, b) then up rows
    [I + a, I + b) of gate_up_proj, and input columns [a, b) of down_proj (whole 32-column
    groups, so the A8 quantization of h[a:b] is the slice of the global one).  Works on numpy
    arrays and on torch tensors (host or device) alike; a, b multiples of 32."""
    H, I = hidden, inter
    ngH, ngI = H // 32, I // 32
    gm = _rows(L["gate_up_proj_meta"], ngH * 4)
    gq = _rows(L["gate_up_proj_quant"], ngH * 64)  # one row per 4-row band
    dm = _rows(L["down_proj_meta"], ngI * 4)
    dq = _rows(L["down_proj_quant"], ngI * 64)
    g0, g1 = a // 32, b // 32
    out = dict(L)
    out["gate_up_proj_meta"] = _cat([gm[a:b], gm[I + a : I + b]]).reshape(-1)
    out["gate_up_proj_quant"] = _cat([gq[a // 4 : b // 4], gq[(I + a) // 4 : (I + b) // 4]]).reshape(-1)
    out["down_proj_meta"] = _cat([dm[:, g0 * 4 : g1 * 4]]).reshape(-1)
    out["down_proj_quant"] = _cat([dq[:, g0 * 64 : g1 * 64]]).reshape(-1)
    return out


class ShardedEngine:
    """The decode engine split over the GPUs of one box: one instance per rank (one process per
    GPU, torch.distributed initialised), each holding its slice of every layer's MLP and of the
    lm_head, the peer all-reduce of the down partials and the in-kernel argmax exchange
    (asdsl_b200_engine_set_shard).  All ranks make the same calls (generate, forward_token_argmax,
    reset_session) and get the same tokens."""

    def __init__(self, engine, vx, xg, inter_range, lm_range):
        self.engine, self.vx, self.xg = engine, vx, xg
        self.inter_range, self.lm_range = inter_range, lm_range

    def __getattr__(self, name):
        if name in ("engine", "vx", "xg"):
            raise AttributeError(name)
        return getattr(self.engine, name)

    def close(self):
        if getattr(self, "engine", None) is not None:
            self.engine.close()
            self.engine = None
        for x in ("vx", "xg"):
            if getattr(self, x, None) is not None:
                getattr(self, x).close()
                setattr(self, x, None)


def sharded_engine_from_model(model: dict, max_seq_len: int | None = None, device=None) -> ShardedEngine:
    """engine_from_model split over the ranks of the default process group: rank r takes
    intermediate rows [a_r, b_r) (128-aligned) of every layer's gate/up and down, and lm_head
    rows [l_r, m_r) (4-aligned) quantized from its slice of the tied fp16 embedding by the engine,
    as the single-GPU engine quantizes the whole.  Fast numerics, per-op chain."""
    from asdsl_b200.kernels._native_unified import EngineConfig, UnifiedEngine

    world, rank = _group()
    dev = device or torch.device("cuda", torch.cuda.current_device())
    c = model["config"]
    H, I, V = c["hidden"], c["inter"], c["vocab"]
    a, b = shard_range(I, world, rank, 128)
    la, lb = shard_range(V, world, rank, 4)
    layers = {i: shard_mlp_blobs(L, H, I, a, b) for i, L in enumerate(model["layers"])}
    emb = model["embed_f16"]
    lm_src = emb[la:lb] if hasattr(emb, "is_cuda") else np.ascontiguousarray(np.asarray(emb).reshape(V, H)[la:lb])
    vx = _VecExchange(world, rank, H, dev)
    xg = _Exchange(world, rank, dev)
    cfg = EngineConfig()
    cfg.num_layers = c["num_layers"]
    cfg.hidden_size = H
    cfg.num_heads = c["n_heads"]
    cfg.num_kv_heads = c["n_kv_heads"]
    cfg.head_dim = c["head_dim"]
    cfg.intermediate_size = b - a
    cfg.vocab_size = V
    cfg.rms_norm_eps = c["eps"]
    cfg.group_size = 32
    cfg.lm_head_group_size = 32
    cfg.max_seq_len = max_seq_len or c["max_seq"]
    cfg.rotary_dim = c["rotary_dim"]
    cfg.weight_format = 0
    try:
        eng = UnifiedEngine(cfg, emb, model["output_norm"], lm_src, model["cos"], model["sin"], layers,
                            numerics="fast", persistent=False,
                            shard={"vx": vx, "xg": xg, "lm_rows": lb - la, "lm_row_base": la})
    except BaseException:
        vx.close()
        xg.close()
        raise
    return ShardedEngine(eng, vx, xg, (a, b), (la, lb))
