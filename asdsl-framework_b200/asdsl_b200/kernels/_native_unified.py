"""Drop-in for the reference's ``asdsl.kernels._native_unified`` module (EngineConfig,
UnifiedEngine), backed by the device-resident decode engine of libasdsl_b200.so.

Reference: asdsl/kernels/native/unified_engine.cpp -- pybind registration :2203-2222
(EngineConfig) and :2655-2713 (UnifiedEngine), weight binding :2240-2442, methods
:2449-2630.  Same constructor arguments, same ``layers_dict`` keys, same method names,
argument meaning and exception classes (std::invalid_argument -> ValueError,
std::out_of_range -> IndexError).

Differences that follow from running on the GPU:
  * weights are copied once into engine-owned device memory (the reference borrows
    the numpy arrays); preq-only layers are repacked to preq2 on the host first;
  * ``forward_token`` returns a reused host buffer like the reference (:2485-2492);
  * ``generate`` replays one CUDA graph per token and copies the tokens back once
    (with stop tokens, once per 16 tokens);
  * an empty prompt raises ValueError (the reference reads stale logits).
The format selection mirrors the reference's environment switches: preq2 blobs
(``*_meta``/``*_quant``) are used unless ``ASDSL_C01`` (gate_up/down) or ``ASDSL_C03``
(qkv/o) select the ``*_g128`` Q4_128 blobs (unified_engine.cpp:1404-1410, :1532-1538).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from asdsl_b200 import _lib
from asdsl_b200.quantization.repack import repack_preq_blocks_to_preq2

_PROJ = ("qkv_proj", "o_proj", "gate_up_proj", "down_proj")


class EngineConfig:
    """unified_engine.h:14-109 (fields bound at unified_engine.cpp:2204-2222)."""

    def __init__(self):
        self.num_layers = 32
        self.hidden_size = 3072
        self.num_heads = 24
        self.num_kv_heads = 8
        self.head_dim = 128
        self.intermediate_size = 8192
        self.vocab_size = 200064
        self.rms_norm_eps = 1e-5
        self.group_size = 32
        self.lm_head_group_size = 0
        self.max_seq_len = 2048
        self.rotary_dim = 96
        self.weight_format = 0

    def _c(self) -> _lib.EngineConfigC:
        c = _lib.EngineConfigC()
        for name, _ in _lib.EngineConfigC._fields_:
            setattr(c, name, getattr(self, name))
        return c


def _env_on(name: str) -> bool:
    v = os.environ.get(name)
    return bool(v) and v[0] != "0"


def _host(a, dtype=None) -> np.ndarray:
    if hasattr(a, "detach"):  # torch tensor
        a = a.detach().cpu().numpy()
    a = np.asarray(a)
    if dtype is not None and a.dtype != dtype:
        a = a.astype(dtype)
    return np.ascontiguousarray(a)


def _ptr(a) -> int:
    if hasattr(a, "data_ptr"):  # torch tensor (CUDA or CPU), contiguous
        return a.data_ptr()
    return a.ctypes.data


def _nbytes(a) -> int:
    return a.numel() * a.element_size() if hasattr(a, "element_size") else a.nbytes


def _blob(a, dtype):
    """A weight / table argument as something with a pointer: CUDA tensors are used where they
    are (the engine copies device to device), everything else becomes a contiguous host array."""
    if hasattr(a, "is_cuda") and a.is_cuda:
        import torch

        tdt = {np.uint8: torch.uint8, np.float32: torch.float32, np.float16: torch.float16}[np.dtype(dtype).type]
        return a.contiguous() if a.dtype == tdt else a.to(tdt).contiguous()
    return _host(a, dtype)


class UnifiedEngine:
    """UnifiedEngine(config, token_embd, output_norm, output_proj, cos_table, sin_table,
    layers_dict, lm_head_preq2_meta=None, lm_head_preq2_quant=None)  (:2662-2682).

    numerics: "fast" (default) or "reference_exact" (every op in the reference's compiled
    operation order: logits and greedy tokens bit-identical to the reference's UnifiedEngine on
    this host; asdsl_b200_engine_set_numerics).  The environment variable ASDSL_B200_NUMERICS
    sets the default."""

    def __init__(self, config, token_embd, output_norm, output_proj, cos_table, sin_table, layers_dict,
                 lm_head_preq2_meta=None, lm_head_preq2_quant=None, persistent: bool | None = None,
                 numerics: str | None = None, shard: dict | None = None):
        lib = _lib.load()
        self._lib = lib
        self.config_ = config
        # shard: {"vx": vector exchange, "xg": argmax exchange, "lm_rows", "lm_row_base"} of
        # asdsl_b200.shard.sharded_engine_from_model (asdsl_b200_engine_set_shard)
        self._shard = shard
        self._e = ctypes.c_void_p()
        _lib.check(lib.asdsl_b200_engine_create(ctypes.byref(config._c()), ctypes.byref(self._e)),
                   "UnifiedEngine")
        try:
            if persistent is not None:
                _lib.check(lib.asdsl_b200_engine_set_persistent(self._e, 1 if persistent else 0), "UnifiedEngine")
            numerics = numerics or os.environ.get("ASDSL_B200_NUMERICS", "fast")
            if numerics not in ("fast", "reference_exact"):
                raise ValueError(f"UnifiedEngine: numerics must be 'fast' or 'reference_exact', got {numerics!r}")
            _lib.check(lib.asdsl_b200_engine_set_numerics(self._e, 1 if numerics == "reference_exact" else 0),
                       "UnifiedEngine")
            self.numerics = numerics
            if shard is not None:
                _lib.check(lib.asdsl_b200_engine_set_shard(self._e, shard["vx"].ptr, shard["xg"].ptr,
                                                           int(shard["lm_rows"]), int(shard["lm_row_base"])),
                           "UnifiedEngine")
            self._load(config, token_embd, output_norm, output_proj, cos_table, sin_table, layers_dict,
                       lm_head_preq2_meta, lm_head_preq2_quant)
        except BaseException:
            lib.asdsl_b200_engine_destroy(self._e)
            self._e = None
            raise
        self._logits = np.empty(config.vocab_size, dtype=np.float32)
        self._vocab = int(config.vocab_size)
        # decode mode as the engine resolved it (asdsl_b200_engine_create reads the same variable)
        self._persistent = bool(persistent) if persistent is not None else \
            os.environ.get("ASDSL_B200_DECODE_KERNEL") == "persistent"

    # ------------------------------------------------------------------ construction
    def _load(self, cfg, token_embd, output_norm, output_proj, cos_table, sin_table, layers_dict, lm_meta,
              lm_quant):
        lib, e = self._lib, self._e
        if hasattr(token_embd, "is_cuda") and token_embd.is_cuda:
            import torch

            emb = token_embd.contiguous() if token_embd.dtype in (torch.float16, torch.float32) else \
                token_embd.float().contiguous()
            emb_f16 = emb.dtype == torch.float16
            emb_n = emb.numel()
        else:
            emb = _host(token_embd)
            if emb.dtype not in (np.float16, np.float32):
                emb = emb.astype(np.float32)
            emb_f16 = emb.dtype == np.float16
            emb_n = emb.size
        if emb_n != cfg.vocab_size * cfg.hidden_size:
            raise ValueError("token_embd must be (vocab_size, hidden_size)")
        norm = _host(output_norm, np.float32).ravel()
        half = cfg.rotary_dim // 2
        cos = _host(cos_table, np.float32)
        sin = _host(sin_table, np.float32)
        if norm.size != cfg.hidden_size:
            raise ValueError("output_norm must have hidden_size elements")
        if cos.size < cfg.max_seq_len * half or sin.size < cfg.max_seq_len * half:
            raise ValueError("cos/sin tables must be (max_seq_len, rotary_dim/2)")
        _lib.check(lib.asdsl_b200_engine_set_globals(e, _ptr(emb), int(emb_f16), _ptr(norm), _ptr(cos), _ptr(sin)),
                   "UnifiedEngine")
        if output_proj is not None:
            if output_proj is token_embd and self._shard is None:
                op, op_f16, op_n = emb, emb_f16, emb_n
            elif hasattr(output_proj, "is_cuda") and output_proj.is_cuda:
                import torch

                op = output_proj.contiguous() if output_proj.dtype in (torch.float16, torch.float32) else \
                    output_proj.float().contiguous()
                op_f16, op_n = op.dtype == torch.float16, op.numel()
            else:
                op = _host(output_proj)
                if op.dtype not in (np.float16, np.float32):
                    op = op.astype(np.float32)
                op_f16, op_n = op.dtype == np.float16, op.size
            lm_rows = int(self._shard["lm_rows"]) if self._shard is not None else cfg.vocab_size
            if op_n != lm_rows * cfg.hidden_size:
                raise ValueError("output_proj must be (vocab_size, hidden_size) (a shard: (lm_rows, hidden_size))")
            _lib.check(lib.asdsl_b200_engine_set_output_proj(e, _ptr(op), int(op_f16)), "UnifiedEngine")
        if lm_meta is not None and lm_quant is not None:
            m = _host(lm_meta, np.uint8).ravel()
            q = _host(lm_quant, np.uint8).ravel()
            _lib.check(lib.asdsl_b200_engine_set_lm_head_preq2(e, _ptr(m), m.size, _ptr(q), q.size), "UnifiedEngine")
        use_c01, use_c03 = _env_on("ASDSL_C01"), _env_on("ASDSL_C03")
        for i in range(cfg.num_layers):
            L = layers_dict[i]
            ra = _blob(L["rms_att"], np.float32).reshape(-1)
            rf = _blob(L["rms_ffn"], np.float32).reshape(-1)
            _lib.check(lib.asdsl_b200_engine_set_layer_norms(e, i, _ptr(ra), _ptr(rf)), "UnifiedEngine")
            for w, name in enumerate(_PROJ):
                rows, cols = self._shape(cfg, w)
                g128 = (use_c01 and name in ("gate_up_proj", "down_proj")) or \
                       (use_c03 and name in ("qkv_proj", "o_proj"))
                if g128 and f"{name}_g128" in L:
                    b = _host(L[f"{name}_g128"], np.uint8).ravel()
                    _lib.check(lib.asdsl_b200_engine_set_projection(e, i, w, _lib.FMT_Q4_128, _ptr(b), b.size,
                                                                    None, 0), "UnifiedEngine")
                    continue
                if f"{name}_meta" in L and f"{name}_quant" in L:
                    m = _blob(L[f"{name}_meta"], np.uint8).reshape(-1)
                    q = _blob(L[f"{name}_quant"], np.uint8).reshape(-1)
                elif name in L:
                    m, q = repack_preq_blocks_to_preq2(_host(L[name], np.uint8).ravel(), rows, cols, 32)
                    m, q = m.ravel(), q.ravel()
                else:
                    raise KeyError(name)
                _lib.check(lib.asdsl_b200_engine_set_projection(e, i, w, _lib.FMT_PREQ2, _ptr(m), _nbytes(m), _ptr(q),
                                                                _nbytes(q)), "UnifiedEngine")
                # the QCSD draft bank (unified_engine.cpp:2387-2440): packed 2-bit codes, fp32 scales
                # and biases, used by forward_token_draft_q2
                qk = f"q2_{name}"
                if qk in L and f"q2_{name[:-5]}_scales" in L and f"q2_{name[:-5]}_biases" in L:
                    qw = _blob(L[qk], np.uint8).reshape(-1)
                    qs = _blob(L[f"q2_{name[:-5]}_scales"], np.float32).reshape(-1)
                    qb = _blob(L[f"q2_{name[:-5]}_biases"], np.float32).reshape(-1)
                    _lib.check(lib.asdsl_b200_engine_set_projection_q2(e, i, w, _ptr(qw), _nbytes(qw), _ptr(qs), _ptr(qb),
                                                                       _nbytes(qs) // 4), "UnifiedEngine")
        _lib.check(lib.asdsl_b200_engine_finalize(e), "UnifiedEngine")

    @staticmethod
    def _shape(cfg, which: int):
        qd = cfg.num_heads * cfg.head_dim
        kvd = cfg.num_kv_heads * cfg.head_dim
        return [(qd + 2 * kvd, cfg.hidden_size), (cfg.hidden_size, qd), (2 * cfg.intermediate_size, cfg.hidden_size),
                (cfg.hidden_size, cfg.intermediate_size)][which]

    def close(self):
        if getattr(self, "_e", None):
            self._lib.asdsl_b200_engine_destroy(self._e)
            self._e = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ decode
    def forward_token(self, token: int, pos: int) -> np.ndarray:
        """Logits of one decode step; the returned buffer is reused by the next call (:2485-2492)."""
        _lib.check(self._lib.asdsl_b200_engine_forward_token(self._e, int(token), int(pos), _ptr(self._logits), None),
                   "forward_token")
        return self._logits

    def forward_token_prefill(self, token: int, pos: int) -> None:
        """Forward one token updating KV; skip lm_head (:2494-2497)."""
        _lib.check(self._lib.asdsl_b200_engine_forward_token(self._e, int(token), int(pos), None, None),
                   "forward_token_prefill")

    def forward_token_draft(self, token: int, pos: int) -> np.ndarray:
        """Draft step: forward_token with the skip-masked layers left out (:2701;
        unified_engine.cpp:1790-1794); the returned buffer is reused."""
        _lib.check(self._lib.asdsl_b200_engine_forward_token_draft(self._e, int(token), int(pos),
                                                                   _ptr(self._logits), None, 0), "forward_token_draft")
        return self._logits

    def forward_token_draft_q2(self, token: int, pos: int) -> np.ndarray:
        """Draft step with the 2-bit draft bank in place of the 4-bit projections where the layer
        has one (UnifiedEngine::forward_token_draft_q2, unified_engine.cpp:1796-1802)."""
        _lib.check(self._lib.asdsl_b200_engine_forward_token_draft(self._e, int(token), int(pos),
                                                                   _ptr(self._logits), None, 1), "forward_token_draft_q2")
        return self._logits

    def set_skip_mask(self, mask) -> None:
        """Layers whose mask entry is true are left out of draft steps (:2711;
        unified_engine.cpp:1309-1317)."""
        m = np.ascontiguousarray(np.asarray(list(mask), dtype=bool).astype(np.uint8))
        _lib.check(self._lib.asdsl_b200_engine_set_skip_mask(self._e, _ptr(m) if m.size else None, int(m.size)),
                   "set_skip_mask")

    def clear_skip_mask(self) -> None:
        _lib.check(self._lib.asdsl_b200_engine_clear_skip_mask(self._e), "clear_skip_mask")

    def forward_token_argmax(self, token: int, pos: int) -> int:
        """Single decode step; returns the argmax token id (:2499-2506)."""
        out = ctypes.c_int32(0)
        logits = None if self._shard is not None else _ptr(self._logits)
        _lib.check(self._lib.asdsl_b200_engine_forward_token(self._e, int(token), int(pos), logits,
                                                             ctypes.byref(out)), "forward_token_argmax")
        return int(out.value)

    def forward_verify_serial_all_logits(self, prompt, start_pos: int) -> np.ndarray:
        """forward_token(prompt[i], start_pos + i) for every i; float32 [len(prompt) * vocab], row i
        the logits of step i (:2602-2611 over forward_verify_serial, unified_engine.cpp:1767-1772).
        All steps run on the device back to back with one copy out."""
        p = np.ascontiguousarray(np.asarray(list(prompt), dtype=np.int32))
        out = np.empty(p.size * self._vocab, dtype=np.float32)
        if p.size:
            _lib.check(self._lib.asdsl_b200_engine_forward_verify(self._e, _ptr(p), int(p.size), int(start_pos),
                                                                  _ptr(out)), "forward_verify_serial_all_logits")
        return out

    def forward_batch_all_logits(self, prompt, start_pos: int) -> np.ndarray:
        """Speculative-verify logits (:2591-2600).  The reference's forward_verify_batch takes the
        serial per-token path whenever preq2 weights are in use (unified_engine.cpp:1783-1787) so
        that PLD stays lossless: the result must equal forward_verify_serial_all_logits.  Here the
        batched forward gives those rows bit for bit with one weight read per pass, so it runs that
        (the persistent-kernel mode, whose K-splits differ, keeps the serial replays)."""
        if self._persistent or self.numerics == "reference_exact":
            return self.forward_verify_serial_all_logits(prompt, start_pos)
        return self.forward_verify_batch_raw_all_logits(prompt, start_pos)

    def forward_batch(self, prompt, start_pos: int) -> np.ndarray:
        """prompt[i] at position start_pos + i, up to 16 tokens per weight read (:2526-2534 over
        UnifiedEngine::forward_batch, unified_engine.cpp:1117); float32 [vocab], the last token's
        logits.  Bit-identical to forward_token over the same tokens (logits and KV cache)."""
        p = np.ascontiguousarray(np.asarray(list(prompt), dtype=np.int32))
        out = np.zeros(self._vocab, dtype=np.float32)
        if p.size:
            _lib.check(self._lib.asdsl_b200_engine_forward_batch(self._e, _ptr(p), int(p.size), int(start_pos),
                                                                 _ptr(out), 0), "forward_batch")
        return out

    def forward_verify_batch_raw_all_logits(self, prompt, start_pos: int) -> np.ndarray:
        """The batched verify (:2613-2625: forward_batch(..., all_logits=true)); float32
        [len(prompt) * vocab].  Here it equals forward_verify_serial_all_logits bit for bit."""
        p = np.ascontiguousarray(np.asarray(list(prompt), dtype=np.int32))
        out = np.empty(p.size * self._vocab, dtype=np.float32)
        if p.size:
            _lib.check(self._lib.asdsl_b200_engine_forward_batch(self._e, _ptr(p), int(p.size), int(start_pos),
                                                                 _ptr(out), 1), "forward_verify_batch_raw_all_logits")
        return out

    def generate(self, prompt, max_tokens: int) -> list[int]:
        return self.generate_with_stops(prompt, max_tokens, [])

    def generate_with_stops(self, prompt, max_tokens: int, stop_tokens) -> list[int]:
        p = np.ascontiguousarray(np.asarray(list(prompt), dtype=np.int32))
        s = np.ascontiguousarray(np.asarray(list(stop_tokens), dtype=np.int32))
        mt = max(int(max_tokens), 0)
        out = np.zeros(p.size + mt + 1, dtype=np.int32)
        n = ctypes.c_int(0)
        rc = self._lib.asdsl_b200_engine_generate(self._e, _ptr(p) if p.size else None, int(p.size), mt,
                                                  _ptr(s) if s.size else None, int(s.size), _ptr(out), int(out.size),
                                                  ctypes.byref(n))
        _lib.check(rc, "generate")
        return [int(t) for t in out[: n.value]]

    # ------------------------------------------------------------------ session / KV
    def reset_session(self) -> None:
        _lib.check(self._lib.asdsl_b200_engine_reset_session(self._e), "reset_session")

    def get_kv_seq_len(self) -> int:
        v = ctypes.c_int(0)
        _lib.check(self._lib.asdsl_b200_engine_get_kv_seq_len(self._e, ctypes.byref(v)), "get_kv_seq_len")
        return int(v.value)

    def truncate_kv(self, new_len: int) -> None:
        _lib.check(self._lib.asdsl_b200_engine_truncate_kv(self._e, int(new_len)), "truncate_kv")

    def snapshot_kv(self) -> None:
        _lib.check(self._lib.asdsl_b200_engine_snapshot_kv(self._e), "snapshot_kv")

    def restore_kv(self) -> None:
        _lib.check(self._lib.asdsl_b200_engine_restore_kv(self._e), "restore_kv")

    def export_lm_head_preq2(self):
        """Copy of the lm_head preq2 blobs (meta, quant) (:2470-2483)."""
        cfg = self.config_
        fmt = ctypes.c_int(-1)
        _lib.check(self._lib.asdsl_b200_engine_export_lm_head(self._e, ctypes.byref(fmt), None, 0, None, 0),
                   "export_lm_head_preq2")
        if fmt.value != _lib.FMT_PREQ2:
            raise RuntimeError("export_lm_head_preq2: lm_head preq2 not ready")
        ng = cfg.hidden_size // 32
        meta = np.empty(cfg.vocab_size * ng * 4, dtype=np.uint8)
        quant = np.empty(((cfg.vocab_size + 3) // 4) * ng * 64, dtype=np.uint8)
        _lib.check(self._lib.asdsl_b200_engine_export_lm_head(self._e, ctypes.byref(fmt), _ptr(meta), meta.size,
                                                              _ptr(quant), quant.size), "export_lm_head_preq2")
        return meta, quant

    # ------------------------------------------------------------------ device-level access
    def stream_ptr(self) -> int:
        s = ctypes.c_void_p()
        _lib.check(self._lib.asdsl_b200_engine_stream(self._e, ctypes.byref(s)), "stream")
        return int(s.value or 0)

    def set_position(self, pos: int, token: int = -1) -> None:
        _lib.check(self._lib.asdsl_b200_engine_set_position(self._e, int(pos), int(token)), "set_position")

    def replay(self, n: int, decode: bool = True) -> None:
        """Enqueue n decode (or prefill) graph replays on the engine stream without synchronising."""
        _lib.check(self._lib.asdsl_b200_engine_replay(self._e, 1 if decode else 0, int(n)), "replay")

    def profile_step(self, decode: bool = True) -> list[dict]:
        """Per-op timing of one persistent decode step at the current position: for each op its
        kind, work time (earliest start to latest end over CTAs) and barrier time, in us."""
        cap = 4 * self.config_.num_layers * 5 + 16
        buf = (ctypes.c_ulonglong * (3 * cap))()
        n = ctypes.c_int(0)
        _lib.check(self._lib.asdsl_b200_engine_profile_step(self._e, 1 if decode else 0, buf, cap, ctypes.byref(n)),
                   "profile_step")
        names = ["embed"]
        for _ in range(self.config_.num_layers):
            names += ["qkv", "attention", "o", "gate_up", "down"]
        names += ["lm_head", "argmax"] if decode else []
        out = []
        for i in range(n.value):
            t0, t1, t2 = buf[3 * i], buf[3 * i + 1], buf[3 * i + 2]
            out.append({"op": names[i] if i < len(names) else str(i), "work_us": (t1 - t0) / 1e3,
                        "barrier_us": (t2 - t1) / 1e3 if t2 >= t1 else 0.0})
        return out

    _BUFFERS = ("resid", "qkv", "att", "h", "logits", "kq", "vq", "ks", "vs")

    def read_buffer(self, name: str) -> np.ndarray:
        """Host copy of an engine buffer (tests): the last layer's values for the activations."""
        cfg = self.config_
        qd, kvd = cfg.num_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim
        per_codes = cfg.num_layers * cfg.max_seq_len * kvd
        per_scales = cfg.num_layers * cfg.max_seq_len * cfg.num_kv_heads * (cfg.head_dim // 64)
        shapes = {"resid": (cfg.hidden_size, np.float32), "qkv": (qd + 2 * kvd, np.float32),
                  "att": (qd, np.float32), "h": (cfg.intermediate_size, np.float32),
                  "logits": (cfg.vocab_size, np.float32), "kq": (per_codes, np.int8), "vq": (per_codes, np.int8),
                  "ks": (per_scales, np.float32), "vs": (per_scales, np.float32)}
        n, dt = shapes[name]
        out = np.empty(n, dtype=dt)
        _lib.check(self._lib.asdsl_b200_engine_read_buffer(self._e, self._BUFFERS.index(name), _ptr(out), out.nbytes),
                   "read_buffer")
        return out


def engine_from_model(model: dict, lm_head_group_size: int = 32, max_seq_len: int | None = None,
                      use_preq2_cache: bool = False, persistent: bool | None = None,
                      numerics: str | None = None) -> UnifiedEngine:
    """UnifiedEngine over a synthetic model of asdsl_b200.inference.synthetic.build_model, wired as
    the reference's unified_bridge.build_unified_engine does (tied fp16 embedding as lm_head source)."""
    c = model["config"]
    cfg = EngineConfig()
    cfg.num_layers = c["num_layers"]
    cfg.hidden_size = c["hidden"]
    cfg.num_heads = c["n_heads"]
    cfg.num_kv_heads = c["n_kv_heads"]
    cfg.head_dim = c["head_dim"]
    cfg.intermediate_size = c["inter"]
    cfg.vocab_size = c["vocab"]
    cfg.rms_norm_eps = c["eps"]
    cfg.group_size = 32
    cfg.lm_head_group_size = lm_head_group_size
    cfg.max_seq_len = max_seq_len or c["max_seq"]
    cfg.rotary_dim = c["rotary_dim"]
    cfg.weight_format = 0
    layers = {i: L for i, L in enumerate(model["layers"])}
    meta = model.get("lm_meta") if use_preq2_cache else None
    quant = model.get("lm_quant") if use_preq2_cache else None
    return UnifiedEngine(cfg, model["embed_f16"], model["output_norm"], None if meta is not None else model["embed_f16"],
                         model["cos"], model["sin"], layers, meta, quant, persistent=persistent, numerics=numerics)
