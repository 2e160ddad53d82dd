"""Python face of the CPU oracle.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker (or the timed CPU baseline); the product
package never does.

Two back ends, same call shapes:
  * ``Oracle``    -- our plain-C restatement (oracle/asdsl_oracle.c -> liboracle.so);
  * ``RefKernels`` -- the reference's own AVX2/OpenMP kernels compiled from its
    sources into oracle/_ref/ (oracle/Makefile), reached through ref_shim.cpp.
"""

from __future__ import annotations

import ctypes
import glob
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_P = ctypes.c_void_p
_I = ctypes.c_int


def _p(a):
    return None if a is None else a.ctypes.data_as(_P)


def reference_root() -> str | None:
    """The reference source tree: $ASDSL_REFERENCE, else a "reference" directory beside the repo."""
    root = os.environ.get("ASDSL_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return root if os.path.isdir(os.path.join(root, "asdsl", "kernels", "native")) else None


def build(ref: bool = False) -> None:
    """Build liboracle.so (and the reference library when `ref` and the sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    root = reference_root()
    if ref and root:
        subprocess.run(["make", "-s", "-C", HERE, "ref", "-j8", f"REF={root}"], check=True)


def host_has_avx_vnni() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return "avx_vnni" in line.split()
    except OSError:
        pass
    return False


def ref_lib_path() -> str | None:
    """The reference library: its -mavxvnni build on hosts with AVX-VNNI (the reference's
    HAVE_AVXVNNI path), else the plain AVX2 build."""
    if host_has_avx_vnni():
        c = glob.glob(os.path.join(REF_DIR, "vnni", "_native_unified*.so"))
        if c:
            return c[0]
    c = glob.glob(os.path.join(REF_DIR, "_native_unified*.so"))
    return c[0] if c else None


class Oracle:
    """Our C restatement of the reference's hot path."""

    def __init__(self, path: str = ORACLE_LIB):
        if not os.path.exists(path):
            build()
        self.lib = ctypes.CDLL(path)
        L = self.lib
        for n in ("or_gemv_preq2_fused", "or_gemv_q4km"):
            getattr(L, n).restype = None
        L.or_engine_create.restype = _P
        L.or_engine_forward_token.restype = _I
        L.or_argmax.restype = _I

    # -- the host's approximate reciprocals and C-library expf (reference-exact checks)
    def host_rcp(self, x: float) -> float:
        f = self.lib.or_host_rcp
        f.restype, f.argtypes = ctypes.c_float, [ctypes.c_float]
        return f(x)

    def host_rsqrt(self, x: float) -> float:
        f = self.lib.or_host_rsqrt
        f.restype, f.argtypes = ctypes.c_float, [ctypes.c_float]
        return f(x)

    def expf_array(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        f = self.lib.or_expf_array
        f.restype, f.argtypes = None, [_P, _P, ctypes.c_long]
        f(_p(x), _p(y), x.size)
        return y

    # -- activation quantization
    def quantize_activation(self, x, gs=32):
        x = np.ascontiguousarray(x, np.float32)
        K = x.size
        xq = np.zeros(K, np.int8)
        xs = np.zeros(K // gs, np.float32)
        xsum = np.zeros(K // gs, np.int32)
        self.lib.or_quantize_activation(_p(x), _p(xq), _p(xs), _p(xsum), _I(K), _I(gs))
        return xq, xs, xsum

    def quantize_activation_q4k(self, x):
        x = np.ascontiguousarray(x, np.float32)
        K = x.size
        xq = np.zeros(K, np.int8)
        xs = np.zeros(K // 32, np.float32)
        self.lib.or_quantize_activation_q4k(_p(x), _p(xq), _p(xs), _I(K))
        return xq, xs

    # -- GEMVs
    def gemv_preq2_q8(self, meta, quant, xq, xs, M, K):
        y = np.zeros(M, np.float32)
        self.lib.or_gemv_preq2_q8(_p(np.ascontiguousarray(meta)), _p(np.ascontiguousarray(quant)),
                                  _p(np.ascontiguousarray(xq)), _p(np.ascontiguousarray(xs, np.float32)),
                                  _p(y), _I(M), _I(K))
        return y

    def gemv_preq2_fused(self, meta, quant, x, M, K):
        y = np.zeros(M, np.float32)
        self.lib.or_gemv_preq2_fused(_p(np.ascontiguousarray(meta)), _p(np.ascontiguousarray(quant)),
                                     _p(np.ascontiguousarray(x, np.float32)), _p(y), _I(M), _I(K))
        return y

    def gemv_preq_q8(self, blocks, xq, xs, M, K):
        y = np.zeros(M, np.float32)
        self.lib.or_gemv_preq_q8(_p(np.ascontiguousarray(blocks)), _p(np.ascontiguousarray(xq)),
                                 _p(np.ascontiguousarray(xs, np.float32)), _p(y), _I(M), _I(K))
        return y

    def gemv_preq_fused(self, blocks, x, M, K):
        xq, xs, _ = self.quantize_activation(x, 32)
        return self.gemv_preq_q8(blocks, xq, xs, M, K)

    def gemv_q4_128_q8(self, blocks, xq, xs, M, K):
        y = np.zeros(M, np.float32)
        self.lib.or_gemv_q4_128_q8(_p(np.ascontiguousarray(blocks)), _p(np.ascontiguousarray(xq)),
                                   _p(np.ascontiguousarray(xs, np.float32)), _p(y), _I(M), _I(K))
        return y

    def gemv_q4_128_fused(self, blocks, x, M, K):
        xq, xs, _ = self.quantize_activation(x, 128)
        return self.gemv_q4_128_q8(blocks, xq, xs, M, K)

    def gemm_q4_128_f32(self, blocks, X, M, K, gs=128, y=None):
        """Batched fp32-activation Q4_128 GEMM (gemm_q4_128_q8_avx2); X [B][K] -> Y [B][M], rows
        b >= 64 left as given in `y` (zeros by default)."""
        X = np.ascontiguousarray(X, np.float32)
        B = X.shape[0]
        y = np.zeros((B, M), np.float32) if y is None else np.array(y, np.float32, copy=True)
        if self.lib.or_gemm_q4_128_f32(_p(np.ascontiguousarray(blocks)), _p(X), _p(y), _I(M), _I(K), _I(gs),
                                       _I(B)):
            raise ValueError("gemm_q4_128_q8_avx2: group_size must be 128")
        return y

    def gemv_s256_q8(self, blocks, xq, xs, M, K):
        y = np.zeros(M, np.float32)
        self.lib.or_gemv_q4_s256_q8(_p(np.ascontiguousarray(blocks)), _p(np.ascontiguousarray(xq)),
                                    _p(np.ascontiguousarray(xs, np.float32)), _p(y), _I(M), _I(K))
        return y

    def gemv_q4km(self, w, x, M, K):
        y = np.zeros(M, np.float32)
        self.lib.or_gemv_q4km(_p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(x, np.float32)), _p(y),
                              _I(M), _I(K))
        return y

    def gemv_q4_packed(self, w, x, s, b, M, K, gs):
        y = np.zeros(M, np.float32)
        self.lib.or_gemv_q4_packed(_p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(x, np.float32)),
                                   _p(np.ascontiguousarray(s, np.float32)), _p(np.ascontiguousarray(b, np.float32)),
                                   _p(y), _I(M), _I(K), _I(gs))
        return y

    def gemv_q2(self, packed, w, x, s, b, M, K, gs):
        y = np.zeros(M, np.float32)
        f = self.lib.or_gemv_q2_packed if packed else self.lib.or_gemv_q2_unpacked
        f(_p(np.ascontiguousarray(w, np.uint8)), _p(np.ascontiguousarray(x, np.float32)),
          _p(np.ascontiguousarray(s, np.float32)), _p(np.ascontiguousarray(b, np.float32)), _p(y), _I(M), _I(K),
          _I(gs))
        return y

    # -- engine-side pieces
    def lmhead_quant_preq2(self, w_f16, rows, cols):
        w = np.ascontiguousarray(w_f16, np.float16).view(np.uint16)
        ng = cols // 32
        meta = np.zeros(rows * ng * 4, np.uint8)
        quant = np.zeros(((rows + 3) // 4) * ng * 64, np.uint8)
        self.lib.or_lmhead_quant_q4_32_preq2(_p(w), _p(meta), _p(quant), _I(rows), _I(cols))
        return meta, quant

    def lmhead_quant_q4_128(self, w_f16, rows, cols):
        w = np.ascontiguousarray(w_f16, np.float16).view(np.uint16)
        out = np.zeros(rows * (cols // 128) * 66, np.uint8)
        self.lib.or_lmhead_quant_q4_128(_p(w), _p(out), _I(rows), _I(cols))
        return out

    def swiglu(self, gate, up):
        g = np.array(gate, np.float32, copy=True)
        self.lib.or_swiglu(_p(g), _p(np.ascontiguousarray(up, np.float32)), _I(g.size))
        return g

    def argmax(self, v):
        v = np.ascontiguousarray(v, np.float32)
        return int(self.lib.or_argmax(_p(v), _I(v.size)))


class OracleEngine:
    """UnifiedEngine::forward_token restated in C (C0 path: preq2 g32 everywhere)."""

    class _Model(ctypes.Structure):
        _fields_ = [(n, _I) for n in ("num_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "inter",
                                      "vocab", "max_seq", "rotary_dim")] + [
            ("eps", ctypes.c_float),
            ("embed_f16", _P), ("output_norm", _P), ("lm_meta", _P), ("lm_quant", _P),
            ("cos_t", _P), ("sin_t", _P), ("rms_att", _P), ("rms_ffn", _P),
            ("qkv_meta", _P), ("qkv_quant", _P), ("o_meta", _P), ("o_quant", _P),
            ("gu_meta", _P), ("gu_quant", _P), ("dn_meta", _P), ("dn_quant", _P)]

    def __init__(self, model: dict, oracle: Oracle | None = None):
        self.o = oracle or Oracle()
        c = model["config"]
        self.cfg = c
        self._keep = []

        def arr(a, dt):
            a = np.ascontiguousarray(a, dt)
            self._keep.append(a)
            return a

        def ptrs(name, dt):
            xs = [arr(layer[name], dt) for layer in model["layers"]]
            t = (_P * len(xs))(*[x.ctypes.data for x in xs])
            self._keep.append(t)
            return ctypes.cast(t, _P)

        m = self._Model()
        for k in ("num_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "inter", "vocab", "max_seq",
                  "rotary_dim"):
            setattr(m, k, int(c[k]))
        m.eps = float(c["eps"])
        m.embed_f16 = arr(model["embed_f16"], np.float16).ctypes.data
        m.output_norm = arr(model["output_norm"], np.float32).ctypes.data
        m.lm_meta = arr(model["lm_meta"], np.uint8).ctypes.data
        m.lm_quant = arr(model["lm_quant"], np.uint8).ctypes.data
        m.cos_t = arr(model["cos"], np.float32).ctypes.data
        m.sin_t = arr(model["sin"], np.float32).ctypes.data
        m.rms_att = ptrs("rms_att", np.float32)
        m.rms_ffn = ptrs("rms_ffn", np.float32)
        for short, name in (("qkv", "qkv_proj"), ("o", "o_proj"), ("gu", "gate_up_proj"), ("dn", "down_proj")):
            setattr(m, short + "_meta", ptrs(name + "_meta", np.uint8))
            setattr(m, short + "_quant", ptrs(name + "_quant", np.uint8))
        self._m = m
        self.h = self.o.lib.or_engine_create(ctypes.byref(m))
        self.logits = np.zeros(int(c["vocab"]), np.float32)

    def forward_token(self, token: int, pos: int, want_logits: bool = True):
        rc = self.o.lib.or_engine_forward_token(_P(self.h), _I(token), _I(pos),
                                                _p(self.logits) if want_logits else None)
        if rc:
            raise IndexError("forward_token: token or pos out of range")
        return self.logits.copy() if want_logits else None

    def generate(self, prompt, max_tokens):
        out = list(prompt)
        logits = None
        for i, t in enumerate(prompt):
            logits = self.forward_token(t, i, i == len(prompt) - 1)
        pos = len(prompt)
        margins = []
        for _ in range(max_tokens):
            srt = np.sort(logits)
            margins.append(float(srt[-1] - srt[-2]))
            best = self.o.argmax(logits)
            out.append(best)
            logits = self.forward_token(best, pos, True)
            pos += 1
        return out, margins

    def close(self):
        if self.h:
            self.o.lib.or_engine_destroy(_P(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


class RefKernels:
    """The reference's compiled kernels (oracle/_ref), via ref_shim.cpp."""

    def __init__(self, path: str | None = None):
        path = path or ref_lib_path()
        if not path:
            raise FileNotFoundError("oracle/_ref not built (make -C oracle ref)")
        self.path = path
        self.lib = ctypes.CDLL(path)

    def _chk(self, rc):
        if rc:
            raise ValueError("reference kernel raised")

    def quantize_activation(self, x, gs=32):
        x = np.ascontiguousarray(x, np.float32)
        xq = np.zeros(x.size, np.int8)
        xs = np.zeros(x.size // gs, np.float32)
        self._chk(self.lib.ref_quantize_activation(_p(x), _p(xq), _p(xs), _I(x.size), _I(gs)))
        return xq, xs

    def gemv_preq2_fused(self, meta, quant, x, M, K):
        y = np.zeros(M, np.float32)
        self._chk(self.lib.ref_gemv_preq2_fused(_p(np.ascontiguousarray(meta)), _p(np.ascontiguousarray(quant)),
                                                _p(np.ascontiguousarray(x, np.float32)), _p(y), _I(M), _I(K), _I(32)))
        return y

    def swiglu(self, gate, up):
        """UnifiedEngine::swiglu_inplace (unified_engine.cpp:836-857): silu(gate) * up."""
        g = np.array(gate, np.float32, copy=True)
        u = np.array(up, np.float32, copy=True)
        self._chk(self.lib.ref_swiglu(_p(g), _p(u), _I(g.size)))
        return g

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        self._chk(self.lib.ref_rmsnorm(_p(out), _p(x), _p(np.ascontiguousarray(w, np.float32)), _I(x.size),
                                       ctypes.c_float(eps)))
        return out

    def gemv_preq_q8(self, blocks, xq, xs, M, K):
        y = np.zeros(M, np.float32)
        self._chk(self.lib.ref_gemv_q4_32_preq(_p(np.ascontiguousarray(blocks)), _p(xq), _p(xs), _p(y), _I(M),
                                               _I(K), _I(32)))
        return y

    def gemv_preq_fused(self, blocks, x, M, K):
        y = np.zeros(M, np.float32)
        self._chk(self.lib.ref_gemv_q4_32_preq_fused(_p(np.ascontiguousarray(blocks)),
                                                     _p(np.ascontiguousarray(x, np.float32)), _p(y), _I(M), _I(K),
                                                     _I(32)))
        return y

    def gemv_q4_128_q8(self, blocks, xq, xs, M, K):
        y = np.zeros(M, np.float32)
        self._chk(self.lib.ref_gemv_q4_128(_p(np.ascontiguousarray(blocks)), _p(xq), _p(xs), _p(y), _I(M), _I(K),
                                           _I(128)))
        return y

    def gemm_q4_128_f32(self, blocks, X, M, K, gs=128, y=None):
        X = np.ascontiguousarray(X, np.float32)
        B = X.shape[0]
        y = np.zeros((B, M), np.float32) if y is None else np.array(y, np.float32, copy=True)
        self._chk(self.lib.ref_gemm_q4_128(_p(np.ascontiguousarray(blocks)), _p(X), _p(y), _I(M), _I(K), _I(gs),
                                           _I(B)))
        return y

    def gemv_s256_q8(self, blocks, xq, xs, M, K):
        y = np.zeros(M, np.float32)
        self._chk(self.lib.ref_gemv_q4_s256(_p(np.ascontiguousarray(blocks)), _p(xq), _p(xs), _p(y), _I(M), _I(K),
                                            _I(32)))
        return y

    def gemv_q4km(self, w, x, M, K):
        y = np.zeros(M, np.float32)
        self._chk(self.lib.ref_gemv_q4km(_p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(x, np.float32)),
                                         _p(y), _I(M), _I(K)))
        return y

    def gemv_q2(self, packed, w, x, s, b, M, K, gs):
        y = np.zeros(M, np.float32)
        f = self.lib.ref_gemv_q2_packed if packed else self.lib.ref_gemv_q2_unpacked
        self._chk(f(_p(np.ascontiguousarray(w, np.uint8)), _p(np.ascontiguousarray(x, np.float32)),
                    _p(np.ascontiguousarray(s, np.float32)), _p(np.ascontiguousarray(b, np.float32)), _p(y), _I(M),
                    _I(K), _I(gs)))
        return y

    def gemv_q4_packed(self, w, x, s, b, M, K, gs):
        y = np.zeros(M, np.float32)
        self._chk(self.lib.ref_gemv_q4_packed(_p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(x, np.float32)),
                                              _p(np.ascontiguousarray(s, np.float32)),
                                              _p(np.ascontiguousarray(b, np.float32)), _p(y), _I(M), _I(K), _I(gs)))
        return y


def rel_err(a, b) -> float:
    """max|a-b| / max|b| -- the north-star GEMV tolerance metric."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / (np.max(np.abs(b)) + 1e-30))
