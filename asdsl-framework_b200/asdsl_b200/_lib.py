"""ctypes binding of the C ABI in include/asdsl_b200.h (libasdsl_b200.so).

The shared library is built in-tree (``__graft_entry__.build()`` or
``python -m asdsl_b200.build``) next to this file.  There is no fallback: if the
library or a CUDA device is missing, every native call raises RuntimeError, as
the reference does when its native extension is absent
(asdsl/kernels/gemv_q4.py:373-374).

Status codes map onto the reference's exception classes:
std::invalid_argument -> ValueError, std::out_of_range -> IndexError,
anything else -> RuntimeError.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# ASDSL_B200_TIMELINE=1 loads the timeline build (per-CTA records compiled into the kernels)
TIMELINE_LIB_PATH = os.path.join(_HERE, "libasdsl_b200_timeline.so")
LIB_PATH = (TIMELINE_LIB_PATH if os.environ.get("ASDSL_B200_TIMELINE", "0") not in ("", "0")
            else os.path.join(_HERE, "libasdsl_b200.so"))

OK, EINVAL, ERANGE, ECUDA, ENCCL, ETIMEOUT, ENOMEM = range(7)

FMT_PREQ2, FMT_PREQ, FMT_Q4_128, FMT_S256, FMT_Q4_128_BANDED, FMT_Q4K = 0, 1, 2, 3, 4, 5

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> argtypes (restype is int unless listed in _RESTYPES)
_SIGS = {
    "asdsl_b200_version": [],
    "asdsl_b200_last_error": [],
    "asdsl_b200_device_status": [_P, _I],
    "asdsl_b200_timeline_set": [_P, ctypes.c_uint],
    "asdsl_b200_layer_create": [_P] * 11 + [_I] * 4 + [_P],
    "asdsl_b200_layer_forward": [_P, _P, _P],
    "asdsl_b200_layer_destroy": [_P],
    "asdsl_b200_host_to_device": [_P, _P, ctypes.c_longlong, _P],
    "asdsl_b200_device_to_host": [_P, _P, ctypes.c_longlong, _P],
    "asdsl_b200_timeline_bytes": [ctypes.c_uint],
    "asdsl_b200_selftest_bounded_wait": [_I, _P],
    "asdsl_b200_set_launch_policy": [_I, _I],
    "asdsl_b200_set_mma_min_tokens": [_I],
    "asdsl_b200_quantize_activation": [_P, _P, _P, _P, _I, _I, _P],
    "asdsl_b200_gemv_preq2_fused": [_P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_gemv_preq2": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_gemv_q4_32_preq": [_P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_gemv_q4_32_preq_fused": [_P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_gemv_q4_128": [_P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_gemv_q4_128_fused": [_P, _P, _P, _I, _I, _P],
    "asdsl_b200_gemv_q4_s256": [_P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_gemv_q4km": [_P, _P, _P, _I, _I, _P],
    "asdsl_b200_gemv_q4_packed": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "asdsl_b200_gemv_q4_unpacked": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_matmul_batch_q4": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "asdsl_b200_argmax_scratch_bytes": [],
    "asdsl_b200_relayout_q4_128": [_P, _P, _P, _I, _I, _P],
    "asdsl_b200_quantize_weights": [_P, ctypes.c_longlong, _I, _I, _I, _I, _P, _P, _P, _P],
    "asdsl_b200_repack_preq2": [_P, _P, _P, _I, _I, _P, _P, _P],
    "asdsl_b200_repack_q4_128_f32": [_P, _I, _I, _P, _P],
    "asdsl_b200_requant_q4_128": [_P, _P, _P, _I, _I, _P, _P],
    "asdsl_b200_gemv_q4_128_banded": [_P, _P, _P, _P, _I, _I, _P],
    "asdsl_b200_gemv_argmax": [_I, _P, _P, _P, _P, _P, _P, _I, _P, _SZ, _I, _I, _P],
    "asdsl_b200_gemv_argmax_static": [_I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_gateup_silu": [_I, _P, _P, _P, _P, _I, _I, _P],
    "asdsl_b200_gemv_multi": [_I, _P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_gemv_preq2_fused_exact": [_P, _P, _P, _P, _F, _P, _I, _I, _P],
    "asdsl_b200_gateup_silu_exact": [_P, _P, _P, _P, _F, _P, _I, _I, _P],
    "asdsl_b200_exact_numerics_init": [_P],
    "asdsl_b200_exact_host_tables": [_P, _P, _P, _I, _P],
    "asdsl_b200_exact_expf": [_P, _P, ctypes.c_longlong, _P],
    "asdsl_b200_xchg_create": [_I, _I, _P, _P],
    "asdsl_b200_xchg_handle_bytes": [],
    "asdsl_b200_xchg_open": [_P, _P],
    "asdsl_b200_xchg_destroy": [_P],
    "asdsl_b200_gemv_argmax_xchg": [_I, _P, _P, _P, _P, _P, _P, _I, _P, _SZ, _I, _I, _P, _P],
    "asdsl_b200_vxchg_create": [_I, _I, _I, _P, _P],
    "asdsl_b200_vxchg_handle_bytes": [],
    "asdsl_b200_vxchg_open": [_P, _P],
    "asdsl_b200_vxchg_destroy": [_P],
    "asdsl_b200_vxchg_set_stamps": [_P, _P, _I],
    "asdsl_b200_engine_set_shard": [_P, _P, _P, _I, _I],
    "asdsl_b200_gemv_q2_packed": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_engine_set_skip_mask": [_P, _P, _I],
    "asdsl_b200_engine_clear_skip_mask": [_P],
    "asdsl_b200_engine_set_projection_q2": [_P, _I, _I, _P, _SZ, _P, _P, _SZ],
    "asdsl_b200_engine_forward_token_draft": [_P, _I, _I, _P, _P, _I],
    "asdsl_b200_gemv_q2_unpacked": [_P, _P, _P, _P, _P, _I, _I, _I, _P],
    "asdsl_b200_xchg_set_stamps": [_P, _P, _I],
    "asdsl_b200_allreduce_peer": [_P, _P, _P, _P, _I, _P],
    # device-resident decode engine
    "asdsl_b200_engine_create": [_P, _P],
    "asdsl_b200_engine_destroy": [_P],
    "asdsl_b200_engine_set_globals": [_P, _P, _I, _P, _P, _P],
    "asdsl_b200_engine_set_output_proj": [_P, _P, _I],
    "asdsl_b200_engine_set_lm_head_preq2": [_P, _P, _SZ, _P, _SZ],
    "asdsl_b200_engine_set_layer_norms": [_P, _I, _P, _P],
    "asdsl_b200_engine_set_projection": [_P, _I, _I, _I, _P, _SZ, _P, _SZ],
    "asdsl_b200_engine_finalize": [_P],
    "asdsl_b200_engine_forward_token": [_P, _I, _I, _P, _P],
    "asdsl_b200_engine_forward_verify": [_P, _P, _I, _I, _P],
    "asdsl_b200_engine_forward_batch": [_P, _P, _I, _I, _P, _I],
    "asdsl_b200_gemm_q4_128_f32": [_P, _P, _P, _I, _I, _I, _I, _P],
    "asdsl_b200_engine_generate": [_P, _P, _I, _I, _P, _I, _P, _I, _P],
    "asdsl_b200_engine_reset_session": [_P],
    "asdsl_b200_engine_get_kv_seq_len": [_P, _P],
    "asdsl_b200_engine_truncate_kv": [_P, _I],
    "asdsl_b200_engine_snapshot_kv": [_P],
    "asdsl_b200_engine_restore_kv": [_P],
    "asdsl_b200_engine_export_lm_head": [_P, _P, _P, _SZ, _P, _SZ],
    "asdsl_b200_engine_stream": [_P, _P],
    "asdsl_b200_engine_set_persistent": [_P, _I],
    "asdsl_b200_engine_set_numerics": [_P, _I],
    "asdsl_b200_engine_profile_step": [_P, _I, _P, _I, _P],
    "asdsl_b200_engine_set_position": [_P, _I, _I],
    "asdsl_b200_engine_replay": [_P, _I, _I],
    "asdsl_b200_engine_read_buffer": [_P, _I, _P, _SZ],
}


class EngineConfigC(ctypes.Structure):
    """asdsl_b200_engine_config (include/asdsl_b200.h)."""

    _fields_ = [
        ("num_layers", _I), ("hidden_size", _I), ("num_heads", _I), ("num_kv_heads", _I), ("head_dim", _I),
        ("intermediate_size", _I), ("vocab_size", _I), ("rms_norm_eps", _F), ("group_size", _I),
        ("lm_head_group_size", _I), ("max_seq_len", _I), ("rotary_dim", _I), ("weight_format", _I),
    ]
_RESTYPES = {
    "asdsl_b200_version": ctypes.c_char_p,
    "asdsl_b200_timeline_bytes": _SZ,
    "asdsl_b200_last_error": ctypes.c_char_p,
    "asdsl_b200_argmax_scratch_bytes": _SZ,
    "asdsl_b200_xchg_handle_bytes": _SZ,
    "asdsl_b200_vxchg_handle_bytes": _SZ,
}

_lib = None
_lock = threading.Lock()


def exported_symbols() -> list[str]:
    """Every symbol the C ABI header declares (used by the load test)."""
    return list(_SIGS) + list(EXTRA_SIGS)


# entry points registered by other modules (engine, sharding) before load()
EXTRA_SIGS: dict[str, tuple[list, object]] = {}


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libasdsl_b200.so once and type every exported symbol."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"asdsl_b200 native library not built ({p} missing); run __graft_entry__.build()"
            )
        lib = ctypes.CDLL(p)
        for name, argtypes in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, _I)
        for name, (argtypes, restype) in EXTRA_SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().asdsl_b200_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str = "") -> None:
    """Raise the exception class the reference would raise for this status."""
    if rc == OK:
        return
    msg = last_error() or what
    if rc == EINVAL:
        raise ValueError(msg)
    if rc == ERANGE:
        raise IndexError(msg)
    if rc == ETIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> int:
    rc = getattr(load(), name)(*args)
    check(rc, name)
    return rc


def device_status(clear: bool = True) -> int:
    """Status bits set by kernels whose bounded waits gave up (0 = healthy)."""
    v = ctypes.c_uint(0)
    check(load().asdsl_b200_device_status(ctypes.byref(v), 1 if clear else 0))
    return int(v.value)
