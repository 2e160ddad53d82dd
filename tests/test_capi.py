"""The C ABI library: it loads, exports every symbol include/asdsl_b200.h declares,
and rejects bad arguments with the reference's exception classes -- all without a
GPU (no compute call is made).  CPU only."""

import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"\b(asdsl_b200_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from asdsl_b200 import _lib
    from asdsl_b200.build import build_library

    build_library()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    from asdsl_b200 import _lib

    declared = _declared_symbols()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared but not exported"
    # and the Python binding types every one of them
    assert set(declared) <= set(_lib.exported_symbols())


def test_version_and_scratch(lib):
    assert b"sm_100a" in lib.asdsl_b200_version()
    assert lib.asdsl_b200_argmax_scratch_bytes() >= 256


def test_argument_errors_map_to_reference_exceptions(lib):
    from asdsl_b200 import _lib

    # null pointers / bad group sizes are rejected on the host before any CUDA call
    with pytest.raises(ValueError, match="null pointer"):
        _lib.call("asdsl_b200_gemv_preq2_fused", None, None, None, None, 16, 64, 32, None)
    with pytest.raises(ValueError, match="group_size must be 32"):
        _lib.call("asdsl_b200_gemv_preq2_fused", 16, 16, 16, 16, 16, 64, 64, None)
    with pytest.raises(ValueError, match="group_size must be 128"):
        _lib.call("asdsl_b200_gemv_q4_128", 16, 16, 16, 16, 16, 256, 32, None)
    with pytest.raises(ValueError, match="divisible by 256"):
        _lib.call("asdsl_b200_gemv_q4km", 16, 16, 16, 4, 100, None)
    with pytest.raises(ValueError, match="n_groups exceeds buffer"):
        _lib.call("asdsl_b200_gemv_q4_32_preq", 16, 16, 16, 16, 4, 32 * 641, 32, None)
    with pytest.raises(ValueError, match="multiple of 8"):
        _lib.call("asdsl_b200_gemv_q4_packed", 16, 16, 16, 16, 16, 4, 36, 12, 1, None)
    # Q4_K with empty shapes returns without work, like the reference
    assert _lib.call("asdsl_b200_gemv_q4km", None, None, None, 0, 256, None) == 0
    # prompt GEMM (gemm_q4_128_q8_avx2): the reference's group-size message first, then this
    # library's own checks; an empty batch is no work
    with pytest.raises(ValueError, match="gemm_q4_128_q8_avx2: group_size must be 128"):
        _lib.call("asdsl_b200_gemm_q4_128_f32", 16, 16, 16, 16, 128, 32, 4, None)
    with pytest.raises(ValueError, match="null pointer"):
        _lib.call("asdsl_b200_gemm_q4_128_f32", None, 16, 16, 16, 128, 128, 4, None)
    with pytest.raises(ValueError, match="divisible by 128"):
        _lib.call("asdsl_b200_gemm_q4_128_f32", 16, 16, 16, 16, 100, 128, 4, None)
    with pytest.raises(ValueError, match="2-byte aligned"):
        _lib.call("asdsl_b200_gemm_q4_128_f32", 17, 16, 16, 16, 128, 128, 4, None)
    with pytest.raises(ValueError, match="16-byte aligned"):
        _lib.call("asdsl_b200_gemm_q4_128_f32", 16, 20, 16, 16, 128, 128, 4, None)
    assert _lib.call("asdsl_b200_gemm_q4_128_f32", 16, 16, 16, 16, 128, 128, 0, None) == 0
    # the cross-GPU argmax packs a 24-bit global row index: a negative row base is rejected
    with pytest.raises(ValueError, match="row_base must be >= 0"):
        _lib.call("asdsl_b200_gemv_argmax_xchg", 0, 16, 16, 16, 16, 16, 16, -4, 16, 1 << 16, 8, 64, None, None)
    # reference-exact entries: the same host-side checks
    with pytest.raises(ValueError, match="null pointer"):
        _lib.call("asdsl_b200_gemv_preq2_fused_exact", None, None, None, None, 0.0, None, 16, 64, None)
    with pytest.raises(ValueError, match="positive multiple of 4"):
        _lib.call("asdsl_b200_gateup_silu_exact", 16, 16, 16, None, 0.0, 16, 6, 64, None)
    # the layer step and the zero-copy transfers: argument checks before any CUDA call
    import ctypes

    h = ctypes.c_void_p()
    with pytest.raises(ValueError, match="layer_create: null pointer"):
        _lib.call("asdsl_b200_layer_create", *([None] * 11), 3072, 5120, 3072, 8192, ctypes.byref(h))
    with pytest.raises(ValueError, match="layer_create: invalid dimensions"):
        _lib.call("asdsl_b200_layer_create", *([16] * 11), 3072, 5120, 6144, 8192, ctypes.byref(h))
    with pytest.raises(ValueError, match="layer_forward: null pointer"):
        _lib.call("asdsl_b200_layer_forward", None, None, None)
    assert _lib.call("asdsl_b200_layer_destroy", None) == 0
    with pytest.raises(ValueError, match="host_to_device: invalid arguments"):
        _lib.call("asdsl_b200_host_to_device", None, 16, 4, None)
    with pytest.raises(ValueError, match="device_to_host: invalid arguments"):
        _lib.call("asdsl_b200_device_to_host", 16, 16, -1, None)
    assert _lib.call("asdsl_b200_host_to_device", 16, 16, 0, None) == 0
    with pytest.raises(ValueError, match="16-byte aligned"):
        _lib.call("asdsl_b200_layer_create", *([16] * 8), 20, 16, 16, 3072, 5120, 3072, 8192, ctypes.byref(h))


def test_python_api_fails_loudly_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from asdsl_b200.kernels import gemv_q4_packed, has_native_kernel

    assert not has_native_kernel()
    with pytest.raises(RuntimeError):
        gemv_q4_packed(np.zeros(32, np.uint8), np.zeros(64, np.float32), np.ones(2, np.float32),
                       np.zeros(2, np.float32), 1, 64, 32)
