"""Host tables of the reference-exact numerics mode (asdsl_b200_exact_host_tables; CPU only).

The reference's compiled engine uses RSQRTSS / RCPPS estimates (Newton-refined) and the C
library's expf (asdsl/kernels/native/unified_engine.cpp:499-524, :836-857, :922-1027).  The
library captures them from the host as tables the GPU evaluates; these tests check the table
model against the host instructions (through the oracle) on random inputs of every exponent, and
the expf exception list against the C library."""

import ctypes

import numpy as np
import pytest


@pytest.fixture(scope="module")
def tables():
    from asdsl_b200 import _lib
    from asdsl_b200.build import build_library

    build_library()
    lib = _lib.load()
    rcp = np.zeros(2048, np.uint32)
    rsq = np.zeros(2048, np.uint32)
    n = ctypes.c_int(0)
    _lib.check(lib.asdsl_b200_exact_host_tables(rcp.ctypes.data, rsq.ctypes.data, None, 0, ctypes.byref(n)),
               "exact_host_tables")
    exc = np.zeros(2 * n.value, np.uint32)
    _lib.check(lib.asdsl_b200_exact_host_tables(None, None, exc.ctypes.data, n.value, ctypes.byref(n)),
               "exact_host_tables")
    return rcp, rsq, exc.reshape(-1, 2)


def _emu_rcp(x, tab):
    """exact_math.cuh emu_rcp_bits, vectorized (normal inputs)."""
    x = x.astype(np.uint32)
    sign = x & np.uint32(0x80000000)
    e = ((x >> 23) & 0xFF).astype(np.int64)
    t = tab[(x >> 12) & 0x7FF]
    re = ((t >> 23) & 0xFF).astype(np.int64) - (e - 127)
    out = sign | (np.clip(re, 0, 255).astype(np.uint32) << 23) | (t & np.uint32(0x7FFFFF))
    return np.where(re <= 0, sign, np.where(re >= 255, sign | np.uint32(0x7F800000), out))


def _emu_rsqrt(x, tab):
    x = x.astype(np.uint32)
    e = ((x >> 23) & 0xFF).astype(np.int64)
    par = (e - 127) & 1
    k = (e - 127 - par) // 2
    t = tab[par * 1024 + ((x >> 13) & 0x3FF)]
    re = ((t >> 23) & 0xFF).astype(np.int64) - k
    return (re.astype(np.uint32) << 23) | (t & np.uint32(0x7FFFFF))


def test_rcp_rsqrt_table_model_matches_host_instructions(tables, oracle):
    rcp, rsq, _ = tables
    rng = np.random.default_rng(0)
    e = rng.integers(1, 255, 4000).astype(np.uint32)
    m = rng.integers(0, 1 << 23, 4000).astype(np.uint32)
    xs = (e << 23) | m
    got_r = _emu_rcp(xs, rcp)
    got_s = _emu_rsqrt(xs, rsq)
    for i, xb in enumerate(xs):
        x = float(np.uint32(xb).view(np.float32))
        assert np.float32(oracle.host_rcp(x)).view(np.uint32) == got_r[i], hex(xb)
        assert np.float32(oracle.host_rsqrt(x)).view(np.uint32) == got_s[i], hex(xb)


def test_expf_exceptions_match_c_library(tables, oracle):
    _, _, exc = tables
    keys = exc[:, 0]
    assert len(keys) > 1000 and np.all(np.diff(keys.astype(np.int64)) > 0), "keys must be ascending"
    assert np.all(keys >= 0x80000000), "the attention only evaluates expf on x <= 0"
    rng = np.random.default_rng(1)
    pick = exc[rng.choice(len(exc), 4000, replace=False)]
    x = pick[:, 0].view(np.float32).copy()
    y = oracle.expf_array(x)
    assert np.array_equal(y.view(np.uint32), pick[:, 1])
    # away from the listed inputs, expf is exp in double rounded to float
    xr = -rng.uniform(0, 104, 300000).astype(np.float32)
    xr = xr[~np.isin(xr.view(np.uint32), keys)]
    yr = oracle.expf_array(xr)
    libm = ctypes.CDLL("libm.so.6")
    libm.exp.restype = ctypes.c_double
    libm.exp.argtypes = [ctypes.c_double]
    ref = np.array([libm.exp(float(v)) for v in xr[:20000]]).astype(np.float32)
    assert np.array_equal(yr[:20000].view(np.uint32), ref.view(np.uint32))
