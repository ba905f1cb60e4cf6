"""Property test of fa_fwd_sm100's argument validation (CPU only).

fa_fwd_sm100 must reject every bad fa_fwd_params with a status code before it
touches a GPU, and name the problem in fa_last_error().  Here hypothesis draws
parameter sets around every boundary the validation has; a Python statement of
the rules, in the library's order, gives the expected code.  A call that passes
every rule returns FA_ERR_UNSUPPORTED, because this machine has no CUDA device.

The pointers are made up, so the test runs only where no GPU is present: on a
GPU a valid parameter set would launch the kernel on them.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from flash_attention_runtime import _lib

pytestmark = pytest.mark.skipif(torch.cuda.is_available(), reason="passes made-up pointers; no-GPU machines only")

MAX_STRIDE = 1 << 39  # elements: 2^40 bytes, the TMA stride limit
MAX_EXTENT = 1 << 47  # elements: 2^48 bytes
INT32_MAX = (1 << 31) - 1

OK_PTRS = [0x10000, 0x7F0000000000, 0x123450]
BAD_PTRS = [0x10008, 0x10001, 0x7F0000000004]


def expected(f: dict) -> int:
    """The library's rules in its order (csrc/fa_sm100.cu, validate())."""
    if not all(f[t] for t in ("Q", "K", "V", "O")):
        return _lib.FA_ERR_BAD_PARAM
    if f["dtype"] not in (0, 1):
        return _lib.FA_ERR_UNSUPPORTED
    d = f["head_dim"]
    if d not in (32, 64, 128):
        return _lib.FA_ERR_UNSUPPORTED
    b, h, n = f["batch"], f["heads"], f["seq_len"]
    if b < 1 or h < 1 or n < 1:
        return _lib.FA_ERR_BAD_SHAPE
    with np.errstate(over="ignore"):  # a double past the float range becomes inf, as in C
        scale = float(np.float32(f["scale"]))
    if not (math.isfinite(scale) and scale > 0):
        return _lib.FA_ERR_BAD_PARAM
    if f["causal"] not in (0, 1):
        return _lib.FA_ERR_BAD_PARAM
    for t in ("Q", "K", "V", "O"):
        if f[t] & 15:
            return _lib.FA_ERR_BAD_ALIGN
        ss = f[f"ss_{t}"]
        hs = f[f"hs64_{t}"] or f[f"hs_{t}"]
        bs = f[f"bs64_{t}"] or f[f"bs_{t}"]
        if ss < d:
            return _lib.FA_ERR_BAD_SHAPE
        if (h > 1 and hs < 1) or (b > 1 and bs < 1):
            return _lib.FA_ERR_BAD_SHAPE
        used = [ss, hs if h > 1 else 8, bs if b > 1 else 8]
        if any(x % 8 for x in used):
            return _lib.FA_ERR_BAD_ALIGN
        if any(x >= MAX_STRIDE for x in used):
            return _lib.FA_ERR_BAD_SHAPE
        extent = (b - 1) * (bs if b > 1 else 0) + (h - 1) * (hs if h > 1 else 0) + (n - 1) * ss + d
        if extent > MAX_EXTENT:
            return _lib.FA_ERR_BAD_SHAPE
    if f["LSE"] & 3:
        return _lib.FA_ERR_BAD_ALIGN
    return _lib.FA_ERR_UNSUPPORTED  # every rule passed; no CUDA device here


def _params(f: dict) -> _lib.FwdParams:
    p = _lib.FwdParams()
    for t in ("Q", "K", "V", "O"):
        setattr(p, t, f[t] or None)
        low = t.lower()
        setattr(p, f"stride_seq_{low}", f[f"ss_{t}"])
        setattr(p, f"stride_head_{low}", f[f"hs_{t}"])
        setattr(p, f"stride_batch_{low}", f[f"bs_{t}"])
    p.stride_head64 = (ctypes.c_int64 * 4)(*[f[f"hs64_{t}"] for t in "QKVO"])
    p.stride_batch64 = (ctypes.c_int64 * 4)(*[f[f"bs64_{t}"] for t in "QKVO"])
    p.batch, p.heads, p.seq_len, p.head_dim = f["batch"], f["heads"], f["seq_len"], f["head_dim"]
    p.softmax_scale = f["scale"]
    p.causal = f["causal"]
    p.dtype = f["dtype"]
    p.LSE = f["LSE"] or None
    return p


def _int32(*special):
    return st.one_of(st.sampled_from([-8, -1, 0, 1, 7, 8, 16, 64, 128, 256, 4096, INT32_MAX, -INT32_MAX - 1,
                                      *special]),
                     st.integers(-INT32_MAX - 1, INT32_MAX),
                     st.integers(0, 1 << 20).map(lambda x: 8 * x))


def _int64(*special):
    return st.one_of(st.just(0), st.just(0), st.sampled_from([8, -8, 4, MAX_STRIDE - 8, MAX_STRIDE, MAX_STRIDE + 8,
                                                              (1 << 31) + 1024, 1 << 62, -(1 << 62), *special]),
                     st.integers(-(1 << 63), (1 << 63) - 1), st.integers(1, 1 << 36).map(lambda x: 8 * x))


def _fields():
    ptr = st.sampled_from(OK_PTRS * 4 + BAD_PTRS + [0])
    tensor = {}
    for t in ("Q", "K", "V", "O"):
        tensor[t] = ptr
        tensor[f"ss_{t}"] = _int32(32, 64, 128, 136)
        tensor[f"hs_{t}"] = _int32(1 << 20, 64 * 1024)
        tensor[f"bs_{t}"] = _int32(1 << 24)
        tensor[f"hs64_{t}"] = _int64()
        tensor[f"bs64_{t}"] = _int64()
    small = st.one_of(st.sampled_from([-1, 0, 1, 2, 3, 128, 129, 4096]), st.integers(-4, 1 << 16),
                      st.sampled_from([1 << 20, INT32_MAX]))
    return st.fixed_dictionaries({
        **tensor,
        "dtype": st.sampled_from([0, 1, 0, 1, 2, -1]),
        "head_dim": st.sampled_from([32, 64, 128, 32, 64, 128, 0, 16, 96, 256, -64]),
        "batch": small, "heads": small, "seq_len": small,
        "scale": st.one_of(st.sampled_from([0.125, 1.0, 0.0, -0.5, math.nan, math.inf, -math.inf, 1e-40, 1e39]),
                           st.floats(allow_nan=True, allow_infinity=True)),
        "causal": st.sampled_from([0, 1, 0, 1, 2, -1]),
        "LSE": st.sampled_from([0, 0x80000, 0x80004, 0x80002, 0x80001]),
    })


@settings(max_examples=1500, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(_fields())
def test_validation_matches_the_rules(f):
    lib = _lib.load()
    want = expected(f)
    got = lib.fa_fwd_sm100(ctypes.byref(_params(f)), None)
    assert got == want, (got, want, lib.fa_last_error())
    msg = lib.fa_last_error()
    assert msg, "every rejection names its reason"
    if want == _lib.FA_ERR_UNSUPPORTED and f["dtype"] in (0, 1) and f["head_dim"] in (32, 64, 128):
        assert b"device" in msg


@settings(max_examples=300, deadline=None)
@given(_fields())
def test_noalloc_entry_point_validates_the_same_way(f):
    lib = _lib.load()
    lib.fa_fwd_sm100_noalloc.argtypes = [ctypes.POINTER(_lib.FwdParams), ctypes.c_void_p]
    lib.fa_fwd_sm100_noalloc.restype = ctypes.c_int
    assert lib.fa_fwd_sm100_noalloc(ctypes.byref(_params(f)), None) == expected(f)


def _valid():
    f = {"dtype": 1, "head_dim": 128, "batch": 2, "heads": 4, "seq_len": 1000, "scale": 0.088, "causal": 1,
         "LSE": 0x80000}
    for t in ("Q", "K", "V", "O"):
        f.update({t: 0x10000, f"ss_{t}": 128, f"hs_{t}": 128 * 1000, f"bs_{t}": 4 * 128 * 1000,
                  f"hs64_{t}": 0, f"bs64_{t}": 0})
    return f


@pytest.mark.parametrize("change,code,words", [
    ({"hs64_K": MAX_STRIDE}, _lib.FA_ERR_BAD_SHAPE, b"2^40"),
    ({"bs64_O": MAX_STRIDE - 8}, _lib.FA_ERR_UNSUPPORTED, b"device"),
    ({"batch": 1 << 20, "bs64_O": MAX_STRIDE - 8}, _lib.FA_ERR_BAD_SHAPE, b"2^48"),
    ({"heads": 1, "hs64_V": 1 << 62}, _lib.FA_ERR_UNSUPPORTED, b"device"),  # a size-1 dimension's stride is unused
    ({"batch": 1, "bs_Q": -8}, _lib.FA_ERR_UNSUPPORTED, b"device"),
    ({"heads": 2, "hs_Q": -8}, _lib.FA_ERR_BAD_SHAPE, b"positive"),
    ({"hs64_O": (1 << 31) + 1024}, _lib.FA_ERR_UNSUPPORTED, b"device"),  # past int32: the 64-bit fields carry it
])
def test_stride_and_extent_limits(change, code, words):
    f = {**_valid(), **change}
    assert expected(f) == code
    lib = _lib.load()
    assert lib.fa_fwd_sm100(ctypes.byref(_params(f)), None) == code
    assert words in lib.fa_last_error()
