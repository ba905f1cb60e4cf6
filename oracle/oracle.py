"""TEST INFRASTRUCTURE ONLY - ctypes loaders for the CPU parity oracle.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this
module.  The product path (``flash_attention_runtime``) never does.

* ``oracle_attention``   - liboracle.so, the C++ restatement of the reference's
  ``cpu_reference_attention`` (benchmark/cpp/correctness_v6.cu:23-72) plus LSE.
* ``ref_attention``      - oracle/_ref/libref_attention.so, the reference's own
  function compiled from its source tree (present when the reference was
  available at build time; it travels with the repository snapshot).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libref_attention.so"

_f32p = ctypes.POINTER(ctypes.c_float)


def build() -> None:
    """Compile liboracle.so (and _ref/ when the reference tree exists)."""
    subprocess.run(["make", "-C", str(HERE), "-s"], check=True)


def _load(path: Path) -> ctypes.CDLL:
    if not path.exists():
        raise FileNotFoundError(f"{path} is not built (run oracle/Makefile)")
    return ctypes.CDLL(str(path))


_ORACLE = None
_REF = None


def _oracle_lib() -> ctypes.CDLL:
    global _ORACLE
    if _ORACLE is None:
        lib = _load(ORACLE_SO)
        lib.oracle_attention_slices.argtypes = [_f32p] * 5 + [ctypes.c_int] * 4 + [ctypes.c_float] + [ctypes.c_int] * 2
        lib.oracle_attention_slices.restype = None
        _ORACLE = lib
    return _ORACLE


def ref_available() -> bool:
    return REF_SO.exists()


def _ref_lib() -> ctypes.CDLL:
    global _REF
    if _REF is None:
        lib = _load(REF_SO)
        lib.ref_cpu_reference_attention.argtypes = [_f32p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_int]
        lib.ref_cpu_reference_attention.restype = None
        lib.ref_cpu_attention_slices.argtypes = [_f32p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_float] + [ctypes.c_int] * 2
        lib.ref_cpu_attention_slices.restype = None
        _REF = lib
    return _REF


def _f32(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def oracle_attention(q, k, v, scale: float, causal: bool, threads: int = 0, slices=None):
    """O (fp32 [B,H,N,D]) and LSE (fp32 [B,H,N]) of the restated oracle.

    ``slices=(begin, end)`` restricts the work to flattened (b,h) slices
    [begin, end); the other slices of O/LSE stay NaN.
    """
    q, k, v = _f32(q), _f32(k), _f32(v)
    b, h, n, d = q.shape
    o = np.full(q.shape, np.nan, dtype=np.float32)
    lse = np.full((b, h, n), np.nan, dtype=np.float32)
    s0, s1 = slices if slices is not None else (0, b * h)
    _oracle_lib().oracle_attention_slices(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), s0, s1, n, d,
                                          float(scale), int(bool(causal)), int(threads))
    return o, lse


def ref_attention(q, k, v, scale: float, causal: bool, threads: int = 0, slices=None):
    """O (fp32 [B,H,N,D]) of the reference's own cpu_reference_attention."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    b, h, n, d = q.shape
    o = np.full(q.shape, np.nan, dtype=np.float32)
    s0, s1 = slices if slices is not None else (0, b * h)
    _ref_lib().ref_cpu_attention_slices(_ptr(q), _ptr(k), _ptr(v), _ptr(o), s0, s1, n, d, float(scale),
                                        int(bool(causal)), int(threads))
    return o


def ref_attention_direct(q, k, v, scale: float, causal: bool):
    """The reference function called once over all of [B,H,N,D] (single thread)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    b, h, n, d = q.shape
    o = np.zeros(q.shape, dtype=np.float32)
    _ref_lib().ref_cpu_reference_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(o), b, h, n, d, float(scale),
                                           int(bool(causal)))
    return o


REF_EXT_SO = HERE / "_ref" / "ext" / "fa_ref_v6.so"


def ref_gpu_available() -> bool:
    return REF_EXT_SO.exists()


def ref_gpu_module():
    """The reference's own pybind module (python/flash_attention_runtime/_ext.cu,
    kernel flash_attention_forward_v6_mma), as built by oracle/build_ref_ext.py.
    Its ``forward(q, k, v, o, benchmark)`` returns ``(o, ms)``; fp16, d = 128,
    non-causal, N % 64 == 0 only."""
    import importlib.util

    import torch  # noqa: F401  (the module links against libtorch)

    if not REF_EXT_SO.exists():
        raise RuntimeError(f"{REF_EXT_SO} is missing: run `python oracle/build_ref_ext.py`")
    spec = importlib.util.spec_from_file_location("fa_ref_v6", str(REF_EXT_SO))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
