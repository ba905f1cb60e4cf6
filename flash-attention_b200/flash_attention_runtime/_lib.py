"""ctypes binding of the C ABI declared in include/fa_sm100.h.

The shared library is built in-tree (flash-attention_b200/csrc/libfa_sm100.so);
there is no fallback: if it is missing, loading raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = _PKG_ROOT / "csrc" / "libfa_sm100.so"

FA_OK = 0
FA_ERR_BAD_SHAPE = 1
FA_ERR_BAD_ALIGN = 2
FA_ERR_UNSUPPORTED = 3
FA_ERR_LAUNCH = 4
FA_ERR_DEVICE_TIMEOUT = 5
FA_ERR_BAD_PARAM = 6

FA_DTYPE_F16 = 0
FA_DTYPE_BF16 = 1

# Every symbol include/fa_sm100.h declares.
EXPORTED_SYMBOLS = (
    "fa_fwd_sm100",
    "fa_fwd_smem_bytes",
    "fa_fwd_workspace_bytes",
    "fa_status_string",
    "fa_last_error",
)


class FwdParams(ctypes.Structure):
    """Mirror of ``fa_fwd_params``: ForwardKernelArgs fields first, then the appended ones."""

    _fields_ = [
        ("Q", ctypes.c_void_p),
        ("K", ctypes.c_void_p),
        ("V", ctypes.c_void_p),
        ("O", ctypes.c_void_p),
        ("stride_batch_q", ctypes.c_int),
        ("stride_seq_q", ctypes.c_int),
        ("stride_head_q", ctypes.c_int),
        ("stride_batch_k", ctypes.c_int),
        ("stride_seq_k", ctypes.c_int),
        ("stride_head_k", ctypes.c_int),
        ("stride_batch_v", ctypes.c_int),
        ("stride_seq_v", ctypes.c_int),
        ("stride_head_v", ctypes.c_int),
        ("stride_batch_o", ctypes.c_int),
        ("stride_seq_o", ctypes.c_int),
        ("stride_head_o", ctypes.c_int),
        ("seq_len", ctypes.c_int),
        ("heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("softmax_scale", ctypes.c_float),
        ("causal", ctypes.c_int),
        ("LSE", ctypes.c_void_p),
        ("dtype", ctypes.c_int),
        ("batch", ctypes.c_int),
        ("stride_batch64", ctypes.c_int64 * 4),
        ("stride_head64", ctypes.c_int64 * 4),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_ulonglong),
    ]


_LIB = None


def load() -> ctypes.CDLL:
    """Load libfa_sm100.so once; raise if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `make -C flash-attention_b200/csrc` "
            "(or __graft_entry__.build()); there is no non-CUDA fallback"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.fa_fwd_sm100.argtypes = [ctypes.POINTER(FwdParams), ctypes.c_void_p]
    lib.fa_fwd_sm100.restype = ctypes.c_int
    lib.fa_fwd_smem_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
    lib.fa_fwd_smem_bytes.restype = ctypes.c_size_t
    lib.fa_fwd_workspace_bytes.argtypes = []
    lib.fa_fwd_workspace_bytes.restype = ctypes.c_size_t
    lib.fa_status_string.argtypes = [ctypes.c_int]
    lib.fa_status_string.restype = ctypes.c_char_p
    lib.fa_last_error.argtypes = []
    lib.fa_last_error.restype = ctypes.c_char_p
    _LIB = lib
    return lib


def status_message(lib: ctypes.CDLL, status: int) -> str:
    name = lib.fa_status_string(status).decode()
    detail = lib.fa_last_error().decode()
    return f"{name}: {detail}" if detail else name
