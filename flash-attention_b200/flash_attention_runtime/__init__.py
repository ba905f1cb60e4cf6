"""flash_attention_runtime - drop-in for wenssir/flash-attention's Python entry points.

Same module name and call shapes as the reference
(python/flash_attention_runtime/__init__.py:30-38):

    forward(q, k, v, o=None)            -> o
    forward_timed(q, k, v, o=None)      -> (o, ms)

extended with keyword-only ``softmax_scale`` (default 1/sqrt(d), as the
reference hard-codes at python/flash_attention_runtime/_ext.cu:93), ``causal``
(default False, the reference's only mode, _ext.cu:94) and ``return_lse``
(default False; with it the result is ``(o, lse)``).  The extension-level call
``ext_forward(q, k, v, o=None, benchmark=False, ...)`` keeps the pybind function's
positional order and ``(o, ms)`` return (_ext.cu:124-173).

Accepted inputs: CUDA tensors of float16 or bfloat16, shape [B, H, N, d] with
d in {32, 64, 128}, any N >= 1, the last dimension contiguous and the other
strides multiples of 8 elements (the reference required contiguous fp16, d=128
and N % 64 == 0).  Violations raise RuntimeError naming the constraint, as the
reference's TORCH_CHECKs do (_ext.cu:19-57).

PyTorch appears only here, at the binding: tensors are handed to the C ABI
(include/fa_sm100.h) as raw device pointers and strides, and the kernel runs on
the current CUDA stream of the tensors' device.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib

__all__ = ["forward", "forward_timed", "ext_forward", "device_status", "reset_device_status", "smem_bytes"]

_DTYPES = {torch.float16: _lib.FA_DTYPE_F16, torch.bfloat16: _lib.FA_DTYPE_BF16}
_STATUS: dict[int, torch.Tensor] = {}


def _status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def device_status(device: Optional[torch.device] = None) -> int:
    """Status word the kernel sets when one of its pipeline waits times out (0 = none).

    Reading it synchronises the device's current stream.
    """
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return int(_status_word(device).item())


def reset_device_status(device: Optional[torch.device] = None) -> None:
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _status_word(device).zero_()


def smem_bytes(head_dim: int, dtype: torch.dtype) -> int:
    """Dynamic shared memory per CTA (the reference's forward_smem_bytes<Cfg>())."""
    if dtype not in _DTYPES:
        return 0
    return int(_lib.load().fa_fwd_smem_bytes(int(head_dim), _DTYPES[dtype]))


def _check_tensor(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype not in _DTYPES:
        raise RuntimeError(f"{name} must be float16 or bfloat16 (got {t.dtype})")
    if t.dim() != 4:
        raise RuntimeError(f"{name} must be a 4D tensor with shape [B, H, N, D]")
    if t.stride(3) != 1:
        raise RuntimeError(f"{name} must have a contiguous last (head) dimension")


def _validate(q, k, v, o) -> None:
    _check_tensor(q, "q")
    _check_tensor(k, "k")
    _check_tensor(v, "v")
    if q.shape != k.shape:
        raise RuntimeError("q and k must have the same shape")
    if q.shape != v.shape:
        raise RuntimeError("q and v must have the same shape")
    if q.dtype != k.dtype:
        raise RuntimeError("q and k must have the same dtype")
    if q.dtype != v.dtype:
        raise RuntimeError("q and v must have the same dtype")
    if k.device != q.device or v.device != q.device:
        raise RuntimeError("q, k and v must be on the same device")
    if q.shape[3] not in (32, 64, 128):
        raise RuntimeError(f"head_dim must be 32, 64 or 128 (got {q.shape[3]})")
    if o is not None:
        _check_tensor(o, "o")
        if o.shape != q.shape:
            raise RuntimeError("o must have the same shape as q")
        if o.dtype != q.dtype:
            raise RuntimeError("o must have the same dtype as q")
        if o.device != q.device:
            raise RuntimeError("o must be on the same device as q")


def _launch(q, k, v, o, lse, softmax_scale: float, causal: bool) -> None:
    lib = _lib.load()
    p = _lib.FwdParams()
    p.Q, p.K, p.V, p.O = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
        setattr(p, f"stride_batch_{name}", 0)
        setattr(p, f"stride_seq_{name}", int(t.stride(2)))
        setattr(p, f"stride_head_{name}", 0)
    p.stride_batch64 = (ctypes.c_int64 * 4)(*[int(t.stride(0)) for t in (q, k, v, o)])
    p.stride_head64 = (ctypes.c_int64 * 4)(*[int(t.stride(1)) for t in (q, k, v, o)])
    b, h, n, d = q.shape
    p.batch, p.heads, p.seq_len, p.head_dim = int(b), int(h), int(n), int(d)
    p.softmax_scale = float(softmax_scale)
    p.causal = 1 if causal else 0
    p.LSE = lse.data_ptr() if lse is not None else None
    p.dtype = _DTYPES[q.dtype]
    p.workspace = None
    p.workspace_bytes = 0
    p.status = _status_word(q.device).data_ptr()
    p.timeout_ns = 0
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = lib.fa_fwd_sm100(ctypes.byref(p), ctypes.c_void_p(stream))
    if rc != _lib.FA_OK:
        raise RuntimeError(f"fa_fwd_sm100 failed: {_lib.status_message(lib, rc)}")


def ext_forward(q, k, v, o=None, benchmark: bool = False, softmax_scale=None, causal: bool = False, lse=None):
    """Extension-level call with the reference pybind signature (_ext.cu:162-172).

    Returns ``(o, ms)``; ``ms`` is 0.0 unless ``benchmark`` is True, in which case
    the launch is bracketed by CUDA events on the current stream and the call
    synchronises (like the reference, _ext.cu:136-155).  ``lse``, when given, is
    an fp32 [B, H, N] contiguous CUDA tensor that receives the logsumexp.
    """
    _validate(q, k, v, o)
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[3])
    if lse is not None:
        if not (lse.is_cuda and lse.dtype == torch.float32 and lse.is_contiguous()
                and tuple(lse.shape) == tuple(q.shape[:3]) and lse.device == q.device):
            raise RuntimeError("lse must be a contiguous float32 CUDA tensor of shape [B, H, N] on q's device")
    if o is None:
        o = torch.empty_like(q)
    ms = 0.0
    with torch.cuda.device(q.device):
        if benchmark:
            stream = torch.cuda.current_stream(q.device)
            start = torch.cuda.Event(enable_timing=True)
            stop = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            _launch(q, k, v, o, lse, softmax_scale, causal)
            stop.record(stream)
            stop.synchronize()
            ms = float(start.elapsed_time(stop))
            st = device_status(q.device)
            if st != 0:
                raise RuntimeError(f"fa_fwd_sm100 kernel reported status 0x{st:x} (pipeline wait timed out)")
        else:
            _launch(q, k, v, o, lse, softmax_scale, causal)
    return o, ms


def forward(q, k, v, o=None, *, softmax_scale=None, causal: bool = False, return_lse: bool = False):
    """O = softmax(softmax_scale * Q K^T [+ causal mask]) V, asynchronously on the current stream."""
    _validate(q, k, v, o)
    lse = torch.empty(tuple(q.shape[:3]), dtype=torch.float32, device=q.device) if return_lse else None
    out, _ = ext_forward(q, k, v, o, False, softmax_scale, causal, lse)
    return (out, lse) if return_lse else out


def forward_timed(q, k, v, o=None, *, softmax_scale=None, causal: bool = False, return_lse: bool = False):
    """Like forward(), but synchronises and also returns the kernel time in ms."""
    _validate(q, k, v, o)
    lse = torch.empty(tuple(q.shape[:3]), dtype=torch.float32, device=q.device) if return_lse else None
    out, ms = ext_forward(q, k, v, o, True, softmax_scale, causal, lse)
    return ((out, lse) if return_lse else out), ms
