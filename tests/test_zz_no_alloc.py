"""GPU test of fa_fwd_sm100_noalloc, the entry point for callers that cannot
allocate device memory: runtimes whose memory pool forbids allocations behind its
back, plug-in hosts that hand a library only its input and output buffers, and
latency-bound loops that cannot take a cudaMalloc's implicit synchronisation.

It runs the same computation as fa_fwd_sm100 but keeps the scheduler's scratch
in a fixed array inside the library instead of a cudaMalloc'd workspace.  The
test calls both entry points through the C ABI on the same inputs and requires
the no-alloc outputs to match within the parity tolerance of the other GPU tests,
on two calls in a row (the second call checks that the shared scratch is cleared
between launches).  This file is collected last, and it also passes when run
alone in a fresh process, where its first call is the one that looks up the
scratch address.
"""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

from parity import compare_lse, compare_output

from flash_attention_runtime import _lib
from flash_attention_runtime.inputs import make_random

pytestmark = pytest.mark.gpu

_DT = {torch.float16: _lib.FA_DTYPE_F16, torch.bfloat16: _lib.FA_DTYPE_BF16}


def _params(q, k, v, o, lse, scale, causal, status):
    p = _lib.FwdParams()
    p.Q, p.K, p.V, p.O = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
        setattr(p, f"stride_batch_{name}", int(t.stride(0)))
        setattr(p, f"stride_head_{name}", int(t.stride(1)))
        setattr(p, f"stride_seq_{name}", int(t.stride(2)))
    b, h, n, d = q.shape
    p.batch, p.heads, p.seq_len, p.head_dim = b, h, n, d
    p.softmax_scale = scale
    p.causal = int(causal)
    p.LSE = lse.data_ptr()
    p.dtype = _DT[q.dtype]
    p.workspace = None
    p.workspace_bytes = 0
    p.status = status.data_ptr()
    p.timeout_ns = 0
    return p


@pytest.mark.parametrize("shape,dtype,causal", [
    ((2, 4, 1000, 128), torch.bfloat16, True),
    ((1, 3, 512, 64), torch.float16, False),
])
def test_noalloc_entry_point_matches_default(shape, dtype, causal):
    lib = _lib.load()
    lib.fa_fwd_sm100_noalloc.argtypes = [ctypes.POINTER(_lib.FwdParams), ctypes.c_void_p]
    lib.fa_fwd_sm100_noalloc.restype = ctypes.c_int
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q, k, v = (t.to(dev) for t in make_random(shape, dtype, seed=77))
    scale = 1.0 / math.sqrt(shape[-1])
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

    o_ref = torch.empty_like(q)
    lse_ref = torch.empty(shape[:3], dtype=torch.float32, device=dev)
    p = _params(q, k, v, o_ref, lse_ref, scale, causal, status)
    assert lib.fa_fwd_sm100(ctypes.byref(p), stream) == _lib.FA_OK, lib.fa_last_error()

    for _ in range(2):
        o = torch.full_like(q, float("nan"))
        lse = torch.full(shape[:3], float("nan"), dtype=torch.float32, device=dev)
        p = _params(q, k, v, o, lse, scale, causal, status)
        rc = lib.fa_fwd_sm100_noalloc(ctypes.byref(p), stream)
        assert rc == _lib.FA_OK, lib.fa_last_error()
        torch.cuda.synchronize(dev)
        assert int(status.item()) == 0
        ro = compare_output(o, o_ref.float().cpu().numpy(), dtype)
        rl = compare_lse(lse, lse_ref.cpu().numpy())
        assert ro["ok"], ro
        assert rl["ok"], rl


def test_noalloc_rejects_a_workspace():
    lib = _lib.load()
    lib.fa_fwd_sm100_noalloc.argtypes = [ctypes.POINTER(_lib.FwdParams), ctypes.c_void_p]
    lib.fa_fwd_sm100_noalloc.restype = ctypes.c_int
    # Valid arguments on real device buffers, plus a caller workspace: the
    # workspace alone is the error, and nothing launches.
    dev = torch.device("cuda", 0)
    shape = (1, 2, 256, 64)
    q, k, v = (t.to(dev) for t in make_random(shape, torch.float16, seed=3))
    o = torch.empty_like(q)
    lse = torch.empty(shape[:3], dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    p = _params(q, k, v, o, lse, 0.125, False, status)
    p.workspace = ws.data_ptr()
    p.workspace_bytes = 256
    assert lib.fa_fwd_sm100_noalloc(ctypes.byref(p), None) == _lib.FA_ERR_BAD_PARAM
    assert b"workspace" in lib.fa_last_error()
    # Bad arguments are reported as such before the workspace is looked at.
    p.head_dim = 96
    assert lib.fa_fwd_sm100_noalloc(ctypes.byref(p), None) == _lib.FA_ERR_UNSUPPORTED
    assert b"head_dim" in lib.fa_last_error()
