"""GPU test of the kernel's bounded waits and abort path.

Every mbarrier wait in the kernel gives up after ``fa_fwd_params.timeout_ns``
(default 2 s).  On expiry the waiting thread writes ``0x100 | site`` to the
caller's status word, raises the CTA's abort flag so that every other role's
waits end too, drains its own TMA loads and MMAs in flight, frees TMEM and
returns; the launch completes and the CUDA context stays usable.

This test reaches that path with a normal launch: a limit of a few nanoseconds
on a configuration-2-sized input (at each head dimension, since each
instantiation carries its own copy of the path), where the first wait that does
not succeed on its first poll expires.  Nothing is left unfinished on the GPU: every wait is
still bounded.  The test then checks that the call returned, that the status
word carries the timeout flag and a known site, and that the next launch on the
same context, with the default limit, matches the CPU oracle.
"""
from __future__ import annotations

import ctypes
import math

import pytest
import torch

from oracle.oracle import oracle_attention
from parity import compare_lse, compare_output

from flash_attention_runtime import _lib
from flash_attention_runtime.inputs import make_random

pytestmark = pytest.mark.gpu

_DT = {torch.float16: _lib.FA_DTYPE_F16, torch.bfloat16: _lib.FA_DTYPE_BF16}
N_SITES = 11  # wait sites numbered 1..11 in the kernel (kWaitSched .. kWaitStatsEmpty)


def _params(q, k, v, o, lse, scale, causal, status, timeout_ns):
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
    p.timeout_ns = timeout_ns
    return p


@pytest.mark.parametrize("timeout_ns,d,dtype,causal", [
    (1, 128, torch.bfloat16, True),
    (300, 128, torch.bfloat16, True),
    (1, 64, torch.float16, False),
    (1, 32, torch.float16, False),
])
def test_expired_waits_abort_cleanly_and_the_context_stays_usable(timeout_ns, d, dtype, causal):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    # configuration-2 sized (B8 H32 N4096), at this head dim / dtype / mask
    shape = (8, 32, 4096, d)
    big = [torch.randn(shape, device=dev, dtype=dtype) for _ in range(3)]
    o = torch.empty_like(big[0])
    lse = torch.empty(shape[:3], dtype=torch.float32, device=dev)
    p = _params(*big, o, lse, 1.0 / math.sqrt(d), causal, status, timeout_ns)
    rc = lib.fa_fwd_sm100(ctypes.byref(p), stream)
    assert rc == _lib.FA_OK, lib.fa_last_error()
    torch.cuda.synchronize(dev)  # the launch finished: no wait was left unbounded
    st = int(status.item())
    assert st & 0x100, hex(st)
    assert 1 <= (st & 0xFF) <= N_SITES, hex(st)
    del big, o, lse

    # The same context, the default limit: a normal launch matches the oracle.
    status.zero_()
    small = (2, 16, 1000, d)
    q, k, v = make_random(small, dtype, seed=41)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    o = torch.full_like(qd, float("nan"))
    lse = torch.full(small[:3], float("nan"), dtype=torch.float32, device=dev)
    scale = 1.0 / math.sqrt(d)
    p = _params(qd, kd, vd, o, lse, scale, causal, status, 0)
    assert lib.fa_fwd_sm100(ctypes.byref(p), stream) == _lib.FA_OK, lib.fa_last_error()
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0
    ref_o, ref_lse = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale, causal)
    ro = compare_output(o, ref_o, dtype)
    rl = compare_lse(lse, ref_lse)
    assert ro["ok"], ro
    assert rl["ok"], rl
