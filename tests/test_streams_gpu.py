"""GPU test of the library-owned scheduler workspace across host threads.

With ``workspace == NULL``, fa_fwd_sm100 keeps one scheduler counter per
(device, stream).  ``cudaStreamPerThread`` is one handle value that names a
different stream in every host thread, so two threads launching on it must get
two counters: their kernels can overlap on the GPU, and a shared counter would
hand units of one launch to the other's CTAs.  Two threads here launch small
grids (fewer units than SMs, so their kernels can run side by side) on
``cudaStreamPerThread`` in a loop, with no ordering between them; every output
must match the CPU oracle.
"""
from __future__ import annotations

import ctypes
import math
import threading

import pytest
import torch

from oracle.oracle import oracle_attention
from parity import compare_lse, compare_output

from flash_attention_runtime import _lib
from flash_attention_runtime.inputs import make_random

pytestmark = pytest.mark.gpu

CUDA_STREAM_PER_THREAD = 0x2  # the runtime's cudaStreamPerThread handle


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
    p.dtype = _lib.FA_DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.FA_DTYPE_F16
    p.workspace = None
    p.workspace_bytes = 0
    p.status = status.data_ptr()
    p.timeout_ns = 0
    return p


def test_two_threads_on_the_per_thread_default_stream():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = (1, 12, 2048, 64)  # 12 slices x 8 units = 96 units per launch, fewer than the SMs
    scale = 1.0 / math.sqrt(shape[-1])
    jobs = []
    for seed in (101, 202):
        q, k, v = make_random(shape, torch.bfloat16, seed=seed)
        qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
        o = torch.full_like(qd, float("nan"))
        lse = torch.full(shape[:3], float("nan"), dtype=torch.float32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        jobs.append(dict(host=(q, k, v), p=_params(qd, kd, vd, o, lse, scale, False, status), o=o, lse=lse,
                         status=status, keep=(qd, kd, vd), rc=[]))
    torch.cuda.synchronize(dev)
    start = threading.Barrier(2)

    def worker(job):
        torch.cuda.set_device(dev)
        start.wait()
        for _ in range(20):
            job["rc"].append(lib.fa_fwd_sm100(ctypes.byref(job["p"]), ctypes.c_void_p(CUDA_STREAM_PER_THREAD)))

    threads = [threading.Thread(target=worker, args=(j,)) for j in jobs]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    torch.cuda.synchronize(dev)
    for job in jobs:
        assert job["rc"] == [_lib.FA_OK] * 20
        assert int(job["status"].item()) == 0
        q, k, v = job["host"]
        ref_o, ref_lse = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale, False)
        ro = compare_output(job["o"], ref_o, torch.bfloat16)
        rl = compare_lse(job["lse"], ref_lse)
        assert ro["ok"], ro
        assert rl["ok"], rl
