"""The reference's own Python callers, run against this module.

The reference gates its pybind kernel with
benchmark/python/tests/test_pybind_correctness.py:86-119: for each case of
``--cases`` (default 2x4x128x64, 2x4x256x64, 2x4x128x128, 2x4x256x128) it draws
q, k, v with ``generate_qkv`` on the device, calls ``fa2.forward(q, k, v)``
(``fa2`` = ``flash_attention_runtime``) and compares with
softmax(Q K^T / sqrt(d)) V from PyTorch under ``torch.allclose`` (fp16: atol
2e-2, rtol 2e-2).  Its benchmark loop (benchmark/python/benchmark_pybind.py:326)
times ``fa2.forward_timed(q, k, v)``, and test_pybind_interface.py prints the
``(out, ms)`` pair it returns.  These tests make the same calls, in the same
order and with the same defaults, and additionally hold the output to this
repository's tolerances against the CPU oracle.
"""
from __future__ import annotations

import math

import pytest
import torch

from oracle.oracle import oracle_attention
from parity import compare_output

import flash_attention_runtime as fa2
from flash_attention_runtime.inputs import generate_qkv

pytestmark = pytest.mark.gpu

DEFAULT_CASES = [(2, 4, 128, 64), (2, 4, 256, 64), (2, 4, 128, 128), (2, 4, 256, 128)]


def pytorch_attention(q, k, v):
    """softmax(Q K^T / sqrt(d)) V in float32 PyTorch."""
    qf, kf, vf = q.float(), k.float(), v.float()
    scores = torch.matmul(qf, kf.transpose(-2, -1)) * (1.0 / math.sqrt(q.shape[-1]))
    return torch.matmul(torch.softmax(scores, dim=-1), vf)


@pytest.mark.parametrize("input_mode", ["random", "structured", "stress"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_pybind_correctness_gate(input_mode, dtype):
    for i, (b, h, n, d) in enumerate(DEFAULT_CASES):
        q, k, v, _ = generate_qkv(batch_size=b, n_heads=h, seq_len=n, d_head=d, dtype=dtype, device="cuda",
                                  input_mode=input_mode, seed=1234, case_index=i)
        out = fa2.forward(q, k, v)
        assert out.shape == q.shape and out.dtype == dtype
        ref = pytorch_attention(q, k, v)
        # the reference's own gate (fp16 tolerances)
        assert torch.allclose(ref, out.float(), atol=2e-2, rtol=2e-2), float((ref - out.float()).abs().max())
        # this repository's tolerances against the CPU oracle
        ref_o, _ = oracle_attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                    1.0 / math.sqrt(d), False)
        if input_mode == "stress":
            r = compare_output(out, ref_o, dtype, atol=2e-2, rtol=2e-2)
        else:
            r = compare_output(out, ref_o, dtype)
        assert r["ok"], (i, r)


def test_benchmark_loop_and_interface_calls():
    """forward_timed(q, k, v) as the benchmark loop calls it: (out, ms), ms > 0,
    the same output as forward(); fp32 input raises as the reference's pybind
    check does (python/flash_attention_runtime/_ext.cu:47)."""
    b, h, n, d = 2, 4, 256, 128
    q, k, v, _ = generate_qkv(batch_size=b, n_heads=h, seq_len=n, d_head=d, dtype=torch.float16, device="cuda",
                              input_mode="random", seed=1234, case_index=0)
    ref = fa2.forward(q, k, v)
    for _ in range(5):
        out, ms = fa2.forward_timed(q, k, v)
        assert isinstance(ms, float) and ms > 0.0
        assert torch.equal(out, ref)
    o = torch.empty_like(q)
    out, ms = fa2.forward_timed(q, k, v, o)
    assert out.data_ptr() == o.data_ptr() and torch.equal(o, ref)
    with pytest.raises(RuntimeError, match="float16 or bfloat16"):
        fa2.forward(q.float(), k.float(), v.float())
    with pytest.raises(RuntimeError, match="head_dim"):
        fa2.forward(q[..., :48], k[..., :48], v[..., :48])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
def test_vs_library_attention(dtype, causal):
    """benchmark/python/tests/test_pybind_vs_official_correctness.py:95-160 compares
    fa2.forward with an official library kernel on its default cases (2x4x{128,256,
    512}x128, inputs from generate_qkv) at fp16 2e-2 / bf16 3e-2 (atol = rtol).
    Here the library kernel is PyTorch's scaled_dot_product_attention on the same
    device; the causal variant uses its is_causal mask (col > row masked)."""
    import torch.nn.functional as F

    tol = 2e-2 if dtype == torch.float16 else 3e-2
    for i, (b, h, n, d) in enumerate([(2, 4, 128, 128), (2, 4, 256, 128), (2, 4, 512, 128)]):
        q, k, v, _ = generate_qkv(batch_size=b, n_heads=h, seq_len=n, d_head=d, dtype=dtype, device="cuda",
                                  input_mode="random", seed=1234, case_index=i)
        out = fa2.forward(q, k, v, causal=causal)
        official = F.scaled_dot_product_attention(q, k, v, is_causal=causal)
        diff = (official.float() - out.float()).abs()
        assert torch.allclose(official.float(), out.float(), atol=tol, rtol=tol), (i, float(diff.max()))
