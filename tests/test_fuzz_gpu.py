"""Seeded random parity cases on the GPU: shapes, dtypes, masks, scales and memory
layouts drawn at random, each checked against the CPU oracle (the restatement of
the reference's cpu_reference_attention, benchmark/cpp/correctness_v6.cu:23-72).

The fixed cases in test_forward_gpu.py cover the configurations and the edge
cases one by one; these combine them: any N from 1 to 700 with either mask, batch
and head counts that give one to a few hundred work units, a softmax scale other
than 1/sqrt(d), and Q, K, V, O as views with their own strides and offsets into
larger buffers ([B,N,H,d] memory, padded rows, a slice of a wider head dimension).
"""
from __future__ import annotations

import math
import random

import pytest
import torch

from oracle.oracle import oracle_attention
from parity import compare_lse, compare_output

import flash_attention_runtime as fa

pytestmark = pytest.mark.gpu

N_CASES = 40


def _view(t: torch.Tensor, layout: str, dev) -> torch.Tensor:
    """A device view with the values of t ([B,H,N,d]) in the given memory layout."""
    b, h, n, d = t.shape
    if layout == "contiguous":
        return t.to(dev)
    if layout == "bnhd":  # [B, N, H, d] memory viewed as [B, H, N, d]
        return t.transpose(1, 2).contiguous().to(dev).transpose(1, 2)
    if layout == "padded_rows":  # every row of d elements padded to d + 8
        buf = torch.full((b, h, n, d + 8), float("nan"), dtype=t.dtype, device=dev)
        buf[..., :d] = t.to(dev)
        return buf[..., :d]
    if layout == "offset":  # a view starting 64 elements into a larger buffer
        buf = torch.full((t.numel() + 64,), float("nan"), dtype=t.dtype, device=dev)
        v = buf[64:].view(b, h, n, d)
        v.copy_(t.to(dev))
        return v
    raise ValueError(layout)


@pytest.mark.parametrize("case", range(N_CASES))
def test_random_case(case):
    rnd = random.Random(1000 + case)
    d = rnd.choice([32, 64, 128])
    dtype = rnd.choice([torch.float16, torch.bfloat16])
    causal = rnd.random() < 0.5
    n = rnd.choice([rnd.randint(1, 130), rnd.randint(1, 700)])
    b = rnd.randint(1, 3)
    h = rnd.randint(1, 5) if n > 64 else rnd.randint(1, 40)
    scale = rnd.uniform(0.05, 0.35)
    layouts = [rnd.choice(["contiguous", "bnhd", "padded_rows", "offset"]) for _ in range(4)]
    with_lse = rnd.random() < 0.8

    g = torch.Generator(device="cpu")
    g.manual_seed(2000 + case)
    # magnitudes up to 1.25x N(0,1): the parity bound then holds for fp16 P rounding too
    q, k, v = (torch.randn((b, h, n, d), generator=g).mul_(rnd.uniform(0.5, 1.25)).to(dtype) for _ in range(3))
    dev = torch.device("cuda", 0)
    qd, kd, vd = (_view(t, lay, dev) for t, lay in zip((q, k, v), layouts))
    od = _view(torch.zeros((b, h, n, d), dtype=dtype), layouts[3], dev)
    lse = torch.empty((b, h, n), dtype=torch.float32, device=dev) if with_lse else None
    fa.reset_device_status(dev)
    out, _ = fa.ext_forward(qd, kd, vd, od, False, scale, causal, lse)
    torch.cuda.synchronize(dev)
    assert fa.device_status(dev) == 0
    assert out.data_ptr() == od.data_ptr()
    ref_o, ref_lse = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale, causal)
    ro = compare_output(od, ref_o, dtype)
    assert ro["ok"], (case, d, dtype, causal, n, b, h, layouts, ro)
    if with_lse:
        rl = compare_lse(lse, ref_lse)
        assert rl["ok"], (case, rl)
    # the inputs were not modified
    for dst, src in zip((qd, kd, vd), (q, k, v)):
        assert torch.equal(dst.cpu(), src)
    assert math.isfinite(ro["max_abs"])
