"""GPU parity tests: the sm_100a kernel (through the C ABI, via flash_attention_runtime)
against the CPU oracle restating the reference's cpu_reference_attention
(benchmark/cpp/correctness_v6.cu:23-72) on the same seeded, dtype-rounded inputs.

Sizes are ones the oracle finishes in seconds; full-size configurations are
checked through size-independent properties at the end of this file.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle.oracle import oracle_attention
from parity import compare_lse, compare_output

import flash_attention_runtime as fa
from flash_attention_runtime.inputs import CONFIGS, generate, make_random, make_stress, make_structured

pytestmark = pytest.mark.gpu


def _run_and_check(q, k, v, causal, scale=None, slices=None, atol=None, rtol=0.0):
    dev = torch.device("cuda", 0)
    dtype = q.dtype
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    fa.reset_device_status(dev)
    out, lse = fa.forward(qd, kd, vd, softmax_scale=scale, causal=causal, return_lse=True)
    torch.cuda.synchronize(dev)
    assert fa.device_status(dev) == 0
    ref_o, ref_lse = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale, causal,
                                      slices=slices)
    if slices is not None:
        b, h = q.shape[:2]
        s0, s1 = slices
        out = out.reshape(b * h, *out.shape[2:])[s0:s1]
        lse = lse.reshape(b * h, -1)[s0:s1]
        ref_o = ref_o.reshape(b * h, *ref_o.shape[2:])[s0:s1]
        ref_lse = ref_lse.reshape(b * h, -1)[s0:s1]
    ro = compare_output(out, ref_o, dtype, atol=atol, rtol=rtol)
    rl = compare_lse(lse, ref_lse)
    assert ro["ok"], ro
    assert rl["ok"], rl
    return ro, rl


def test_cfg0_correctness_case():
    """Config 0: B1 H4 N256 d64 fp16, seed 0, non-causal, scale 1/8, with LSE."""
    cfg = CONFIGS["cfg0"]
    q, k, v = generate(cfg)
    _run_and_check(q, k, v, cfg.causal, cfg.scale)


def test_cfg1_full():
    """Config 1: B4 H16 N1024 d64 fp16, seed 1, non-causal - every slice checked."""
    cfg = CONFIGS["cfg1"]
    q, k, v = generate(cfg)
    _run_and_check(q, k, v, cfg.causal, cfg.scale)


@pytest.mark.parametrize("d", [32, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
def test_head_dims_dtypes_masks(d, dtype, causal):
    q, k, v = make_random((2, 3, 512, d), dtype, seed=100 + d)
    _run_and_check(q, k, v, causal)


@pytest.mark.parametrize("n", [1, 7, 64, 127, 128, 129, 200, 255, 256, 257, 383, 640, 1000])
@pytest.mark.parametrize("causal", [False, True])
def test_ragged_seq_len(n, causal):
    """Sequence lengths that are not multiples of the 128-row tiles (tail masking)."""
    q, k, v = make_random((1, 2, n, 64), torch.bfloat16, seed=7 + n)
    _run_and_check(q, k, v, causal)


@pytest.mark.parametrize("n,d", [(100, 64), (129, 128), (300, 32), (300, 128), (1000, 64)])
@pytest.mark.parametrize("causal", [False, True])
def test_ragged_many_units(n, d, causal):
    """200 (b,h) slices, more work units than the 148 persistent CTAs, so each CTA
    runs several units back to back (the next unit's first S is issued inside the
    last key block of the current one), including units whose second 128-row query
    tile lies past the sequence end (n = 100, 300).  Every slice is checked."""
    dtype = torch.float16 if causal else torch.bfloat16
    q, k, v = make_random((2, 100, n, d), dtype, seed=31 + n + d)
    _run_and_check(q, k, v, causal)


def _run_config_and_check_slices(cfg, slices):
    """One forward of the whole configuration on the GPU; the listed (b,h) slices
    of O and LSE checked against the oracle (run on host threads over just those
    slices)."""
    q, k, v = generate(cfg)
    dev = torch.device("cuda", 0)
    fa.reset_device_status(dev)
    out, lse = fa.forward(q.to(dev), k.to(dev), v.to(dev), softmax_scale=cfg.scale, causal=cfg.causal,
                          return_lse=True)
    torch.cuda.synchronize(dev)
    assert fa.device_status(dev) == 0
    s = cfg.slices
    idx = torch.tensor(slices)
    pick = lambda t: t.reshape(s, *t.shape[2:])[idx].unsqueeze(0)  # noqa: E731
    ref_o, ref_lse = oracle_attention(pick(q).float().numpy(), pick(k).float().numpy(), pick(v).float().numpy(),
                                      cfg.scale, cfg.causal)
    ro = compare_output(pick(out.cpu()), ref_o, cfg.dtype)
    rl = compare_lse(pick(lse.cpu()), ref_lse)
    assert ro["ok"], ro
    assert rl["ok"], rl
    return out, lse, (q, k, v)


@pytest.mark.parametrize("d", [32, 64, 128])
def test_cfg4_full_every_slice(d):
    """Configuration 4 at full size (B16 H16 N2048, fp16, non-causal, 1% of Q/K
    entries x20): all 256 slices against the oracle, for each head dim."""
    cfg = CONFIGS[f"cfg4_d{d}"]
    _run_config_and_check_slices(cfg, list(range(cfg.slices)))


def test_stress_and_structured_modes():
    """The reference's `stress` and `structured` input modes (input_data.py:33-60)."""
    # |O| up to ~60 here: the reference's own tolerance for this mode (see tests/parity.py).
    _run_and_check(*make_stress((1, 2, 384, 128), torch.float16, seed=11), causal=False, atol=2e-2, rtol=2e-2)
    _run_and_check(*make_structured((2, 2, 256, 64), torch.bfloat16), causal=True)


def test_user_scale():
    q, k, v = make_random((1, 2, 256, 64), torch.float16, seed=3)
    _run_and_check(q, k, v, causal=True, scale=0.37)


def test_cfg2_every_slice():
    """Headline configuration 2 (B8 H32 N4096 d128 bf16 causal) at full size: all
    256 (b,h) slices of O and LSE against the oracle."""
    cfg = CONFIGS["cfg2"]
    _run_config_and_check_slices(cfg, list(range(cfg.slices)))


def test_masked_keys_contribute_exactly_zero():
    """Causal, bf16: V rows 64..127 set to 2^120, far beyond any other value, so a
    masked key's P must be exactly 0 (a P of even 2^-125 would move the output by
    about 2^-5).  Rows 0..63 mask keys 64..127 inside their first key block, on
    both the MUFU and the FMA-pipe exp2 columns; their output must match the
    oracle, which masks with P = exp(-inf) = 0."""
    q, k, v = make_random((2, 3, 256, 128), torch.bfloat16, seed=55)
    v[:, :, 64:128] = 2.0 ** 120
    dev = torch.device("cuda", 0)
    out, lse = fa.forward(q.to(dev), k.to(dev), v.to(dev), causal=True, return_lse=True)
    torch.cuda.synchronize(dev)
    scale = 1.0 / math.sqrt(128)
    ref_o, ref_lse = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale, True)
    ro = compare_output(out[:, :, :64], ref_o[:, :, :64], torch.bfloat16)
    assert ro["ok"], ro
    assert compare_lse(lse, ref_lse)["ok"]


def test_strided_bnhd_layout():
    """[B, N, H, d] memory viewed as [B, H, N, d] (non-contiguous, last dim contiguous)."""
    q, k, v = make_random((2, 3, 256, 64), torch.bfloat16, seed=21)
    dev = torch.device("cuda", 0)
    qs, ks, vs = (t.to(dev).transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    assert not qs.is_contiguous()
    out, lse = fa.forward(qs, ks, vs, causal=True, return_lse=True)
    torch.cuda.synchronize(dev)
    ref_o, ref_lse = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), 1 / 8, True)
    assert compare_output(out, ref_o, torch.bfloat16)["ok"]
    assert compare_lse(lse, ref_lse)["ok"]


@pytest.mark.parametrize("big_dim", [0, 1])
def test_strides_past_2_31_elements(big_dim):
    """A batch (big_dim=0) or head (big_dim=1) stride of 2^31 + 1024 elements, which
    only the 64-bit stride fields of fa_fwd_params can carry.  Q, K, V and O are
    views at different offsets into one 4.3 GB buffer, each touching two 32K-element
    islands 2^31 + 1024 elements apart; nothing else of the buffer is read."""
    shape = (2, 2, 256, 64) if big_dim == 0 else (1, 2, 256, 64)
    b, h, n, d = shape
    big = (1 << 31) + 1024
    inner = h * n * d if big_dim == 0 else n * d  # span below the big stride
    strides = (big, n * d, d, 1) if big_dim == 0 else (h * big, big, d, 1)
    dev = torch.device("cuda", 0)
    buf = torch.empty(big + 4 * inner, dtype=torch.bfloat16, device=dev)
    views = [buf.as_strided(shape, strides, storage_offset=i * inner) for i in range(4)]
    q, k, v = make_random(shape, torch.bfloat16, seed=31 + big_dim)
    for dst, src in zip(views, (q, k, v)):
        dst.copy_(src.to(dev))
    out = views[3]
    out.fill_(float("nan"))
    assert max(t.stride(big_dim) for t in views) > 2 ** 31
    lse = torch.empty((b, h, n), dtype=torch.float32, device=dev)
    ret, _ = fa.ext_forward(views[0], views[1], views[2], out, False, 0.125, True, lse)
    assert ret.data_ptr() == out.data_ptr()
    torch.cuda.synchronize(dev)
    ref_o, ref_lse = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), 0.125, True)
    ro = compare_output(out, ref_o, torch.bfloat16)
    rl = compare_lse(lse, ref_lse)
    assert ro["ok"], ro
    assert rl["ok"], rl
    # the inputs were not overwritten
    for view, src in zip(views, (q, k, v)):
        assert torch.equal(view.cpu(), src)
    del views, out, buf
    torch.cuda.empty_cache()


def test_forward_timed_and_reference_call_shape():
    """forward(q,k,v) with the reference defaults, forward_timed returns (o, ms)."""
    q, k, v = make_random((1, 2, 256, 128), torch.float16, seed=5)
    dev = torch.device("cuda", 0)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    o1 = fa.forward(qd, kd, vd)
    o2, ms = fa.forward_timed(qd, kd, vd)
    assert ms > 0.0
    assert torch.equal(o1, o2)
    o3 = torch.empty_like(qd)
    ret, _ = fa.ext_forward(qd, kd, vd, o3, False)
    assert ret.data_ptr() == o3.data_ptr()
    assert torch.equal(o3, o1)


def test_deterministic_repeat():
    q, k, v = make_random((2, 4, 1024, 128), torch.bfloat16, seed=9)
    dev = torch.device("cuda", 0)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    a = fa.forward(qd, kd, vd, causal=True)
    b = fa.forward(qd, kd, vd, causal=True)
    assert torch.equal(a, b)


def test_cfg3_every_slice_and_properties():
    """Configuration 3 (B2 H32 N16384 d128 bf16 causal) at full size: all 64 (b,h)
    slices against the oracle, then size-independent checks: causal row 0 equals
    V row 0, every output row is a convex combination of V rows (within
    [min V, max V] per column), LSE of row 0 equals scale*q0.k0, and a second run
    is bit-identical."""
    cfg = CONFIGS["cfg3"]
    out, lse, (q, k, v) = _run_config_and_check_slices(cfg, list(range(cfg.slices)))
    dev = out.device
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    out2 = fa.forward(qd, kd, vd, causal=True)
    torch.cuda.synchronize(dev)
    assert torch.equal(out, out2)
    assert torch.equal(out[:, :, 0], vd[:, :, 0])
    vmin = vd.float().amin(dim=2, keepdim=True)
    vmax = vd.float().amax(dim=2, keepdim=True)
    of = out.float()
    assert bool(((of >= vmin - 1e-2) & (of <= vmax + 1e-2)).all())
    l0 = (qd[:, :, 0].float() * kd[:, :, 0].float()).sum(-1) * cfg.scale
    assert float((lse[:, :, 0] - l0).abs().max()) < 1e-4 * max(1.0, float(l0.abs().max()))
    assert bool(torch.isfinite(lse).all())


@pytest.mark.parametrize("shape,dtype,causal", [
    ((1, 8, 3001, 128), torch.bfloat16, True),    # ragged causal, 12 units per slice, last one partial
    ((2, 3, 2049, 64), torch.float16, False),     # one row past a 2048-row multiple
    ((1, 4, 5000, 32), torch.float16, True),      # long ragged causal at the smallest head dim
])
def test_large_ragged_sequences(shape, dtype, causal):
    """Sequence lengths far from the 128-row tiles at sizes with many key blocks per
    unit: every slice against the oracle."""
    q, k, v = make_random(shape, dtype, seed=61 + shape[2])
    _run_and_check(q, k, v, causal)


def test_thousands_of_tiny_slices():
    """B64 H64 N64 d32: 4096 slices of one work unit each, so every CTA chains about
    28 units across several scheduling groups; every slice against the oracle."""
    q, k, v = make_random((64, 64, 64, 32), torch.bfloat16, seed=62)
    _run_and_check(q, k, v, causal=True)


@pytest.mark.parametrize("scale", [1e-3, 2.0])
def test_extreme_softmax_scales(scale):
    """A scale of 1e-3 makes the attention nearly uniform over the keys (a long
    accumulation of similar P); 2.0 makes it nearly one-hot (rescales of O as the
    running maximum jumps)."""
    q, k, v = make_random((2, 3, 777, 64), torch.float16, seed=63)
    _run_and_check(q, k, v, causal=False, scale=scale)
    _run_and_check(q, k, v, causal=True, scale=scale)
