"""CPU check of the kernel's FMA-pipe exp2 (exp2_fma in csrc/fa_fwd_kernel.cuh).

The kernel computes 2 of every 8 column pairs of P = 2^(s*scale*log2e - m) with
a polynomial on the FMA pipe instead of the MUFU unit.  This test restates that
routine in numpy float32 arithmetic, with the coefficients read from the kernel
source, and checks the properties the online softmax relies on
(src/softmax/online_softmax.cuh:89-172 computes the same P with exp2):

  * a masked score (x = -inf) gives exactly +0.0, so masked keys contribute
    nothing to P V in either output dtype (causal spec: col > row masked);
  * the row-max element (x = 0) gives exactly 1.0;
  * over the range the kernel passes (x <= 8), the relative error against exact
    2^x stays below 3e-6 wherever 2^x is a normal float.
"""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np

KERNEL = Path(__file__).resolve().parent.parent / "flash-attention_b200" / "csrc" / "fa_fwd_kernel.cuh"


def _coeffs():
    src = KERNEL.read_text()
    c = {}
    for k in (1, 2, 3, 4):
        m = re.search(rf"constexpr float kExp2C{k} = ([0-9.eE+-]+)f;", src)
        assert m, f"kExp2C{k} not found in the kernel source"
        c[k] = np.float32(m.group(1))
    return c


def _fma(a, b, c):
    # a*b is exact in float64 for float32 operands; one rounding to float32 after the add
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_fma(x: np.ndarray) -> np.ndarray:
    """numpy restatement of the kernel's exp2_fma, one lane at a time."""
    c = _coeffs()
    x = np.maximum(x.astype(np.float32), np.float32(-127.0))
    shift = np.float32(12582912.0)
    t = (x + shift).astype(np.float32)
    n = (t - shift).astype(np.float32)
    f = _fma(n, np.full_like(n, -1.0), x)
    q = _fma(np.full_like(f, c[4]), f, np.full_like(f, c[3]))
    q = _fma(q, f, np.full_like(f, c[2]))
    q = _fma(q, f, np.full_like(f, c[1]))
    q = _fma(q, f, np.full_like(f, 1.0))
    bits = (t.view(np.uint32).astype(np.uint64) * 8388608 + q.view(np.uint32).astype(np.uint64)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_masked_score_gives_exact_zero():
    r = exp2_fma(np.array([-np.inf, -np.inf], dtype=np.float32))
    assert r.view(np.uint32).tolist() == [0, 0]


def test_row_max_element_gives_exact_one():
    assert exp2_fma(np.array([0.0], dtype=np.float32))[0] == np.float32(1.0)


def test_relative_error_bound():
    rng = np.random.default_rng(0)
    x = np.concatenate([np.linspace(-126.0, 8.0, 400001, dtype=np.float32),
                        rng.uniform(-20.0, 0.0, 200000).astype(np.float32),
                        np.arange(-126, 9, dtype=np.float32) + np.float32(0.5)])
    r = exp2_fma(x).astype(np.float64)
    exact = np.exp2(x.astype(np.float64))
    rel = np.abs(r / exact - 1.0)
    assert rel.max() < 3e-6, float(rel.max())
    assert np.all(np.isfinite(r)) and np.all(r > 0)


def test_below_the_normal_range_flushes_to_zero_or_stays_tiny():
    x = np.linspace(-200.0, -126.5, 1001, dtype=np.float32)
    r = exp2_fma(x)
    assert np.all(r >= 0) and np.all(r < np.float32(2.0 ** -126))
