"""Shared parity helpers: run the CUDA path and compare with the CPU oracle.

Tolerances (from the performance/parity targets):
  * O, float16 inputs : max |out - ref| <= 2e-3
  * O, bfloat16 inputs: max |out - ref| <= 1e-2
    The output itself is stored in the input dtype, so an exact result already
    carries up to half an output ulp of rounding error (0.0156 for bf16 values in
    [4, 8)).  The bound checked is therefore atol + ulp(ref)/2 per element; the
    plain max-abs error and the number of |ref| >= 4 elements are reported too.
  * The reference's `stress` input mode (Q, K x32, V x16, |O| up to ~60) is
    checked with the reference's own fp16 tolerance for its Python test
    (benchmark/python/tests/test_pybind_correctness.py:46-49: atol 2e-2, rtol
    2e-2): rounding P to the input dtype before P V, as the reference kernel does
    (src/forward/forward_v6_mma.cuh:86-98), costs ~|V| * 2^-11 there.
  * LSE: |lse - ref| / max(1, |ref|) <= 1e-4 (the plain relative error is
    ill-conditioned for rows whose logsumexp is near 0, e.g. causal row 0).
"""
from __future__ import annotations

import numpy as np
import torch

ATOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
LSE_RTOL = 1e-4
_MANT_BITS = {torch.float16: 10, torch.bfloat16: 7}


def ulp(x: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    """Spacing of `dtype` numbers at |x| (normal range)."""
    m = _MANT_BITS[dtype]
    ax = np.maximum(np.abs(x), np.float32(2.0 ** -14))
    e = np.floor(np.log2(ax))
    return np.exp2(e - m).astype(np.float32)


def compare_output(out: torch.Tensor, ref: np.ndarray, dtype: torch.dtype, atol=None, rtol=0.0) -> dict:
    o = out.float().cpu().numpy()
    err = np.abs(o - ref)
    bound = (ATOL[dtype] if atol is None else atol) + rtol * np.abs(ref) + 0.5 * ulp(ref, dtype)
    finite = bool(np.isfinite(o).all())
    return {
        "max_abs": float(err.max()) if err.size else 0.0,
        "mean_abs": float(err.mean()) if err.size else 0.0,
        "worst_excess": float((err - bound).max()) if err.size else 0.0,
        "n_big_ref": int((np.abs(ref) >= 4).sum()),
        "ok": finite and bool((err <= bound).all()),
    }


def compare_lse(lse: torch.Tensor, ref: np.ndarray) -> dict:
    x = lse.float().cpu().numpy()
    d = np.abs(x - ref)
    guarded = d / np.maximum(1.0, np.abs(ref))
    plain = d / np.maximum(np.abs(ref), 1e-30)
    return {
        "max_guarded_rel": float(guarded.max()),
        "max_plain_rel": float(plain.max()),
        "ok": bool(np.isfinite(x).all()) and bool((guarded <= LSE_RTOL).all()),
    }
