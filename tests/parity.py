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

Every comparison also records the plain max-abs error against the fp32 oracle
and against the oracle rounded to the output dtype (the bound an exactly
rounded result would meet), with the largest |ref| among elements over the plain
bound; conftest.py prints these per test at the end of the session.
"""
from __future__ import annotations

import os

import numpy as np
import torch

# (test id, figures) of every compare_output / compare_lse call in this process
RECORDS: list = []

ATOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
LSE_RTOL = 1e-4
_MANT_BITS = {torch.float16: 10, torch.bfloat16: 7}


def ulp(x: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    """Spacing of `dtype` numbers at |x| (normal range)."""
    m = _MANT_BITS[dtype]
    ax = np.maximum(np.abs(x), np.float32(2.0 ** -14))
    e = np.floor(np.log2(ax))
    return np.exp2(e - m).astype(np.float32)


def _test_id() -> str:
    return os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]


def compare_output(out: torch.Tensor, ref: np.ndarray, dtype: torch.dtype, atol=None, rtol=0.0) -> dict:
    o = out.float().cpu().numpy()
    ref = np.asarray(ref, dtype=np.float32).reshape(o.shape)
    err = np.abs(o - ref)
    plain = ATOL[dtype] if atol is None else atol
    bound = plain + rtol * np.abs(ref) + 0.5 * ulp(ref, dtype)
    finite = bool(np.isfinite(o).all())
    rounded = torch.from_numpy(ref).to(dtype).float().numpy()
    err_r = np.abs(o - rounded)
    over = err > plain + rtol * np.abs(ref)
    r = {
        "max_abs": float(err.max()) if err.size else 0.0,
        "max_abs_vs_rounded_ref": float(err_r.max()) if err.size else 0.0,
        "mean_abs": float(err.mean()) if err.size else 0.0,
        "plain_bound": plain,
        "n_over_plain_bound": int(over.sum()),
        "max_ref_over_plain_bound": float(np.abs(ref[over]).max()) if over.any() else 0.0,
        "worst_excess": float((err - bound).max()) if err.size else 0.0,
        "n_big_ref": int((np.abs(ref) >= 4).sum()),
        "ok": finite and bool((err <= bound).all()),
    }
    RECORDS.append((_test_id(), "O", r))
    return r


def compare_lse(lse: torch.Tensor, ref: np.ndarray) -> dict:
    x = lse.float().cpu().numpy()
    d = np.abs(x - ref)
    guarded = d / np.maximum(1.0, np.abs(ref))
    plain = d / np.maximum(np.abs(ref), 1e-30)
    r = {
        "max_guarded_rel": float(guarded.max()),
        "max_plain_rel": float(plain.max()),
        "ok": bool(np.isfinite(x).all()) and bool((guarded <= LSE_RTOL).all()),
    }
    RECORDS.append((_test_id(), "LSE", r))
    return r
