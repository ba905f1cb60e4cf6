"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on a CPU-only machine: oracle pinning against the golden
fixtures, layout/descriptor bit math, the C ABI's exports and struct layout, host
validation and the gloo multi-rank sharding logic.  `-m gpu` runs the parity
tests proper through the C ABI on a B200.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "flash-attention_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def pytest_terminal_summary(terminalreporter):
    """Per-test parity figures (max-abs against the oracle, and against the
    oracle rounded to the output dtype), so a run's log carries them."""
    try:
        import parity
    except ImportError:
        return
    if not parity.RECORDS:
        return
    tr = terminalreporter
    tr.write_sep("-", "parity figures (O: max|d| vs fp32 oracle / vs oracle rounded to dtype; LSE: max guarded rel)")
    agg: dict = {}
    for test, kind, r in parity.RECORDS:
        a = agg.get((test, kind))
        if a is None:
            agg[(test, kind)] = dict(r)
            continue
        for key in ("max_abs", "max_abs_vs_rounded_ref", "max_guarded_rel", "max_ref_over_plain_bound"):
            if key in r:
                a[key] = max(a[key], r[key])
        if "n_over_plain_bound" in r:
            a["n_over_plain_bound"] += r["n_over_plain_bound"]
    for (test, kind), a in agg.items():
        if kind == "O":
            tr.write_line(f"{test} O: max_abs {a['max_abs']:.3e} vs_rounded {a['max_abs_vs_rounded_ref']:.3e} "
                          f"plain_bound {a['plain_bound']:.0e} over {a['n_over_plain_bound']} "
                          f"(max|ref| there {a['max_ref_over_plain_bound']:.2f})")
        else:
            tr.write_line(f"{test} LSE: max_guarded_rel {a['max_guarded_rel']:.3e}")
