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
