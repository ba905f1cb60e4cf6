"""CPU tests: pin the oracle (oracle/cpu_attention.cpp) to the reference.

The golden fixtures hold outputs of the reference's own cpu_reference_attention
(benchmark/cpp/correctness_v6.cu:23-72) built from its sources; the oracle must
reproduce them bit for bit.  The logsumexp (which the reference lacks) is
checked against float64 numpy.
"""
from __future__ import annotations

import hashlib
import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from flash_attention_runtime.inputs import CONFIGS, generate, make_random

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not orc.ORACLE_SO.exists():
        orc.build()


def _load_case(name):
    meta = MANIFEST["cases"][name]
    z = np.load(GOLDEN / meta["file"])
    shape = tuple(meta["shape"])
    if "q" in z:
        q, k, v = z["q"], z["k"], z["v"]
    else:
        dt = torch.float16 if meta["dtype"] == "float16" else torch.bfloat16
        q, k, v = (torch.from_numpy(z[f"{n}_bits"].astype(np.int16)).view(dt).float().numpy().reshape(shape)
                   for n in "qkv")
    return q, k, v, z, meta


@pytest.mark.parametrize("name", sorted(MANIFEST["cases"]))
def test_oracle_bit_exact_vs_reference_golden(name):
    q, k, v, z, meta = _load_case(name)
    o, lse = orc.oracle_attention(q, k, v, meta["scale"], meta["causal"])
    assert o.shape == z["o_ref"].shape
    assert np.array_equal(o, z["o_ref"]), float(np.abs(o - z["o_ref"]).max())
    rel = np.abs(lse.astype(np.float64) - z["lse64"]) / np.maximum(1.0, np.abs(z["lse64"]))
    assert rel.max() < 2e-6


def test_cfg0_full_output_checksum():
    """Full configuration 0 (all 4 heads): oracle output hashes to the reference's."""
    cfg = CONFIGS["cfg0"]
    q, k, v = generate(cfg)
    o, _ = orc.oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), cfg.scale, False)
    assert hashlib.sha256(np.ascontiguousarray(o).tobytes()).hexdigest() == MANIFEST["cfg0_full_o_sha256"]


def test_oracle_vs_float64_softmax():
    q, k, v = (t.float().numpy() for t in make_random((2, 2, 96, 32), torch.float16, seed=5))
    for causal in (False, True):
        o, _ = orc.oracle_attention(q, k, v, 0.3, causal)
        s = np.einsum("bhid,bhjd->bhij", q.astype(np.float64), k.astype(np.float64)) * 0.3
        if causal:
            s = np.where(np.triu(np.ones((96, 96), bool), 1), -np.inf, s)
        p = np.exp(s - s.max(-1, keepdims=True))
        ref = (p / p.sum(-1, keepdims=True)) @ v.astype(np.float64)
        assert np.abs(o - ref).max() < 1e-5


def test_threads_do_not_change_bits():
    q, k, v = (t.float().numpy() for t in make_random((2, 3, 64, 64), torch.bfloat16, seed=2))
    o1, l1 = orc.oracle_attention(q, k, v, 0.125, True, threads=1)
    o4, l4 = orc.oracle_attention(q, k, v, 0.125, True, threads=4)
    assert np.array_equal(o1, o4) and np.array_equal(l1, l4)


def test_slice_subset():
    q, k, v = (t.float().numpy() for t in make_random((2, 2, 32, 32), torch.float16, seed=8))
    full, _ = orc.oracle_attention(q, k, v, 0.2, False)
    part, _ = orc.oracle_attention(q, k, v, 0.2, False, slices=(1, 3))
    f = full.reshape(4, 32, 32)
    p = part.reshape(4, 32, 32)
    assert np.array_equal(f[1:3], p[1:3])
    assert np.isnan(p[0]).all() and np.isnan(p[3]).all()


@pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("causal", [False, True])
def test_oracle_bit_exact_vs_reference_live(causal):
    """Random causal/non-causal case through the reference build directly."""
    q, k, v = (t.float().numpy() for t in make_random((1, 3, 160, 64), torch.bfloat16, seed=44))
    scale = 1.0 / math.sqrt(64)
    o, _ = orc.oracle_attention(q, k, v, scale, causal)
    r = orc.ref_attention(q, k, v, scale, causal, threads=3)
    assert np.array_equal(o, r)
