"""CPU tests of the input generators (flash_attention_runtime/inputs.py).

``generate_qkv`` is the interface the reference's own drivers call
(benchmark/python/input_data.py:115-145, used by
benchmark/python/tests/test_pybind_correctness.py and benchmark_pybind.py):
per-case seeds ``seed + 100003 * case_index``, draws in the requested dtype on
the requested device, and replay files in [B, H, N, d] or [B, N, H, d].
"""
from __future__ import annotations

import pytest
import torch

from flash_attention_runtime.inputs import CONFIGS, case_seed, generate, generate_qkv, make_structured


def _gen(mode, case_index=0, seed=1234, dtype=torch.float16, shape=(2, 4, 128, 64), **kw):
    b, h, n, d = shape
    return generate_qkv(batch_size=b, n_heads=h, seq_len=n, d_head=d, dtype=dtype, device="cpu",
                        input_mode=mode, seed=seed, case_index=case_index, **kw)


def test_case_seeds_and_random_draws():
    assert case_seed(1234, 0) == 1234 and case_seed(1234, 3) == 1234 + 3 * 100003
    q, k, v, path = _gen("random", case_index=2)
    assert path is None and q.dtype == torch.float16 and q.is_contiguous()
    g = torch.Generator(device="cpu")
    g.manual_seed(1234 + 2 * 100003)
    assert torch.equal(q, torch.randn(q.shape, dtype=torch.float16, generator=g))
    assert torch.equal(k, torch.randn(q.shape, dtype=torch.float16, generator=g))
    q2, _, _, _ = _gen("random", case_index=3)
    assert not torch.equal(q, q2)


def test_structured_and_stress_modes():
    q, k, v, _ = _gen("structured", dtype=torch.bfloat16)
    rq, rk, rv = make_structured((2, 4, 128, 64), torch.bfloat16)
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)
    q, k, v, _ = _gen("stress")
    # x32 / x16 scales plus sparse +256 (Q), -256 (K) and +64 (V) outliers
    assert float(q.float().abs().max()) > 200 and float(k.float().abs().max()) > 200
    assert float(v.float().std()) == pytest.approx(16.0, rel=0.1)


def test_replay_bnhd_is_permuted(tmp_path):
    q, k, v, _ = _gen("random", shape=(1, 3, 16, 32))
    torch.save({"q": q.permute(0, 2, 1, 3), "k": k.permute(0, 2, 1, 3), "v": v.permute(0, 2, 1, 3)},
               tmp_path / "case.pt")
    rq, rk, rv, path = _gen("replay", shape=(1, 3, 16, 32), replay_dir=tmp_path)
    assert path == tmp_path / "case.pt"
    assert torch.equal(rq, q) and torch.equal(rk, k) and torch.equal(rv, v)
    torch.save([q, k, v], tmp_path / "b.pt")
    rq, _, _, _ = _gen("replay", shape=(1, 3, 16, 32), replay_dir=tmp_path, replay_file="b.pt")
    assert torch.equal(rq, q)
    with pytest.raises(RuntimeError, match="not found"):
        _gen("replay", shape=(1, 3, 16, 32), replay_dir=tmp_path, replay_file="missing.pt")
    with pytest.raises(RuntimeError, match="Unsupported"):
        _gen("bogus")


def test_baseline_configurations():
    cfg = CONFIGS["cfg2"]
    assert (cfg.batch, cfg.heads, cfg.seq_len, cfg.head_dim, cfg.causal, cfg.seed) == (8, 32, 4096, 128, True, 2)
    assert cfg.flops() == 4 * 8 * 32 * 4096 ** 2 * 128 / 2
    q, k, v = generate(CONFIGS["cfg0"])
    g = torch.Generator(device="cpu")
    g.manual_seed(0)
    assert torch.equal(q, torch.randn(q.shape, generator=g).to(torch.float16))
