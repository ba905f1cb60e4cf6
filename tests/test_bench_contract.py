"""CPU checks of bench.py's output contract.

The reference arm (the reference's CPU attention, compiled from its sources into
oracle/_ref, or the restated oracle where that build is absent) runs here without
a GPU and must print exactly one JSON line with the fields the harness reads.
Our arm must fail loudly without a GPU rather than print a number.  The L2 policy
flushes between timed launches exactly when a rank's tensors could stay in L2.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def _bench(*args, timeout=600):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *map(str, args)], capture_output=True,
                          text=True, timeout=timeout, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    r = _bench("--impl", "reference", "--workload", "cfg0", "--steps", 2, "--warmup", 1)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.strip().splitlines()
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "TFLOPS" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["vs_baseline"] is None
    assert d["config"]["workload"] == "cfg0"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port")
    assert 1 <= cb["cores"] <= 4  # cfg0 has 4 (b,h) slices: no more threads than slices
    assert cb["sample"].startswith(f"{cb['cores']} of the 4 (b,h) slices of cfg0")
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "rotating" in d["config"]["l2"]


def test_reference_arm_under_torchrun_prints_once_from_rank_0():
    """Launched like the multi-GPU arms (torchrun, two ranks): rank 0 alone runs the
    CPU reference and prints its line; the other rank exits 0 without output."""
    import os
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = {**os.environ, "OMP_NUM_THREADS": "1"}
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), str(ROOT / "bench.py"),
                        "--impl", "reference", "--gpus", "2", "--workload", "cfg0", "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.strip().splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["config"]["workload"] == "cfg0"


def test_our_arm_fails_loudly_without_a_gpu():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = _bench("--workload", "cfg0", "--steps", 2, "--warmup", 1)
    assert r.returncode != 0
    assert r.stdout.strip() == ""


def test_l2_policy_rotates_input_copies_for_small_ranks():
    sys.path.insert(0, str(ROOT))
    import bench

    from flash_attention_runtime.inputs import CONFIGS

    rotated = {name for name, cfg in CONFIGS.items() if bench.input_copies(cfg, 1, "strong") > 1}
    assert {"cfg0", "cfg1", "cfg4_d32"} <= rotated
    assert not rotated & {"cfg2", "cfg3", "cfg4_d128"}
    # Strong scaling splits the slices: at 8 ranks configuration 2 is 134 MB per rank,
    # so three copies rotate (two launches, 268 MB, between uses of one copy).
    assert bench.input_copies(CONFIGS["cfg2"], 8, "strong") == 3
    assert bench.input_copies(CONFIGS["cfg2"], 8, "weak") == 1
    for name, cfg in CONFIGS.items():
        n = bench.input_copies(cfg, 1, "strong")
        assert n == 1 or (n - 1) * bench.rank_bytes(cfg, 1, "strong") >= 2 * bench.L2_BYTES
    assert bench.rank_bytes(CONFIGS["cfg2"], 1, "weak") == 4 * 8 * 32 * 4096 * 128 * 2
    assert "inputs larger than L2" in bench.l2_note(CONFIGS["cfg2"], 1, "weak")
    assert "rotating over 3 copies" in bench.l2_note(CONFIGS["cfg2"], 8, "strong")


def test_strong_split_is_the_default_and_checked_slices_are_strided():
    sys.path.insert(0, str(ROOT))
    import bench

    from flash_attention_runtime.inputs import CONFIGS

    args = bench.parse_args([])
    assert args.scaling == "strong" and args.gpus == 1 and args.warmup >= 3
    assert bench.check_slices(256, 8) == [0, 36, 73, 109, 146, 182, 219, 255]
    assert bench.check_slices(4, 8) == [0, 1, 2, 3]
    assert bench.check_slices(64, 0) == []
    c = bench.workload_config(CONFIGS["cfg2"], 8, "strong")
    assert c["slices"] == 256 and c["slices_per_rank"] == 32 and c["global_batch"] == 8
    c = bench.workload_config(CONFIGS["cfg2"], 8, "weak")
    assert c["slices"] == 8 * 256 and c["slices_per_rank"] == 256 and c["batch_per_rank"] == 8


def test_peak_follows_the_timed_region_length():
    sys.path.insert(0, str(ROOT))
    import bench

    peaks = {"bf16_tflops": 1663.7, "bf16_tflops_sustained": 1389.2}
    assert bench.pick_peak(peaks, 0.02) == (1663.7, "bf16_tflops")
    assert bench.pick_peak(peaks, 1.5) == (1389.2, "bf16_tflops_sustained")


def test_verify_accepts_the_exact_result_and_rejects_a_planted_error():
    """The gathered-output check on CPU tensors: the float64 result rounded to the
    output dtype passes; the same with one element moved by 2e-2 fails."""
    sys.path.insert(0, str(ROOT))
    import bench

    from flash_attention_runtime.inputs import AttnConfig, generate

    cfg = AttnConfig("tiny", 1, 3, 96, 32, torch.bfloat16, True, 5)
    q, k, v = generate(cfg)
    outs, lses = [], []
    for i in range(cfg.slices):
        o, l = bench.reference_slice(q[0, i], k[0, i], v[0, i], cfg.scale, cfg.causal)
        outs.append(o.to(torch.bfloat16))
        lses.append(l.float())
    o_all, l_all = torch.stack(outs), torch.stack(lses)
    r = bench.verify(cfg, (q, k, v), o_all, l_all, [0, 1, 2], torch.device("cpu"))
    assert r["ok"] and r["all_finite"] and r["max_abs_vs_ref_rounded_to_dtype"] == 0.0
    bad = o_all.clone()
    bad[1, 50, 7] += 2e-2
    r = bench.verify(cfg, (q, k, v), bad, l_all, [0, 1, 2], torch.device("cpu"))
    assert not r["ok"]
    r = bench.verify(cfg, (q, k, v), o_all, l_all + 1e-3, [0, 2], torch.device("cpu"))
    assert not r["ok"]


def test_rank_inputs_partition_the_configuration():
    """Strong scaling: rank r's Q, K, V are slices [r*S/N, (r+1)*S/N) of the one
    seeded configuration, and the ranks together hold every slice once."""
    sys.path.insert(0, str(ROOT))
    import bench

    from flash_attention_runtime.inputs import CONFIGS, generate

    cfg = CONFIGS["cfg0"]  # 4 slices
    q, k, v = generate(cfg)
    flat = q.reshape(cfg.slices, cfg.seq_len, cfg.head_dim)
    got = []
    for r in range(3):
        (qr, kr, vr), full, first = bench.rank_inputs(cfg, r, 3, "strong")
        assert qr.shape[0] == 1 and qr.is_contiguous()
        assert torch.equal(full[0], q)
        n = qr.shape[1]
        assert torch.equal(qr[0], flat[first:first + n])
        got.append((first, n))
    assert got == [(0, 2), (2, 1), (3, 1)]
    # weak scaling: every rank a full batch of its own seed
    (q0, _, _), _, _ = bench.rank_inputs(cfg, 0, 2, "weak")
    (q1, _, _), _, _ = bench.rank_inputs(cfg, 1, 2, "weak")
    assert q0.shape == q.shape and torch.equal(q0, q) and not torch.equal(q1, q)
    # --share-of 8 on one process stands in for rank 0 of an 8-way split
    assert bench.parse_args(["--share-of", "8"]).share_of == 8
    assert bench.input_copies(CONFIGS["cfg2"], 8, "strong") == 3
