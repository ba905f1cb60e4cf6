"""The C++ driver (flash-attention_b200/csrc/fa_driver): the reference's C++
benchmark/correctness drivers (benchmark/cpp/benchmark_v6.cu,
benchmark/cpp/correctness_v6.cu) re-pointed at fa_fwd_sm100, with no Python or
torch on the launch path.

CPU tests check its command line: usage, argument errors, and a clean error
where no GPU is present.  GPU tests run it with --dump and check the inputs it
generated and the outputs it computed against the CPU oracle, and check its
JSON line.
"""
from __future__ import annotations

import json
import math
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from parity import compare_lse, compare_output

ROOT = Path(__file__).resolve().parent.parent
DRIVER = ROOT / "flash-attention_b200" / "csrc" / "fa_driver"


def _run(*args, timeout=600):
    if not DRIVER.exists():
        pytest.skip("fa_driver is not built")
    return subprocess.run([str(DRIVER), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def test_usage_names_the_reference_options():
    r = _run("--help")
    assert r.returncode == 0
    for opt in ("--mode benchmark|ncu", "--warmup-iters", "--benchmark-iters", "BxHxNxD", "cfg2"):
        assert opt in r.stdout


@pytest.mark.parametrize("args,msg", [
    (["1x2"], "not a workload name or BxHxNxD shape"),
    (["1x2x3x4x5"], "not a workload name or BxHxNxD shape"),
    (["0x2x128x64"], "not a workload name or BxHxNxD shape"),
    (["--mode", "fast"], "invalid --mode"),
    (["--dtype", "f32"], "invalid --dtype"),
    (["--benchmark-iters", "0"], "bad --benchmark-iters"),
    (["--scale", "-1"], "bad --scale"),
    (["--warmup-iters"], "needs a value"),
    (["--bogus"], "unknown option"),
    (["cfg0", "cfg1"], "unexpected extra argument"),
])
def test_argument_errors(args, msg):
    r = _run(*args)
    assert r.returncode == 2
    assert msg in r.stderr


def test_no_device_is_a_clean_error():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = _run("cfg0")
    assert r.returncode == 1
    assert "no CUDA device" in r.stderr


def _load16(path: Path, dtype: str, shape) -> np.ndarray:
    u = np.fromfile(path, dtype=np.uint16).reshape(shape)
    if dtype == "bf16":
        return (u.astype(np.uint32) << 16).view(np.float32)
    return u.view(np.float16).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("args", [
    ["cfg0", "--seed", "7"],
    ["1x3x300x128", "--dtype", "bf16", "--causal", "--seed", "3"],
    ["2x2x129x32", "--dtype", "f16", "--non-causal", "--scale", "0.3"],
    ["1x2x1000x64", "--dtype", "bf16", "--causal", "--flush"],
])
def test_driver_output_matches_the_oracle(tmp_path, args):
    from oracle.oracle import oracle_attention

    r = _run(*args, "--warmup-iters", 1, "--benchmark-iters", 3, "--dump", tmp_path)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["status"] == 0 and line["nonfinite"] == 0 and line["iters"] == 3
    meta = json.loads((tmp_path / "meta.json").read_text())
    shape, dt, causal, scale = tuple(meta["shape"]), meta["dtype"], bool(meta["causal"]), meta["scale"]
    assert list(shape) == line["shape"] and dt == line["dtype"]
    q, k, v = (_load16(tmp_path / f"{t}.bin", dt, shape) for t in "qkv")
    # the generator draws N(0, 1)
    assert abs(float(q.mean())) < 0.05 and 0.9 < float(q.std()) < 1.1
    o = _load16(tmp_path / "o.bin", dt, shape)
    lse = np.fromfile(tmp_path / "lse.bin", dtype=np.float32).reshape(shape[:3])
    ref_o, ref_lse = oracle_attention(q, k, v, scale, causal)
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    ro = compare_output(torch.from_numpy(o), ref_o, tdt)
    rl = compare_lse(torch.from_numpy(lse), ref_lse)
    assert ro["ok"], ro
    assert rl["ok"], rl


@pytest.mark.gpu
def test_driver_benchmark_line_cfg1():
    r = _run("cfg1", "--warmup-iters", 3, "--benchmark-iters", 20, "--flush")
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["workload"] == "cfg1" and line["shape"] == [4, 16, 1024, 64] and line["dtype"] == "f16"
    assert line["causal"] == 0 and line["l2_flush"] is True
    assert math.isclose(line["scale"], 0.125, rel_tol=1e-6)
    assert line["ms_min"] <= line["ms_median"] and line["tflops"] > 0
    assert line["status"] == 0 and line["nonfinite"] == 0
