"""Generate the golden fixtures in tests/golden/ from the REFERENCE'S OWN code.

The outputs come from `cpu_reference_attention` (wenssir/flash-attention
benchmark/cpp/correctness_v6.cu:23-72), compiled from the reference tree where it
lies into oracle/_ref/libref_attention.so by oracle/Makefile.  The reference has
no logsumexp, so the fixtures' LSE is computed independently in float64 numpy
from the same inputs.  Run in a container that has the reference tree:

    make -C oracle && python tests/golden/make_golden.py

Cases:
  ref_v6_case   the reference driver's own case (correctness_v6.cu:110-131):
                srand(17), glibc rand() drawn q,k,v interleaved per element,
                (r/RAND_MAX - 0.5) * 0.2, B1 H1 N64 D128, scale 1/sqrt(128),
                non-causal, unrounded fp32 inputs
  cfg0_head0    configuration 0 (B1 H4 N256 d64 fp16, seed 0), head 0 only;
                the full configuration-0 output is pinned by its sha256
  causal_tail   bf16, B1 H1 N200 d64 causal (N not a multiple of the tile)
  outlier_d32   fp16, B1 H2 N256 d32, 1% of Q/K entries x20 (configuration-4 style)
  stress        fp16, B1 H1 N128 d64, the reference's `stress` input mode
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "flash-attention_b200"))

from oracle import oracle as orc  # noqa: E402
from flash_attention_runtime.inputs import CONFIGS, AttnConfig, generate, make_random, make_stress  # noqa: E402


def glibc_rand_inputs(n_elems: int, seed: int):
    libc = ctypes.CDLL("libc.so.6")
    libc.rand.restype = ctypes.c_int
    libc.srand.argtypes = [ctypes.c_uint]
    libc.srand(seed)
    rand_max = 2147483647
    q = np.empty(n_elems, np.float32)
    k = np.empty(n_elems, np.float32)
    v = np.empty(n_elems, np.float32)
    for i in range(n_elems):
        # float32 arithmetic as in the C++ driver: (float(rand()) / RAND_MAX - 0.5f) * 0.2f
        q[i] = (np.float32(libc.rand()) / np.float32(rand_max) - np.float32(0.5)) * np.float32(0.2)
        k[i] = (np.float32(libc.rand()) / np.float32(rand_max) - np.float32(0.5)) * np.float32(0.2)
        v[i] = (np.float32(libc.rand()) / np.float32(rand_max) - np.float32(0.5)) * np.float32(0.2)
    return q, k, v


def lse64(q, k, scale, causal):
    q = q.astype(np.float64)
    k = k.astype(np.float64)
    s = np.einsum("bhid,bhjd->bhij", q, k) * scale
    if causal:
        n = s.shape[-1]
        s = np.where(np.triu(np.ones((n, n), bool), 1), -np.inf, s)
    m = s.max(-1, keepdims=True)
    return (m[..., 0] + np.log(np.exp(s - m).sum(-1))).astype(np.float64)


def to_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def save_case(name, q, k, v, scale, causal, dtype_name, bits=None):
    o = orc.ref_attention_direct(q, k, v, scale, causal)
    payload = {"o_ref": o, "lse64": lse64(q, k, scale, causal), "scale": np.float32(scale),
               "causal": np.int32(causal)}
    if bits is not None:
        payload.update({"q_bits": bits[0], "k_bits": bits[1], "v_bits": bits[2]})
    else:
        payload.update({"q": q, "k": k, "v": v})
    np.savez_compressed(HERE / f"{name}.npz", **payload)
    return {"file": f"{name}.npz", "shape": list(q.shape), "dtype": dtype_name, "scale": float(scale),
            "causal": bool(causal)}


def torch_case(name, q, k, v, scale, causal):
    dname = {torch.float16: "float16", torch.bfloat16: "bfloat16"}[q.dtype]
    return save_case(name, q.float().numpy(), k.float().numpy(), v.float().numpy(), scale, causal, dname,
                     bits=(to_bits(q), to_bits(k), to_bits(v)))


def main():
    if not orc.ref_available():
        raise SystemExit("oracle/_ref/libref_attention.so missing: run `make -C oracle` with the reference tree")
    manifest = {"generator": "tests/golden/make_golden.py",
                "source": "benchmark/cpp/correctness_v6.cu:23-72 (cpu_reference_attention), built in place",
                "cases": {}}
    cases = manifest["cases"]

    qf, kf, vf = glibc_rand_inputs(64 * 128, 17)
    shape = (1, 1, 64, 128)
    cases["ref_v6_case"] = save_case("ref_v6_case", qf.reshape(shape), kf.reshape(shape), vf.reshape(shape),
                                     1.0 / math.sqrt(128.0), False, "float32")

    cfg = CONFIGS["cfg0"]
    q, k, v = generate(cfg)
    cases["cfg0_head0"] = torch_case("cfg0_head0", q[:, :1], k[:, :1], v[:, :1], cfg.scale, False)
    full = orc.ref_attention_direct(q.float().numpy(), k.float().numpy(), v.float().numpy(), cfg.scale, False)
    manifest["cfg0_full_o_sha256"] = hashlib.sha256(np.ascontiguousarray(full).tobytes()).hexdigest()

    q, k, v = make_random((1, 1, 200, 64), torch.bfloat16, seed=31)
    cases["causal_tail"] = torch_case("causal_tail", q, k, v, 0.125, True)

    oc = AttnConfig("outlier_small", 1, 2, 256, 32, torch.float16, False, 4, outliers=True)
    q, k, v = generate(oc)
    cases["outlier_d32"] = torch_case("outlier_d32", q, k, v, oc.scale, False)

    q, k, v = make_stress((1, 1, 128, 64), torch.float16, seed=11)
    cases["stress"] = torch_case("stress", q, k, v, 0.125, False)

    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
