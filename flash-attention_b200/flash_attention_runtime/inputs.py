"""Seeded synthetic Q/K/V for the benchmark and parity configurations.

Restates the reference's input generators (benchmark/python/input_data.py:25-60:
``random``, ``structured``, ``stress``) and adds the named configurations the
performance targets are quoted on.  Everything is drawn on the CPU with
``torch.Generator('cpu')`` so inputs do not depend on the GPU box; the reference
drew on the device with per-case seed offsets (input_data.py:11-30), this module
uses fixed seeds per configuration instead.

Draw order per configuration: Q, then K, then V with ``torch.randn`` in fp32;
for the outlier sweep the same generator then draws ``rand < 0.01`` masks for
Q and then K and multiplies the selected entries by 20; finally all three are
rounded to the configuration's dtype.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass(frozen=True)
class AttnConfig:
    name: str
    batch: int
    heads: int
    seq_len: int
    head_dim: int
    dtype: torch.dtype
    causal: bool
    seed: int
    outliers: bool = False

    @property
    def shape(self):
        return (self.batch, self.heads, self.seq_len, self.head_dim)

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    @property
    def slices(self) -> int:
        return self.batch * self.heads

    def flops(self, slices: Optional[int] = None) -> float:
        """Algorithmic FLOPs 4*B*H*N^2*d, halved for causal (per forward, or per `slices` slices)."""
        s = self.slices if slices is None else slices
        f = 4.0 * s * self.seq_len * self.seq_len * self.head_dim
        return f / 2 if self.causal else f

    def hbm_bytes(self, slices: Optional[int] = None, lse: bool = True) -> int:
        """Compulsory HBM traffic: read Q, K, V and write O (+ fp32 LSE)."""
        s = self.slices if slices is None else slices
        per = self.seq_len * self.head_dim * 2
        return s * (4 * per + (4 * self.seq_len if lse else 0))


# The configurations of the performance targets: 0 is the CPU-runnable
# correctness case, 2 the headline (1 GPU and sharded 2/4/8), 4 a head-dim sweep.
CONFIGS = {
    "cfg0": AttnConfig("cfg0", 1, 4, 256, 64, torch.float16, False, 0),
    "cfg1": AttnConfig("cfg1", 4, 16, 1024, 64, torch.float16, False, 1),
    "cfg2": AttnConfig("cfg2", 8, 32, 4096, 128, torch.bfloat16, True, 2),
    "cfg3": AttnConfig("cfg3", 2, 32, 16384, 128, torch.bfloat16, True, 3),
    "cfg4_d32": AttnConfig("cfg4_d32", 16, 16, 2048, 32, torch.float16, False, 4, outliers=True),
    "cfg4_d64": AttnConfig("cfg4_d64", 16, 16, 2048, 64, torch.float16, False, 4, outliers=True),
    "cfg4_d128": AttnConfig("cfg4_d128", 16, 16, 2048, 128, torch.float16, False, 4, outliers=True),
    # fp16 non-causal companion of configuration 2: the largest of these shapes the
    # reference's own GPU kernel supports (fp16, d = 128, non-causal, N % 64 == 0).
    "cfg2_f16nc": AttnConfig("cfg2_f16nc", 8, 32, 4096, 128, torch.float16, False, 2),
}


def generate(cfg: AttnConfig, batch: Optional[int] = None, seed_offset: int = 0):
    """CPU tensors (q, k, v) of cfg.dtype for cfg (optionally with another batch size)."""
    shape = (cfg.batch if batch is None else batch, cfg.heads, cfg.seq_len, cfg.head_dim)
    g = torch.Generator(device="cpu")
    g.manual_seed(cfg.seed + seed_offset)
    q = torch.randn(shape, dtype=torch.float32, generator=g)
    k = torch.randn(shape, dtype=torch.float32, generator=g)
    v = torch.randn(shape, dtype=torch.float32, generator=g)
    if cfg.outliers:
        qm = torch.rand(shape, generator=g) < 0.01
        km = torch.rand(shape, generator=g) < 0.01
        q = torch.where(qm, q * 20.0, q)
        k = torch.where(km, k * 20.0, k)
    return q.to(cfg.dtype), k.to(cfg.dtype), v.to(cfg.dtype)


def make_random(shape, dtype, seed: int):
    """Reference ``random`` mode (input_data.py:25-30), drawn on the CPU."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return tuple(torch.randn(shape, dtype=torch.float32, generator=g).to(dtype) for _ in range(3))


def make_structured(shape, dtype):
    """Reference ``structured`` mode (input_data.py:33-43): deterministic sin/cos."""
    b, h, n, d = shape
    bf = torch.arange(b, dtype=torch.float32).view(b, 1, 1, 1)
    hf = torch.arange(h, dtype=torch.float32).view(1, h, 1, 1)
    nf = torch.arange(n, dtype=torch.float32).view(1, 1, n, 1)
    df = torch.arange(d, dtype=torch.float32).view(1, 1, 1, d)
    q = torch.sin((nf + 1.0) * (hf + 1.0) / 17.0) + 0.01 * df + 0.05 * bf
    k = torch.cos((nf + 1.0) * (hf + 1.0) / 19.0) + 0.02 * df + 0.03 * bf
    v = torch.sin((df + 1.0) * (hf + 1.0) / 23.0) + 0.001 * nf + 0.02 * bf
    return q.to(dtype).contiguous(), k.to(dtype).contiguous(), v.to(dtype).contiguous()


def make_stress(shape, dtype, seed: int):
    """Reference ``stress`` mode (input_data.py:46-60): x32 / x16 scales plus 0.1% outliers."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    q = torch.randn(shape, dtype=torch.float32, generator=g) * 32.0
    k = torch.randn(shape, dtype=torch.float32, generator=g) * 32.0
    v = torch.randn(shape, dtype=torch.float32, generator=g) * 16.0
    qm = torch.rand(shape, generator=g) < 0.001
    km = torch.rand(shape, generator=g) < 0.001
    vm = torch.rand(shape, generator=g) < 0.001
    q = q + qm.to(torch.float32) * 256.0
    k = k - km.to(torch.float32) * 256.0
    v = v + vm.to(torch.float32) * 64.0
    return q.to(dtype).contiguous(), k.to(dtype).contiguous(), v.to(dtype).contiguous()
