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

``generate_qkv`` is the reference callers' own generator interface
(benchmark/python/input_data.py:115-145): the same keyword arguments, draws on
the given device in the given dtype, and a per-case seed ``seed + 100003 *
case_index`` (input_data.py:11-12), so the reference's correctness gate and
benchmark loop run unchanged against this module.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from pathlib import Path
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


# ---------------------------------------------------------------------------
# The reference callers' generator (benchmark/python/input_data.py), drawn on a
# device.  Same modes and argument names; the formulas are the ones above.

_CASE_SEED_STRIDE = 100_003  # input_data.py:11-12


def case_seed(seed: int, case_index: int) -> int:
    """Seed of case `case_index` of a run with base seed `seed`."""
    return int(seed + case_index * _CASE_SEED_STRIDE)


def _device_gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _draw_random(shape, dtype, device, seed):
    g = _device_gen(seed, device)
    return tuple(torch.randn(shape, device=device, dtype=dtype, generator=g).contiguous() for _ in range(3))


def _draw_stress(shape, dtype, device, seed):
    g = _device_gen(seed, device)
    base = [torch.randn(shape, device=device, dtype=torch.float32, generator=g) * s for s in (32.0, 32.0, 16.0)]
    masks = [torch.rand(shape, device=device, generator=g) < 0.001 for _ in range(3)]
    q = base[0] + masks[0].to(torch.float32) * 256.0
    k = base[1] - masks[1].to(torch.float32) * 256.0
    v = base[2] + masks[2].to(torch.float32) * 64.0
    return tuple(t.to(dtype=dtype).contiguous() for t in (q, k, v))


def _load_replay(shape, dtype, device, replay_dir, replay_file):
    """q, k, v from a saved .pt (dict with q/k/v, or a 3-sequence); [B, N, H, d]
    tensors are permuted to [B, H, N, d] (input_data.py:65-112)."""
    replay_dir = Path(replay_dir) if replay_dir is not None else Path(".")
    if replay_file:
        path = Path(replay_file).expanduser()
        if not path.is_absolute():
            path = replay_dir / path
        if not path.exists():
            raise RuntimeError(f"Replay file not found: {path}")
    else:
        found = sorted(replay_dir.glob("*.pt"))
        if not found:
            raise RuntimeError(f"Replay mode selected but no .pt file found in: {replay_dir}")
        path = found[0]
    obj = torch.load(path, map_location="cpu")
    if isinstance(obj, dict) and all(key in obj for key in ("q", "k", "v")):
        tensors = (obj["q"], obj["k"], obj["v"])
    elif isinstance(obj, (list, tuple)) and len(obj) >= 3:
        tensors = tuple(obj[:3])
    else:
        raise RuntimeError("Replay file must be a dict(q,k,v) or tuple/list(q,k,v)")
    b, h, n, d = shape
    out = []
    for t in tensors:
        if tuple(t.shape) == (b, n, h, d) and (b, n, h, d) != tuple(shape):
            t = t.permute(0, 2, 1, 3)
        elif tuple(t.shape) != tuple(shape):
            raise RuntimeError(f"Replay tensor shape {tuple(t.shape)} does not match {tuple(shape)} or [B,N,H,D]")
        out.append(t.to(device=device, dtype=dtype).contiguous())
    return out[0], out[1], out[2], path


def generate_qkv(*, batch_size: int, n_heads: int, seq_len: int, d_head: int, dtype: torch.dtype, device,
                 input_mode: str, seed: int, case_index: int, replay_dir=None, replay_file: str = ""):
    """(q, k, v, replay_path) for one case of the reference's benchmark/correctness
    drivers: ``random``, ``structured``, ``stress`` or ``replay`` inputs of shape
    [batch_size, n_heads, seq_len, d_head] in `dtype` on `device`."""
    shape = (batch_size, n_heads, seq_len, d_head)
    seeded = case_seed(seed, case_index)
    if input_mode == "random":
        return (*_draw_random(shape, dtype, device, seeded), None)
    if input_mode == "structured":
        q, k, v = make_structured(shape, dtype)
        return q.to(device), k.to(device), v.to(device), None
    if input_mode == "stress":
        return (*_draw_stress(shape, dtype, device, seeded), None)
    if input_mode == "replay":
        return _load_replay(shape, dtype, device, replay_dir, replay_file)
    raise RuntimeError(f"Unsupported input_mode: {input_mode}")
