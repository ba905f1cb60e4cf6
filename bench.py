#!/usr/bin/env python3
"""Benchmark of the sm_100a FlashAttention-2 forward (the hot path) - driver contract.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg2] [--scaling strong|weak]

A step is one forward over one batch of synthetic seeded input (configuration 2
by default: B8 H32 N4096 d128 bf16 causal, the configuration the headline target
is quoted on), O and the logsumexp written.  Under torchrun each rank is one GPU.
By default ("strong") the configuration's B*H (batch, head) slices are split
across the ranks, rank r taking slices [r*S/N, (r+1)*S/N): the same total work at
every N, with no collective on the data path.  ("weak": every rank runs a full
batch of its own slices.)  Timing: W warm-up steps, then K steps between a
barrier + synchronize on each side, device time from CUDA events on the launching
stream, max over ranks.  `value` is the whole job's TFLOPS (all ranks' FLOPs over
the slowest rank's time); `per_gpu` is value / N.

After the timed region the ranks all-gather O and LSE (NCCL over NVLink) and rank
0 checks a strided set of slices of the gathered result against a float64
evaluation of softmax(scale * Q K^T [causal]) V on its GPU; the line carries the
result under `parity`, and a failed check makes the run exit non-zero.

`--impl reference` times the reference's own CPU attention
(benchmark/cpp/correctness_v6.cu:23-72, built from its sources into oracle/_ref)
on the host cores, one bounded sample of the same workload per step; it falls
back to the restated oracle port if oracle/_ref was not built.  With
`--ref-device gpu` it times the reference's own CUDA kernel instead, on the
workloads that kernel supports (fp16, d=128, non-causal: cfg4_d128, cfg2_f16nc).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "flash-attention_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from flash_attention_runtime.inputs import CONFIGS, AttnConfig  # noqa: E402

METRIC = ("attention fwd TFLOPS of the whole job over n_gpus (4*B*H*N^2*d/t, halved for causal); "
          "per_gpu = value/n_gpus, and % of dense bf16 peak in roofline")
REF_BUDGET_S = 150.0
E2E_BUDGET_S = 10.0   # the end-to-end leg runs min(--steps, what fits in this) steps
E2E_CHUNKS = 8            # at most; a chunk carries at least E2E_CHUNK_BYTES of Q+K+V
E2E_CHUNK_BYTES = 16 << 20
PRE_SPIN_CYCLES = 2_000_000  # GPU cycles the stream spins before the timed region (about 1 ms at 1965 MHz)
SUSTAINED_AFTER_S = 1.0  # timed regions at least this long are compared with the sustained peak
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
ATOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
LSE_RTOL = 1e-4


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # The default is a seconds-long run (the GPU settles at its power cap; the line
    # compares it with the sustained peak); the driver passes its own --steps.
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--verify-slices", type=int, default=8,
                    help="slices of the gathered output checked against float64 (0: no check)")
    ap.add_argument("--share-of", type=int, default=1,
                    help="on one GPU without torchrun: time rank 0's share of an N-way strong split "
                         "(to profile one rank's launch)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-device", choices=["cpu", "gpu"], default="cpu",
                    help="with --impl reference: gpu times the reference's own CUDA kernel instead "
                         "(fp16, d=128, non-causal workloads only, e.g. cfg4_d128 or cfg2_f16nc)")
    return ap.parse_args(argv)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def pick_peak(peaks: dict, timed_region_s: float):
    """Dense bf16 peak to divide by: the burst figure for a timed region shorter
    than SUSTAINED_AFTER_S (the GPU has not settled at its power cap yet), the
    sustained one for a seconds-long region."""
    if timed_region_s >= SUSTAINED_AFTER_S:
        return float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])), \
            "bf16_tflops_sustained"
    return float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])), "bf16_tflops"


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def check_slices(num_slices: int, count: int):
    """Slices 0 and S-1 plus evenly strided ones in between, `count` in all."""
    if count <= 0 or num_slices <= 0:
        return []
    if count >= num_slices:
        return list(range(num_slices))
    return sorted({round(i * (num_slices - 1) / (count - 1)) for i in range(count)} if count > 1 else {0})


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []  # (t, sm_mhz, max_mhz, reasons set)
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def wait_first_sample(self, timeout_s: float = 10.0):
        """Block until nvidia-smi has reported once (its NVML start-up is over), so
        that start-up does not overlap the timed region."""
        t_end = time.time() + timeout_s
        while self.proc is not None and not self.samples and time.time() < t_end and self.proc.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, mx = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
            reasons = {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}
            self.samples.append((time.time(), sm, mx, reasons))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0: float, t1: float):
        window = [s for s in self.samples if t0 <= s[0] <= t1]
        use = window if window else self.samples
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = sorted(set().union(*[s[3] for s in use]))
        return {"sm_mhz": statistics.median(s[1] for s in use), "sm_max_mhz": max(s[2] for s in use),
                "reasons": reasons, "samples": len(use), "in_timed_window": bool(window)}


# ----------------------------------------------------------------------------- CPU leg

def cpu_sample(cfg: AttnConfig, q: np.ndarray, k: np.ndarray, v: np.ndarray, threads: int, use_ref: bool):
    """Run the CPU attention on [1, S, N, d] float32 slices; returns (seconds, O)."""
    from oracle import oracle as orc

    t0 = time.perf_counter()
    if use_ref:
        o = orc.ref_attention(q, k, v, cfg.scale, cfg.causal, threads=threads)
    else:
        o, _ = orc.oracle_attention(q, k, v, cfg.scale, cfg.causal, threads=threads)
    return time.perf_counter() - t0, o


def cpu_inputs(cfg: AttnConfig, n_slices: int):
    """The first `n_slices` (b,h) slices of the workload's seeded inputs, as float32 numpy."""
    from flash_attention_runtime.inputs import generate

    q, k, v = generate(cfg)
    s = cfg.slices
    return tuple(t.reshape(1, s, cfg.seq_len, cfg.head_dim)[:, :n_slices].float().contiguous().numpy()
                 for t in (q, k, v))


def cpu_kind():
    from oracle import oracle as orc

    return orc.ref_available(), ("reference" if orc.ref_available() else "port")


def run_reference_gpu(args, cfg: AttnConfig):
    """The reference's own GPU forward (flash_attention_forward_v6_mma, mma.sync,
    through its pybind source compiled by oracle/build_ref_ext.py), timed like our
    arm on one GPU: inputs resident in HBM, W warm-up steps, K steps between
    synchronizes, CUDA events on the current stream."""
    from oracle import oracle as orc

    base = {"impl": "reference", "device": "gpu", "metric": METRIC, "unit": "TFLOPS", "higher_is_better": True,
            "config": workload_config(cfg, 1, "strong"),
            "kernel": "flash_attention_forward_v6_mma (src/forward/forward_v6_mma.cuh:325-412), mma.sync, sm_100"}
    why = None
    if cfg.dtype != torch.float16 or cfg.head_dim != 128 or cfg.causal or cfg.seq_len % 64:
        why = "the reference GPU kernel supports fp16, d=128, non-causal, N % 64 == 0 only"
    elif not torch.cuda.is_available():
        why = "no CUDA device"
    elif not orc.ref_gpu_available():
        why = f"{orc.REF_EXT_SO} not built (python oracle/build_ref_ext.py)"
    if why:
        print(json.dumps({**base, "unavailable": why}), flush=True)
        return
    from flash_attention_runtime.inputs import generate

    mod = orc.ref_gpu_module()
    dev = torch.device("cuda", 0)
    q, k, v = (x.to(dev) for x in generate(cfg))
    o = torch.empty_like(q)
    for _ in range(max(args.warmup, 3)):
        mod.forward(q, k, v, o, False)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        mod.forward(q, k, v, o, False)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    value = cfg.flops() / (ms * 1e-3) / 1e12
    print(json.dumps({**base, "value": value, "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
                      "ms_per_step": ms, "dtype": "f16", "data": "synthetic",
                      "l2": "inputs larger than L2 (126 MB); no flush needed"}), flush=True)


def run_reference_arm(args, cfg: AttnConfig):
    rank, world, _ = dist_env()
    if rank != 0:
        return  # the reference CPU path does not shard; rank 0 alone runs it
    if args.ref_device == "gpu":
        run_reference_gpu(args, cfg)
        return
    from oracle import oracle as orc

    use_ref, kind = cpu_kind()
    # one slice per host thread per step, at most the workload's own slice count
    threads = min(orc.host_threads(), cfg.slices)
    n_slices = threads
    q, k, v = cpu_inputs(cfg, n_slices)
    # A step takes seconds on the CPU: run at most three warm-up steps, and only
    # as many timed steps as fit in REF_BUDGET_S (the line reports the steps run).
    warm = min(args.warmup, 3)
    times = []
    for _ in range(warm):
        times.append(cpu_sample(cfg, q, k, v, threads, use_ref)[0])
    est = float(np.median(times)) if times else None
    steps = args.steps if est is None else max(1, min(args.steps, int(REF_BUDGET_S / max(est, 1e-3))))
    times = [cpu_sample(cfg, q, k, v, threads, use_ref)[0] for _ in range(steps)]
    t = float(np.mean(times))
    value = cfg.flops(n_slices) / t / 1e12
    sample = (f"{n_slices} of the {cfg.slices} (b,h) slices of {cfg.name} per step "
              f"(N={cfg.seq_len}, d={cfg.head_dim}, causal={cfg.causal}), one per host thread")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
        "steps": steps, "warmup": warm, "requested_steps": args.steps, "requested_warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(cfg, world, args.scaling),
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU leg

L2_BYTES = 126 * 2 ** 20


def rank_slices(cfg: AttnConfig, world: int, scaling: str) -> int:
    """Most (b,h) slices any rank holds."""
    return cfg.slices if scaling == "weak" else -(-cfg.slices // world)


def rank_bytes(cfg: AttnConfig, world: int, scaling: str) -> int:
    """Q, K, V and O bytes one rank holds."""
    return 4 * rank_slices(cfg, world, scaling) * cfg.seq_len * cfg.head_dim * 2


def input_copies(cfg: AttnConfig, world: int, scaling: str) -> int:
    """Copies of a rank's Q, K, V, O that consecutive timed launches rotate over, so
    that the launches between two uses of one copy move at least twice the L2
    through it: 1 when one copy is already that large."""
    b = rank_bytes(cfg, world, scaling)
    return 1 if b >= 2 * L2_BYTES else -(-2 * L2_BYTES // b) + 1


def l2_note(cfg: AttnConfig, world: int, scaling: str) -> str:
    mb = rank_bytes(cfg, world, scaling) / 1e6
    n = input_copies(cfg, world, scaling)
    if n > 1:
        return (f"launches back to back, rotating over {n} copies of the inputs and outputs "
                f"(Q+K+V+O {mb:.0f} MB per copy per rank, {n * mb:.0f} MB in all against the 126 MB L2): "
                f"the {n - 1} launches between two uses of a copy move {(n - 1) * mb:.0f} MB through L2")
    return f"launches back to back; inputs larger than L2 (Q+K+V+O per rank {mb:.0f} MB against 126 MB)"


def workload_config(cfg: AttnConfig, world: int, scaling: str):
    strong = scaling == "strong"
    return {
        "workload": cfg.name,
        "batch_per_rank": None if strong else cfg.batch,
        "global_batch": cfg.batch if strong else cfg.batch * world,
        "heads": cfg.heads, "seq_len": cfg.seq_len, "head_dim": cfg.head_dim, "causal": cfg.causal,
        "input_dtype": str(cfg.dtype).replace("torch.", ""),
        "slices": cfg.slices if strong else cfg.slices * world,
        "slices_per_rank": rank_slices(cfg, world, scaling),
        "parallelism": (f"bh-shard x{world}: rank r owns (b,h) slices [r*S/{world}, (r+1)*S/{world})" if strong
                        else f"bh-shard x{world}: every rank a full batch of its own slices"),
        "l2": l2_note(cfg, world, scaling),
        "lse": True,
    }


def rank_inputs(cfg: AttnConfig, rank: int, world: int, scaling: str):
    """This rank's Q, K, V (CPU, drawn seeded) as [1, S_r, N, d] for strong scaling
    or the full [B, H, N, d] of its own seed for weak; plus (full q, k, v or None,
    first slice index)."""
    from flash_attention_runtime.inputs import generate
    from flash_attention_runtime.sharding import slice_range

    if scaling == "weak":
        q, k, v = generate(cfg, seed_offset=1000 * rank)
        return (q, k, v), (q, k, v), 0
    q, k, v = generate(cfg)
    s = cfg.slices
    lo, hi = slice_range(s, rank, world)
    part = tuple(t.reshape(1, s, cfg.seq_len, cfg.head_dim)[:, lo:hi].contiguous() for t in (q, k, v))
    return part, (q, k, v), lo


def reference_slice(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool):
    """float64 softmax(scale * q k^T [causal]) v and its natural-log logsumexp, for
    one [N, d] slice on q's device: the checker for the gathered output."""
    qd, kd, vd = q.double(), k.double(), v.double()
    s = (qd @ kd.transpose(0, 1)) * scale
    if causal:
        n = s.shape[0]
        s.masked_fill_(torch.ones(n, n, dtype=torch.bool, device=s.device).triu_(1), float("-inf"))
    m = s.amax(dim=1, keepdim=True)
    p = torch.exp(s - m)
    l = p.sum(dim=1, keepdim=True)
    o = (p @ vd) / l
    return o, (m + torch.log(l)).squeeze(1)


def half_ulp(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Half the spacing of `dtype` numbers at |x| (normal range)."""
    mant = {torch.float16: 10, torch.bfloat16: 7}[dtype]
    e = torch.floor(torch.log2(x.abs().clamp(min=2.0 ** -14)))
    return torch.exp2(e - mant - 1)


def verify(cfg: AttnConfig, full, o_all: torch.Tensor, lse_all: torch.Tensor, slices, dev):
    """Check `slices` of the gathered O / LSE ([S, N, d] / [S, N]) against float64."""
    q, k, v = full  # the slices behind o_all, [B, H, N, d] or [S, N, d], on the CPU
    flat = lambda t: t.reshape(-1, cfg.seq_len, cfg.head_dim)  # noqa: E731
    qf, kf, vf = flat(q), flat(k), flat(v)
    atol = ATOL[cfg.dtype]
    max_abs = max_rounded = lse_rel = worst_excess = 0.0
    for i in slices:
        ro, rl = reference_slice(qf[i].to(dev), kf[i].to(dev), vf[i].to(dev), cfg.scale, cfg.causal)
        out = o_all[i].to(dev).double()
        err = (out - ro).abs()
        max_abs = max(max_abs, float(err.max()))
        max_rounded = max(max_rounded, float((out - ro.to(cfg.dtype).double()).abs().max()))
        worst_excess = max(worst_excess, float((err - atol - half_ulp(ro, cfg.dtype)).max()))
        lr = lse_all[i].to(dev).double()
        lse_rel = max(lse_rel, float(((lr - rl).abs() / rl.abs().clamp(min=1.0)).max()))
        del ro, rl, out, err
    finite = bool(torch.isfinite(o_all).all()) and bool(torch.isfinite(lse_all).all())
    return {
        "checker": "float64 softmax(scale*QK^T)V and logsumexp on rank 0's GPU",
        "slices": list(slices), "max_abs": max_abs, "max_abs_vs_ref_rounded_to_dtype": max_rounded,
        "bound": atol, "bound_rule": "|dO| <= bound + half an output ulp of the reference, per element",
        "worst_excess_over_bound": worst_excess, "lse_max_rel": lse_rel, "lse_bound": LSE_RTOL,
        "all_finite": finite,
        "ok": finite and worst_excess <= 0.0 and lse_rel <= LSE_RTOL,
    }


def run_ours(args, cfg: AttnConfig):
    import torch.distributed as dist

    import flash_attention_runtime as fa
    from flash_attention_runtime.sharding import gather

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        # Keep rank 0's stdout to the one JSON line: NCCL prints its version line on
        # stdout when its communicator is created (at NCCL_DEBUG=VERSION or INFO,
        # whatever the environment set), so the setup and a first barrier run with
        # file descriptor 1 pointed at stderr.
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            dist.barrier()
            torch.cuda.synchronize(dev)
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # --share-of N on a single process stands in for rank 0 of an N-way strong split
    share = args.share_of if (world == 1 and args.scaling == "strong" and args.share_of > 1) else 1
    split_world = world * share
    # nvidia-smi starts now and reports once before the device work begins: its
    # start-up on every rank at once, inside a timed region of a few milliseconds
    # (20 steps of one rank's share), would otherwise be timed with it.
    sampler = ClockSampler(local)
    sampler.start()
    (qh, kh, vh), full, first_slice = rank_inputs(cfg, rank, split_world, args.scaling)
    n_slices = qh.shape[0] * qh.shape[1]
    n_copies = input_copies(cfg, split_world, args.scaling)
    copies = []
    for _ in range(n_copies):
        q, k, v = qh.to(dev), kh.to(dev), vh.to(dev)
        copies.append((q, k, v, torch.empty_like(q), torch.empty(q.shape[:3], dtype=torch.float32, device=dev)))
    q, k, v, o, lse = copies[0]
    stream = torch.cuda.current_stream(dev)

    def step(i):
        cq, ck, cv, co, cl = copies[i % n_copies]
        fa.ext_forward(cq, ck, cv, co, False, cfg.scale, cfg.causal, cl)

    fa.reset_device_status(dev)
    sampler.wait_first_sample()
    warmup = max(args.warmup, 3)
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    # The stream first spins for about a millisecond, so that the host enqueues
    # the start event and the first launches while the GPU is busy: the timed
    # region then holds the K launches back to back, without the host's latency
    # to submit the first one (tens of microseconds through Python, against a
    # region of a few milliseconds for one rank's share).  Host costs are in e2e.
    torch.cuda._sleep(PRE_SPIN_CYCLES)
    start.record(stream)
    for i in range(args.steps):
        step(i)
    end.record(stream)
    torch.cuda.synchronize(dev)
    t_wall1 = time.time()
    barrier()
    # Launches run back to back: the average launch duration is the region's time
    # over the launch count.
    total_ms = start.elapsed_time(end)
    launch_ms = total_ms / args.steps
    sampler.stop()
    status = fa.device_status(dev)
    if status != 0:
        raise RuntimeError(f"kernel status 0x{status:x}")
    # every copy holds the same inputs, so copy 0's O and LSE stand for all of them
    del copies[1:]

    rank_ms = [total_ms / args.steps]
    if world > 1:
        t = torch.tensor([total_ms / args.steps], dtype=torch.float64, device=dev)
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        rank_ms = [float(x.item()) for x in parts]
    ms_per_step = max_over_ranks(total_ms / args.steps)
    launch_ms_max = max_over_ranks(launch_ms)
    flops_rank = cfg.flops(n_slices)
    total_flops = flops_rank * world if args.scaling == "weak" else cfg.flops() / share
    value = total_flops / (ms_per_step * 1e-3) / 1e12
    timed_region_s = ms_per_step * args.steps / 1e3

    # ---- verification: gather O and LSE (NCCL all-gather; local at one rank) and
    # check strided slices of the whole result against float64 on rank 0.
    parity = None
    if args.verify_slices > 0:
        s_total = cfg.slices  # strong: the whole configuration; weak: rank 0's own batch
        o_loc = o.reshape(1, n_slices, cfg.seq_len, cfg.head_dim)
        l_loc = lse.reshape(1, n_slices, cfg.seq_len)
        if share > 1:
            o_all, l_all = o_loc[0], l_loc[0]
            gathered = f"local (rank 0's share of a {share}-way split)"
        elif args.scaling == "strong" and world > 1:
            o_all = gather(o_loc, s_total)
            l_all = gather(l_loc, s_total)
            gathered = f"NCCL all_gather of O and LSE over {world} ranks"
        else:
            o_all, l_all = o_loc[0], l_loc[0]  # weak: each rank checks its own batch
            gathered = "local (one rank holds every slice)" if world == 1 else "local (weak scaling, rank 0's batch)"
        torch.cuda.synchronize(dev)
        if rank == 0:
            if share > 1:
                s_total = n_slices
                q_, k_, v_ = full
                cut = lambda t: t.reshape(cfg.slices, cfg.seq_len, cfg.head_dim)[:n_slices]  # noqa: E731
                full = (cut(q_), cut(k_), cut(v_))
            parity = verify(cfg, full, o_all, l_all, check_slices(s_total, args.verify_slices), dev)
            parity["gathered"] = gathered
        del o_all, l_all
        barrier()

    # ---- end to end through the public API: pinned host -> device, forward, device -> host.
    # The rank's slices go through in chunks so the upload of chunk c+1 (one copy
    # engine), the forward of chunk c and the download of chunk c-1 (the other copy
    # engine) overlap; only the last chunk's forward and download follow the uploads.
    # Up to E2E_CHUNKS chunks of at least E2E_CHUNK_BYTES of Q+K+V: 32 chunks measured
    # slower than 8 (five copies per chunk, each with its own set-up cost).  Events
    # keep buffer reuse across steps ordered.
    s_all = n_slices
    flat = lambda t: t.reshape(1, s_all, *t.shape[2:])  # noqa: E731
    qp, kp, vp = (flat(t).pin_memory() for t in (qh, kh, vh))
    op = torch.empty(qp.shape, dtype=qh.dtype).pin_memory()
    lp = torch.empty((1, s_all, qh.shape[2]), dtype=torch.float32).pin_memory()
    qd, kd, vd = torch.empty_like(flat(q)), torch.empty_like(flat(k)), torch.empty_like(flat(v))
    od = torch.empty_like(qd)
    ld = torch.empty((1, s_all, qh.shape[2]), dtype=torch.float32, device=dev)
    in_bytes = sum(t.numel() * t.element_size() for t in (qh, kh, vh))
    n_chunks = max(1, min(E2E_CHUNKS, s_all, in_bytes // E2E_CHUNK_BYTES))
    bounds = [(c * s_all // n_chunks, (c + 1) * s_all // n_chunks) for c in range(n_chunks)]
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in bounds]
    ev_fwd = [torch.cuda.Event() for _ in bounds]
    ev_out = [torch.cuda.Event() for _ in bounds]

    def e2e_step(start_event):
        up.wait_event(start_event)
        for c, (a, b) in enumerate(bounds):
            with torch.cuda.stream(up):
                up.wait_event(ev_fwd[c])  # previous step's forward of this chunk has read it
                qd[:, a:b].copy_(qp[:, a:b], non_blocking=True)
                kd[:, a:b].copy_(kp[:, a:b], non_blocking=True)
                vd[:, a:b].copy_(vp[:, a:b], non_blocking=True)
                ev_in[c].record(up)
            stream.wait_event(ev_in[c])
            stream.wait_event(ev_out[c])  # previous step's download of this chunk is done
            fa.ext_forward(qd[:, a:b], kd[:, a:b], vd[:, a:b], od[:, a:b], False, cfg.scale, cfg.causal,
                           ld[:, a:b])
            ev_fwd[c].record(stream)
            with torch.cuda.stream(down):
                down.wait_event(ev_fwd[c])
                op[:, a:b].copy_(od[:, a:b], non_blocking=True)
                lp[:, a:b].copy_(ld[:, a:b], non_blocking=True)
                ev_out[c].record(down)
        stream.wait_stream(down)

    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0.record(stream)
    e2e_step(w0)
    w1.record(stream)
    torch.cuda.synchronize(dev)
    warm_ms = max_over_ranks(w0.elapsed_time(w1))
    if args.e2e_steps is not None:
        e2e_steps = max(1, args.e2e_steps)
    else:
        e2e_steps = max(1, min(args.steps, int(E2E_BUDGET_S * 1e3 / max(warm_ms, 1e-3))))
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step(e0)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    e2e_value = total_flops / (e2e_ms * 1e-3) / 1e12
    h2d = sum(t.numel() * t.element_size() for t in (qh, kh, vh))
    e2e_ok = torch.equal(op.reshape(o.shape), o.cpu()) and torch.equal(lp.reshape(lse.shape), lse.cpu())
    d2h = op.numel() * op.element_size() + lp.numel() * lp.element_size()

    peaks, peak_src = load_peaks()
    peak, peak_key = pick_peak(peaks, timed_region_s)
    achieved = flops_rank / (launch_ms_max * 1e-3) / 1e12
    traffic = None
    tfile = ROOT / "profiles" / f"traffic_{cfg.name}.json"
    if tfile.exists():
        try:
            # per launch of the whole configuration; a rank's launch covers its share of the slices
            traffic = json.loads(tfile.read_text()).get("bytes_per_launch")
            if traffic is not None:
                traffic = traffic * n_slices / cfg.slices
        except (ValueError, OSError):
            traffic = None

    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            from oracle import oracle as orc

            use_ref, kind = cpu_kind()
            threads = min(orc.host_threads(), cfg.slices)
            n_cpu = max(1, threads)
            cq, ck, cv = cpu_inputs(cfg, n_cpu)
            secs, cpu_o = cpu_sample(cfg, cq, ck, cv, threads, use_ref)
            # The CPU leg ran the reference's own attention on the workload's first
            # slices: its output doubles as a check of the GPU output there.
            gpu_o = o.reshape(n_slices, cfg.seq_len, cfg.head_dim)[:n_cpu].float().cpu().numpy()
            cpu = {"value": cfg.flops(n_cpu) / secs / 1e12, "unit": "TFLOPS", "cores": threads, "kind": kind,
                   "sample": f"the first {n_cpu} (b,h) slices of {cfg.name} (N={cfg.seq_len}, d={cfg.head_dim}, "
                             f"causal={cfg.causal}), one per host thread, {secs:.1f} s",
                   "max_abs_vs_gpu": float(np.abs(gpu_o - cpu_o.reshape(gpu_o.shape)).max())}
        frac_burst = achieved / float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        frac_sust = achieved / float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        result = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "per_gpu": value / world, "n_gpus": world,
            "steps": args.steps, "warmup": warmup, "ms_per_step": ms_per_step, "rank_ms_per_step": rank_ms,
            "timed_region_s": timed_region_s,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": "bf16" if cfg.dtype == torch.bfloat16 else "f16",
            "data": "synthetic (seeded N(0,1), generated on CPU)",
            "config": {**workload_config(cfg, split_world, args.scaling), **({"share_of": share} if share > 1 else {})},
            "parity": parity,
            "e2e": {"value": e2e_value, "unit": "TFLOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms, "steps": e2e_steps, "chunks": n_chunks,
                    "matches_device_timed_output": e2e_ok},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": (f"{peak_src} {peak_key}: timed region {timed_region_s:.3f} s "
                                         f"({'at least' if peak_key.endswith('sustained') else 'under'} "
                                         f"{SUSTAINED_AFTER_S:.0f} s)"),
                         "frac_of_burst_peak": frac_burst, "frac_of_sustained_peak": frac_sust,
                         "kernel": "fa_fwd_sm100_kernel", "launch_ms": launch_ms_max,
                         "algorithmic_flops_per_launch": flops_rank,
                         "traffic_note": "ncu dram bytes of one whole-configuration launch, scaled by this "
                                         "rank's share of the slices"},
            "cpu_baseline": cpu,
            "clocks": sampler.summary(t_wall0, t_wall1),
            "gpu_launches": args.steps,
        }
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and parity is not None and not parity["ok"]:
        raise SystemExit(f"parity check failed: {parity}")
    return result


def main():
    args = parse_args()
    cfg = CONFIGS[args.workload]
    if args.impl == "reference":
        run_reference_arm(args, cfg)
        return
    run_ours(args, cfg)


if __name__ == "__main__":
    main()
