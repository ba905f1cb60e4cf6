"""Tests of the (batch x head) sharding and the verification gather.

On CPU, two gloo ranks each take their slices of the same seeded inputs, run the
CPU oracle on them (standing in for the GPU kernel, whose per-slice results are
independent of the other slices) and all-gather O and LSE; the gathered result
must be bit-identical to the oracle over the whole batch.

On a box with two or more GPUs, two NCCL ranks run the kernel on their slices,
one GPU each, and all-gather O and LSE; the gathered result must match the
oracle within the parity tolerances.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_attention_runtime.sharding import gather, shard, slice_range

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (64, 8), (7, 3), (3, 4)])
def test_slice_ranges_partition(n, world):
    ranges = [slice_range(n, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert b == c
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_shard_is_contiguous_byte_range():
    t = torch.arange(2 * 3 * 4 * 8, dtype=torch.float32).reshape(2, 3, 4, 8)
    parts = [shard(t, r, 4) for r in range(4)]
    assert torch.equal(torch.cat([p[0] for p in parts]), t.reshape(6, 4, 8))
    with pytest.raises(ValueError):
        slice_range(10, 3, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    for p in (str(ROOT), str(ROOT / "flash-attention_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle.oracle import oracle_attention
    from flash_attention_runtime.inputs import make_random
    from flash_attention_runtime.sharding import gather as g, shard as sh

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = make_random((2, 3, 96, 32), torch.bfloat16, seed=12)
        s = 6
        o_loc, l_loc = oracle_attention(sh(q.float().contiguous(), rank, world).numpy(),
                                        sh(k.float().contiguous(), rank, world).numpy(),
                                        sh(v.float().contiguous(), rank, world).numpy(), 0.2, True, threads=1)
        o_all = g(torch.from_numpy(o_loc), s)
        l_all = g(torch.from_numpy(l_loc), s)
        if rank == 0:
            o_ref, l_ref = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), 0.2, True,
                                            threads=1)
            ok = np.array_equal(o_all.numpy(), o_ref.reshape(s, 96, 32)) and np.array_equal(
                l_all.numpy(), l_ref.reshape(s, 96))
            Path(result_path).write_text("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_shard_and_gather(tmp_path):
    out = tmp_path / "result.txt"
    mp.start_processes(_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True, start_method="spawn")
    assert out.read_text() == "ok"


def _gpu_worker(rank, world, port, result_path):
    for p in (str(ROOT), str(ROOT / "flash-attention_b200"), str(ROOT / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import flash_attention_runtime as fa
    from flash_attention_runtime.inputs import make_random
    from flash_attention_runtime.sharding import gather as g, shard as sh
    from oracle.oracle import oracle_attention
    from parity import compare_lse, compare_output

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        shape, scale = (2, 3, 300, 64), 0.125
        q, k, v = make_random(shape, torch.bfloat16, seed=14)
        s = shape[0] * shape[1]
        ql, kl, vl = (sh(t.contiguous(), rank, world).to(dev) for t in (q, k, v))
        o, lse = fa.forward(ql, kl, vl, softmax_scale=scale, causal=True, return_lse=True)
        o_all = g(o, s)
        l_all = g(lse, s)
        torch.cuda.synchronize(dev)
        if rank == 0:
            o_ref, l_ref = oracle_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale, True)
            ro = compare_output(o_all, o_ref.reshape(s, *shape[2:]), torch.bfloat16)
            rl = compare_lse(l_all, l_ref.reshape(s, shape[2]))
            Path(result_path).write_text("ok" if ro["ok"] and rl["ok"] else f"mismatch {ro} {rl}")
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_gpu_nccl_shard_and_gather(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = tmp_path / "result.txt"
    mp.start_processes(_gpu_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True, start_method="spawn")
    assert out.read_text() == "ok"
