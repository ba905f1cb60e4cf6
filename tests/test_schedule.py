"""CPU tests of the work-unit schedule (csrc/schedule.h), compiled for the host.

The kernel replaces the reference's grid of one CTA per 64-row query tile
(src/forward/forward_v6_mma.cuh:325-412, grid (N/64, H, B)) by persistent CTAs
that take 256-row units from an atomic counter; these tests check that the
counter order covers every (batch, head, unit) exactly once, with the key-block
counts the masks need, in the intended order.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "flash-attention_b200" / "csrc"


class Plan(ctypes.Structure):
    _fields_ = [("n_pairs", ctypes.c_int), ("n_kv", ctypes.c_int), ("num_tiles", ctypes.c_int),
                ("group_bh", ctypes.c_int), ("grid", ctypes.c_int)]


class Tile(ctypes.Structure):
    _fields_ = [("b", ctypes.c_int), ("h", ctypes.c_int), ("pair", ctypes.c_int), ("n0", ctypes.c_int),
                ("n1", ctypes.c_int)]


@pytest.fixture(scope="module")
def sched(tmp_path_factory):
    d = tmp_path_factory.mktemp("sched")
    src = d / "probe.cpp"
    src.write_text(
        '#include "schedule.h"\n'
        'extern "C" {\n'
        "fa::SchedPlan s_plan(int b, int h, int n, int d, int kb, int sms, int causal)"
        " { return fa::plan_schedule(b, h, n, d, kb, sms, causal != 0); }\n"
        "fa::TileInfo s_decode(int t, int b, int h, int n, int np, int nkv, int g, int kb, int causal)"
        " { return fa::decode_unit(t, b, h, n, np, nkv, g, kb, causal != 0); }\n"
        "}\n")
    so = d / "probe.so"
    subprocess.run(["g++", "-O1", "-std=c++17", "-shared", "-fPIC", f"-I{CSRC}", str(src), "-o", str(so)], check=True)
    lib = ctypes.CDLL(str(so))
    lib.s_plan.restype = Plan
    lib.s_plan.argtypes = [ctypes.c_int] * 7
    lib.s_decode.restype = Tile
    lib.s_decode.argtypes = [ctypes.c_int] * 9
    return lib


KEY_BLOCK = 128  # kBlockN of the kernel


def _cdiv(a, b):
    return -(-a // b)


@pytest.mark.parametrize("b,h,n", [(8, 32, 4096), (2, 32, 16384), (16, 16, 2048), (4, 16, 1024), (1, 4, 256),
                                   (2, 100, 100), (3, 7, 1000), (1, 1, 1), (1, 200, 129), (5, 3, 777)])
@pytest.mark.parametrize("causal", [False, True])
def test_units_cover_every_slice_pair_once(sched, b, h, n, causal):
    sms = 148
    p = sched.s_plan(b, h, n, 128, KEY_BLOCK, sms, int(causal))
    assert p.n_pairs == _cdiv(n, 256) and p.n_kv == _cdiv(n, KEY_BLOCK)
    assert p.num_tiles == b * h * p.n_pairs
    assert p.grid == min(p.num_tiles, sms)
    assert 1 <= p.group_bh <= b * h
    seen = set()
    for t in range(p.num_tiles):
        u = sched.s_decode(t, b, h, n, p.n_pairs, p.n_kv, p.group_bh, KEY_BLOCK, int(causal))
        assert 0 <= u.b < b and 0 <= u.h < h and 0 <= u.pair < p.n_pairs
        key = (u.b, u.h, u.pair)
        assert key not in seen
        seen.add(key)
        # key blocks: everything for non-causal, up to the tile's last row for causal
        q0_end = u.pair * 256 + 128
        exp0 = min(_cdiv(q0_end, KEY_BLOCK), p.n_kv) if causal else p.n_kv
        exp1 = 0 if q0_end >= n else (min(_cdiv(q0_end + 128, KEY_BLOCK), p.n_kv) if causal else p.n_kv)
        assert (u.n0, u.n1) == (exp0, exp1)
        assert u.n0 >= 1 and (u.n1 == 0 or u.n1 >= u.n0)
    assert len(seen) == b * h * p.n_pairs


@pytest.mark.parametrize("causal", [False, True])
def test_order_groups_slices_and_puts_heavy_causal_units_first(sched, causal):
    b, h, n, sms = 8, 32, 4096, 148
    p = sched.s_plan(b, h, n, 128, KEY_BLOCK, sms, int(causal))
    units = [sched.s_decode(t, b, h, n, p.n_pairs, p.n_kv, p.group_bh, KEY_BLOCK, int(causal))
             for t in range(p.num_tiles)]
    per_group = p.group_bh * p.n_pairs
    for g0 in range(0, p.num_tiles, per_group):
        grp = units[g0:g0 + per_group]
        slices = {(u.b, u.h) for u in grp}
        assert len(slices) <= p.group_bh  # a group touches only its own slices
        work = [u.n0 + u.n1 for u in grp]
        if causal:
            assert work == sorted(work, reverse=True)  # heaviest first
        else:
            assert len(set(work)) == 1


def test_causal_groups_fit_the_l2_budget_and_are_balanced(sched):
    budget = 64 << 20  # kL2GroupBytes
    for b, h, n, d in [(8, 32, 4096, 128), (2, 32, 16384, 128), (16, 16, 2048, 32), (1, 32, 4096, 128),
                       (1, 8, 16384, 128), (3, 7, 1000, 64), (1, 200, 129, 128)]:
        p = sched.s_plan(b, h, n, d, KEY_BLOCK, 148, 1)
        bh = b * h
        kv = 4 * n * d  # K and V bytes of one slice
        wave = _cdiv(148, p.n_pairs)
        groups = _cdiv(bh, p.group_bh)
        if p.group_bh > min(wave, bh):
            assert p.group_bh * kv <= budget + kv  # within one slice of the budget (balanced rounding)
        # groups differ by at most the rounding of an even split
        assert p.group_bh == max(min(wave, bh), _cdiv(bh, max(1, _cdiv(bh * kv, budget))))
        assert groups * p.group_bh >= bh
    # the headline configuration: 8 groups of 32 slices (64 MB of K and V each);
    # a rank of an 8-way split of it (32 slices) is one group
    assert sched.s_plan(8, 32, 4096, 128, KEY_BLOCK, 148, 1).group_bh == 32
    assert sched.s_plan(1, 32, 4096, 128, KEY_BLOCK, 148, 1).group_bh == 32
    p = sched.s_plan(1, 1, 4096, 128, KEY_BLOCK, 148, 1)
    assert p.group_bh == 1 and p.grid == 16


def test_non_causal_groups_are_one_wave(sched):
    # equal-cost units: a group is about one unit per SM
    p = sched.s_plan(16, 16, 2048, 128, KEY_BLOCK, 148, 0)
    assert p.n_pairs == 8 and p.group_bh == 19
    p = sched.s_plan(4, 16, 1024, 64, KEY_BLOCK, 148, 0)
    assert p.group_bh == 37
    p = sched.s_plan(8, 32, 4096, 128, KEY_BLOCK, 148, 0)
    assert p.group_bh == 10


def _makespan(units, sms, cost):
    """List schedule of `units` in counter order on `sms` CTAs, each claiming its
    next unit when it becomes free (the kernel's late claim)."""
    import heapq

    heap = [(0.0, c) for c in range(sms)]
    end = 0.0
    for u in units:
        t, c = heapq.heappop(heap)
        t += cost(u)
        end = max(end, t)
        heapq.heappush(heap, (t, c))
    return end


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_causal_headline_share_is_balanced(sched, ranks):
    """One rank's share of configuration 2 (256 slices split over `ranks` GPUs):
    with the counter order and late claiming, the busiest CTA has at most a few
    percent more work than the average, in a model where a key block costs 2
    with both query tiles busy, 1.6 with one, and every unit 1 more."""
    b, h, n, sms = 1, 256 // ranks, 4096, 148
    p = sched.s_plan(b, h, n, 128, KEY_BLOCK, sms, 1)
    units = [sched.s_decode(t, b, h, n, p.n_pairs, p.n_kv, p.group_bh, KEY_BLOCK, 1) for t in range(p.num_tiles)]

    def cost(u):
        both = min(u.n0, u.n1)
        return 2.0 * both + 1.6 * (max(u.n0, u.n1) - both) + 1.0

    avg = sum(cost(u) for u in units) / sms
    assert avg / _makespan(units, sms, cost) >= (0.97 if ranks < 8 else 0.95)
