"""CPU tests of the host-visible pieces: UMMA descriptor / swizzle bit math,
the C ABI (exports, struct layout, status codes, argument validation) and the
Python binding's input checks.  No kernel is launched here."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

import flash_attention_runtime as fa
from flash_attention_runtime import _lib

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "flash-attention_b200" / "csrc"
INCLUDE = ROOT / "include"


@pytest.fixture(scope="module")
def layout_lib(tmp_path_factory):
    """umma_layout.h compiled for the host with g++ into a probe library."""
    d = tmp_path_factory.mktemp("layout")
    src = d / "probe.cpp"
    src.write_text(
        '#include "umma_layout.h"\n'
        'extern "C" {\n'
        "unsigned long long p_smem_desc(unsigned a, unsigned l, unsigned s, unsigned t)"
        " { return fa::make_smem_desc(a, l, s, t); }\n"
        "unsigned long long p_kmajor(unsigned base, unsigned rows, unsigned sw, unsigned kk)"
        " { return fa::kmajor_desc(base, rows, sw, kk); }\n"
        "unsigned long long p_mnmajor(unsigned base, unsigned rows, unsigned sw, unsigned kk)"
        " { return fa::mnmajor_desc(base, rows, sw, kk); }\n"
        "unsigned p_idesc(int bf16, int m, int n, int am, int bm) { return fa::make_idesc_f16(bf16, m, n, am, bm); }\n"
        "unsigned p_tile_off(unsigned r, unsigned c, unsigned rows, unsigned sw)"
        " { return fa::tile_offset_bytes(r, c, rows, sw); }\n"
        "unsigned p_sw(int d) { return fa::swizzle_bytes(d); }\n"
        "}\n")
    so = d / "probe.so"
    subprocess.run(["g++", "-O1", "-std=c++17", "-shared", "-fPIC", f"-I{CSRC}", str(src), "-o", str(so)], check=True)
    lib = ctypes.CDLL(str(so))
    for name in ("p_smem_desc", "p_kmajor", "p_mnmajor"):
        getattr(lib, name).restype = ctypes.c_ulonglong
        getattr(lib, name).argtypes = [ctypes.c_uint] * 4
    lib.p_idesc.restype = ctypes.c_uint
    lib.p_idesc.argtypes = [ctypes.c_int] * 5
    lib.p_tile_off.restype = ctypes.c_uint
    lib.p_tile_off.argtypes = [ctypes.c_uint] * 4
    lib.p_sw.restype = ctypes.c_uint
    lib.p_sw.argtypes = [ctypes.c_int]
    return lib


def _field(x, lo, width):
    return (x >> lo) & ((1 << width) - 1)


def test_smem_descriptor_fields(layout_lib):
    desc = layout_lib.p_smem_desc(0x12340, 16384, 1024, 2)
    assert _field(desc, 0, 14) == 0x12340 >> 4
    assert _field(desc, 16, 14) == 16384 >> 4
    assert _field(desc, 32, 14) == 1024 >> 4
    assert _field(desc, 46, 2) == 1  # descriptor version for sm_100
    assert _field(desc, 49, 3) == 0  # base offset
    assert _field(desc, 52, 1) == 0  # LBO mode
    assert _field(desc, 61, 3) == 2  # 128B swizzle


@pytest.mark.parametrize("d", [32, 64, 128])
def test_kmajor_k_steps(layout_lib, d):
    """Step kk of the K loop starts 32 bytes further in the row, and jumps to the
    next column chunk (rows*SW bytes) every SW/32 steps."""
    sw = layout_lib.p_sw(d)
    assert sw == (64 if d == 32 else 128)
    base = 0x4000
    for kk in range(d // 16):
        desc = layout_lib.p_kmajor(base, 128, sw, kk)
        start = _field(desc, 0, 14) << 4
        assert start == base + (kk * 32 // sw) * 128 * sw + (kk * 32) % sw
        assert _field(desc, 32, 14) << 4 == 8 * sw
        assert _field(desc, 61, 3) == (2 if sw == 128 else 4)


@pytest.mark.parametrize("d", [32, 64, 128])
def test_mnmajor_v_steps(layout_lib, d):
    sw = layout_lib.p_sw(d)
    base = 0x8000
    for kk in range(8):
        desc = layout_lib.p_mnmajor(base, 128, sw, kk)
        assert _field(desc, 0, 14) << 4 == base + kk * 16 * sw
        assert _field(desc, 16, 14) << 4 == 128 * sw  # next SW/2-column chunk
        assert _field(desc, 32, 14) << 4 == 8 * sw    # next 8 rows


def test_instruction_descriptor(layout_lib):
    # bf16 x bf16 -> f32, M=128, N=128, both K-major (S = Q K^T)
    v = layout_lib.p_idesc(1, 128, 128, 0, 0)
    assert _field(v, 4, 2) == 1 and _field(v, 7, 3) == 1 and _field(v, 10, 3) == 1
    assert _field(v, 15, 1) == 0 and _field(v, 16, 1) == 0
    assert _field(v, 17, 6) == 128 >> 3 and _field(v, 24, 5) == 128 >> 4
    assert _field(v, 0, 4) == 0 and _field(v, 13, 2) == 0 and _field(v, 23, 1) == 0 and _field(v, 29, 3) == 0
    # f16, M=128, N=64, B MN-major (O += P V)
    v = layout_lib.p_idesc(0, 128, 64, 0, 1)
    assert _field(v, 7, 3) == 0 and _field(v, 10, 3) == 0 and _field(v, 16, 1) == 1
    assert _field(v, 17, 6) == 8


@pytest.mark.parametrize("sw,rows", [(128, 128), (64, 128)])
def test_tile_offsets_match_tma_swizzle(layout_lib, sw, rows):
    """tile_offset_bytes equals the TMA swizzle rule: within each 1024-byte (SW=128)
    or 512-byte (SW=64) atom, 16-byte chunk bits [4,7) XOR address bits [7,10)."""
    mask = 7 if sw == 128 else 3
    seen = set()
    for r in range(rows):
        for c in range(sw // 2):
            a = r * sw + c * 2
            expect = a ^ (((a >> 7) & mask) << 4)
            got = layout_lib.p_tile_off(r, c, rows, sw)
            assert got == expect
            seen.add(got)
    assert len(seen) == rows * sw // 2


def test_bank_conflict_free_rows(layout_lib):
    """The 8 rows of one atom put the same column chunk in 8 distinct 16-byte bank groups."""
    for c16 in range(8):
        banks = {(layout_lib.p_tile_off(r, c16 * 8, 128, 128) // 16) % 8 for r in range(8)}
        assert len(banks) == 8


# ------------------------------------------------------------------ C ABI

def _declared_symbols():
    names = []
    for h in INCLUDE.glob("*.h"):
        names += re.findall(r"FA_API\s+[\w\s\*]+?\b(fa_\w+)\s*\(", h.read_text())
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_symbols()
    assert set(_lib.EXPORTED_SYMBOLS) <= set(declared)
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(declared) <= exported


def test_params_struct_layout_matches_header(tmp_path):
    fields = [f[0] for f in _lib.FwdParams._fields_]
    prog = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "fa_sm100.h"', "int main(void) {",
             '  printf("sizeof %zu\\n", sizeof(fa_fwd_params));']
    lines += [f'  printf("{f} %zu\\n", offsetof(fa_fwd_params, {f}));' for f in fields]
    lines += ["  return 0;", "}"]
    prog.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", f"-I{INCLUDE}", str(prog), "-o", str(exe)], check=True)
    got = dict(ln.split() for ln in subprocess.run([str(exe)], capture_output=True, text=True,
                                                    check=True).stdout.splitlines())
    assert int(got["sizeof"]) == ctypes.sizeof(_lib.FwdParams)
    for f in fields:
        assert int(got[f]) == getattr(_lib.FwdParams, f).offset, f


def test_smem_bytes_and_status_strings():
    lib = _lib.load()
    for d in (32, 64, 128):
        for dt in (0, 1):
            n = lib.fa_fwd_smem_bytes(d, dt)
            assert 0 < n <= 227 * 1024
    assert lib.fa_fwd_smem_bytes(96, 0) == 0
    assert lib.fa_fwd_smem_bytes(64, 7) == 0
    assert lib.fa_fwd_workspace_bytes() >= 4
    assert lib.fa_status_string(0) == b"FA_OK"
    assert lib.fa_status_string(5) == b"FA_ERR_DEVICE_TIMEOUT"
    assert lib.fa_status_string(99) == b"FA_ERR_UNKNOWN"


def _good_params():
    p = _lib.FwdParams()
    p.Q, p.K, p.V, p.O = 0x10000, 0x20000, 0x30000, 0x40000
    for t in "qkvo":
        setattr(p, f"stride_seq_{t}", 64)
        setattr(p, f"stride_head_{t}", 64 * 256)
        setattr(p, f"stride_batch_{t}", 64 * 256 * 4)
    p.seq_len, p.heads, p.head_dim, p.batch = 256, 4, 64, 1
    p.softmax_scale = 0.125
    p.causal = 0
    p.dtype = _lib.FA_DTYPE_F16
    return p


@pytest.mark.parametrize("mutate,code", [
    (lambda p: setattr(p, "Q", None), _lib.FA_ERR_BAD_PARAM),
    (lambda p: setattr(p, "dtype", 5), _lib.FA_ERR_UNSUPPORTED),
    (lambda p: setattr(p, "head_dim", 96), _lib.FA_ERR_UNSUPPORTED),
    (lambda p: setattr(p, "seq_len", 0), _lib.FA_ERR_BAD_SHAPE),
    (lambda p: setattr(p, "heads", 0), _lib.FA_ERR_BAD_SHAPE),
    (lambda p: setattr(p, "softmax_scale", 0.0), _lib.FA_ERR_BAD_PARAM),
    (lambda p: setattr(p, "softmax_scale", float("nan")), _lib.FA_ERR_BAD_PARAM),
    (lambda p: setattr(p, "causal", 3), _lib.FA_ERR_BAD_PARAM),
    (lambda p: setattr(p, "K", 0x20008), _lib.FA_ERR_BAD_ALIGN),
    (lambda p: setattr(p, "stride_seq_v", 68), _lib.FA_ERR_BAD_ALIGN),
    (lambda p: setattr(p, "stride_seq_o", 32), _lib.FA_ERR_BAD_SHAPE),
    (lambda p: setattr(p, "LSE", 0x50002), _lib.FA_ERR_BAD_ALIGN),
])
def test_c_abi_rejects_bad_params_before_launch(mutate, code):
    lib = _lib.load()
    p = _good_params()
    mutate(p)
    assert lib.fa_fwd_sm100(ctypes.byref(p), None) == code
    assert lib.fa_last_error() != b""


def test_c_abi_null_params():
    lib = _lib.load()
    assert lib.fa_fwd_sm100(None, None) == _lib.FA_ERR_BAD_PARAM


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_c_abi_without_device_is_unsupported():
    lib = _lib.load()
    p = _good_params()
    assert lib.fa_fwd_sm100(ctypes.byref(p), None) == _lib.FA_ERR_UNSUPPORTED


# ------------------------------------------------------------------ Python binding checks (host side)

def test_binding_rejects_cpu_and_bad_inputs():
    q = torch.zeros(1, 2, 128, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        fa.forward(q, q, q)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        fa.forward_timed(q, q, q, causal=True)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        fa.ext_forward(q, q, q, None, False)
