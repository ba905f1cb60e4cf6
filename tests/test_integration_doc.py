"""Doc test: the binding examples of the repository's integration guide stay in
step with the header and the library.  The C++ driver snippet compiles against
include/fa_sm100.h, and the ctypes stub runs against libfa_sm100.so (here without
a GPU, so the call must return an error with a message instead of launching)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
DOC = (ROOT / "INTEGRATION.md").read_text()


def _block(lang: str, after: str) -> str:
    start = DOC.index(after)
    m = re.search(r"```" + lang + r"\n(.*?)```", DOC[start:], re.S)
    assert m, f"no {lang} block after {after!r}"
    return m.group(1)


def test_cpp_driver_snippet_compiles(tmp_path):
    body = _block("cpp", "## 4. C++ drivers")
    includes = [ln for ln in body.splitlines() if ln.startswith("#include")]
    code = [ln for ln in body.splitlines() if not ln.startswith("#include")]
    src = tmp_path / "driver.cpp"
    src.write_text("\n".join(["#include <cmath>", "#include <cstdio>", *includes,
                              "bool driver(void* dQ, void* dK, void* dV, void* dO, int B, int H, int N, int D) {",
                              *code, "  return true;", "}", ""]))
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", f"-I{ROOT / 'include'}", str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_ctypes_stub_runs_and_reports_errors():
    stub = _block("python", "## 3. ctypes stub")
    from flash_attention_runtime import _lib

    import torch

    if not _lib.LIB_PATH.exists():
        pytest.skip("libfa_sm100.so is not built")
    if torch.cuda.is_available():
        pytest.skip("runs the stub only where no kernel can launch")
    # Misaligned pointers as well: the C ABI rejects them before any launch.
    env = {"q_ptr": 0x10001, "k_ptr": 0x20001, "v_ptr": 0x30001, "o_ptr": 0x40001, "lse_ptr": None,
           "B": 1, "H": 2, "N": 128, "D": 64, "stream": 0}
    cwd = os.getcwd()
    os.chdir(ROOT)
    try:
        with pytest.raises(RuntimeError) as e:
            exec(compile(stub, "integration-guide-ctypes-stub", "exec"), env)  # noqa: S102
    finally:
        os.chdir(cwd)
    assert str(e.value)  # the library's own message, e.g. that no CUDA device is present
    assert isinstance(env["p"], _lib.FwdParams) and env["p"].head_dim == 64 and env["p"].causal == 1
