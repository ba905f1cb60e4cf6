"""TEST INFRASTRUCTURE: builds the reference's own GPU forward for timing beside ours.

The reference binds its kernel `flash_attention_forward_v6_mma` (sm_80-style
mma.sync, src/forward/forward_v6_mma.cuh:325-412) through the pybind source
python/flash_attention_runtime/_ext.cu, which its package JIT-builds with
torch.utils.cpp_extension (python/flash_attention_runtime/__init__.py:10-27).
This script compiles that same source in place from the reference tree, with the
same flags, into oracle/_ref/ext/ (git-ignored; it travels to the GPU box with the
rest of oracle/_ref).  Only `bench.py --impl reference --ref-device gpu` loads
it, to time the reference kernel on the shapes it supports: fp16, d = 128,
non-causal, N % 64 == 0.  Nothing in the product path uses it.

Usage: python oracle/build_ref_ext.py <reference_root>   (or FA_REFERENCE_ROOT in the environment)
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "ext"
NAME = "fa_ref_v6"


def built_module_path() -> Path:
    return OUT / f"{NAME}.so"


def main(argv: list[str]) -> int:
    root = argv[1] if len(argv) > 1 else os.environ.get("FA_REFERENCE_ROOT", "")
    if not root:
        print("usage: build_ref_ext.py <reference_root> (or set FA_REFERENCE_ROOT); "
              f"keeping any prebuilt {built_module_path()}")
        return 0
    ref = Path(root)
    src = ref / "python" / "flash_attention_runtime" / "_ext.cu"
    if not src.exists():
        print(f"reference source {src} not found; keeping any prebuilt {built_module_path()}")
        return 0
    # The kernel is plain mma.sync; compile it for the B200 (compute capability 10.0).
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load

    OUT.mkdir(parents=True, exist_ok=True)
    load(
        name=NAME,
        sources=[str(src)],
        extra_include_paths=[str(ref)],
        extra_cflags=["-O3", "-std=c++20"],
        extra_cuda_cflags=["-O3", "--use_fast_math", "-lineinfo", "-std=c++20"],
        build_directory=str(OUT),
        verbose=False,
    )
    print(f"built {built_module_path()}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
