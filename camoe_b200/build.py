"""Build the in-tree CUDA library camoe_b200/libcamoe_wkv7.so for sm_100a.

    python -m camoe_b200.build

nvcc cross-compiles without a GPU.  The library links the CUDA runtime
statically, so it loads with or without torch in the process.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libcamoe_wkv7.so")
GENCODE = "arch=compute_100a,code=sm_100a"


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def nvcc_command(out: str = LIB, extra: list[str] | None = None) -> list[str]:
    nvcc = os.environ.get("NVCC", "nvcc")
    return [nvcc, "-gencode", GENCODE, "-O3", "-lineinfo", "-std=c++17",
            "-Xcompiler", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"),
            *(extra or []), "-o", out, *sources()]


def up_to_date(out: str = LIB) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    deps = sources() + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = nvcc_command(extra=["-Xptxas", "-v"] if verbose else None)
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
