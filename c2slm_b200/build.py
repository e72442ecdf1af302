"""Builds libc2slm_b200.so (sm_100a) in-tree with nvcc.

python -m c2slm_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libc2slm_b200.so")
SOURCES = [os.path.join(HERE, "csrc", "c2s_engine.cu")]
DEPS = SOURCES + [os.path.join(HERE, "csrc", f) for f in ("c2s_device.cuh", "c2s_rows.cuh", "c2s_kernels.cuh", "c2s_persistent.cuh")] + \
    [os.path.join(ROOT, "include", "c2slm_b200.h")]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_cmd(out: str = LIB, extra: list[str] | None = None) -> list[str]:
    return [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
            "-Xcompiler", "-fPIC,-O2", "-shared", "-o", out, *SOURCES, "-lcudart", *(extra or [])]


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if force or needs_build():
        cmd = nvcc_cmd(extra=["-Xptxas", "-v"] if verbose else None)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc failed building libc2slm_b200.so")
        if verbose:
            sys.stderr.write(r.stderr)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB)
