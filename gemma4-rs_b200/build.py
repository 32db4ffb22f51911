"""Builds libg4attn.so in-tree for sm_100a (B200) with nvcc.

The library is the product: the C ABI of include/g4attn.h over hand-written
CUDA kernels. It is built into gemma4-rs_b200/g4attn/ so that it travels with
the source tree; no JIT cache is involved.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OUT = HERE / "g4attn" / "libg4attn.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
         f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "g4attn.h"]
    if OUT.exists() and all(OUT.stat().st_mtime >= d.stat().st_mtime for d in deps) and not extra:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    objs = []
    build_dir = HERE / "_build"
    build_dir.mkdir(exist_ok=True)
    for s in srcs:
        o = build_dir / (s.name + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, *(extra or []), "-c", str(s), "-o", str(o)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(o))
    cmd = [NVCC, *ARCH, "-shared", "-o", str(OUT), *objs]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:] or None)
