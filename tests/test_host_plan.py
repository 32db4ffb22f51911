"""The decode planner's host logic on the CPU: tests/host_plan_check.cpp
compiles gemma4-rs_b200/csrc/g4attn_host.cpp with host stand-ins for the
CUDA runtime and checks every plan of random batches (windows of
eng/mod.rs:10-36, rows covered once per task, 64-row cuts, disjoint partial
slots, the persistent-CTA table and its longest-first balance)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CUDA_INC = Path("/usr/local/cuda/include")


def test_decode_plans(tmp_path):
    gxx = shutil.which("g++")
    if not gxx or not (CUDA_INC / "cuda_runtime.h").exists():
        pytest.skip("g++ or the CUDA headers are not available")
    exe = tmp_path / "host_plan_check"
    subprocess.run([gxx, "-O1", "-std=c++17", "-w", f"-I{ROOT / 'include'}", f"-I{ROOT / 'gemma4-rs_b200' / 'csrc'}",
                    f"-I{CUDA_INC}", str(ROOT / "tests" / "host_plan_check.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.startswith("ok"), out.stdout + out.stderr
