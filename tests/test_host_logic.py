"""Host logic of the library on the CPU: the C++ host files are compiled
with host stand-ins for the CUDA runtime (tests/cuda_host_stubs.h) and the
kernel launchers, and checked through their own functions and the C ABI.

* tests/host_plan_check.cpp: every decode plan of random batches (windows of
  eng/mod.rs:10-36, rows covered once per task, 64-row cuts, disjoint
  partial slots, the persistent-CTA table and its longest-first balance).
* tests/host_model_check.cpp: the decoder's steps for prompts
  (g4a_model_prefill's chunks, rows, positions, head rows; one position per
  chunk as decode steps; rejected calls launch nothing) and for generate
  with eos ids (generate.rs:58-60)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "gemma4-rs_b200" / "csrc"
CUDA_INC = Path("/usr/local/cuda/include")


def build_and_run(tmp_path, sources):
    gxx = shutil.which("g++")
    if not gxx or not (CUDA_INC / "cuda_runtime.h").exists():
        pytest.skip("g++ or the CUDA headers are not available")
    exe = tmp_path / "check"
    subprocess.run([gxx, "-O1", "-std=c++17", "-w", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{ROOT / 'tests'}",
                    f"-I{CUDA_INC}", *map(str, sources), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.startswith("ok"), out.stdout + out.stderr


def test_decode_plans(tmp_path):
    build_and_run(tmp_path, [ROOT / "tests" / "host_plan_check.cpp"])


def test_decoder_steps(tmp_path):
    build_and_run(tmp_path, [ROOT / "tests" / "host_model_check.cpp", CSRC / "g4attn_host.cpp",
                             CSRC / "model_host.cpp"])
