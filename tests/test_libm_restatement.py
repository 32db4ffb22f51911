"""The device restatement of glibc's expf and tanhf (libm_glibc.cuh) against
this machine's C library, which the reference's f32::exp / f32::tanh and the
oracle call. The header compiles as plain C++ for this check; the same code
runs on the GPU in the decoder's softmax, GELU and soft-cap. A full sweep of
all 2^32 inputs found no difference; here a strided sweep (every exponent,
about a million inputs per function) keeps the check to a few seconds.
"""
import shutil
import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


def run_check(tmp_path, stride=4099):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path / "libm_check"
    subprocess.run([gxx, "-O2", "-std=c++17", "-ffp-contract=off", "-o", str(exe), str(HERE / "libm_check.cpp")],
                   check=True)
    out = subprocess.run([str(exe), str(stride)], capture_output=True, text=True)
    bad, checked = (int(v) for v in out.stdout.split())
    return bad, checked


def test_expf_tanhf_match_host_libm(tmp_path):
    bad, checked = run_check(tmp_path)
    assert checked > 2_000_000 and bad == 0, (bad, checked)
