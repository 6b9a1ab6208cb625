"""CPU: the x87-precision arithmetic the GPU codebook builder uses for the
reference's long-double factors (csrc/bs_x87.hpp) against the host compiler's
own long double, on random, boundary and near-cancelling inputs."""
import os
import platform
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "beam_search_collab_b200", "csrc")
SRC = os.path.join(ROOT, "tests", "native", "x87_check.cpp")


@pytest.mark.skipif(platform.machine() != "x86_64", reason="long double is the x87 format only on x86-64")
def test_x87_emulation_matches_host_long_double(tmp_path):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    exe = str(tmp_path / "x87_check")
    subprocess.run([cxx, "-std=c++17", "-O2", "-I", CSRC, SRC, "-o", exe], check=True)
    r = subprocess.run([exe, "300000"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    bad, n = map(int, r.stdout.split()[-2:])
    assert bad == 0 and n > 800000
