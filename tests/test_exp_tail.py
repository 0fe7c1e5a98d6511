"""exp_tail (csrc/c4s_exp.cuh), the double exponential of the list kernel's
exact tail sums, compiled for the host and checked against long-double expl:
relative error below 2^-51 over (-700, 0], the bound behind the tail error
(2^-50 of the tail) that a refinement hands to the top-p decision."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_exp_tail_error_bound(tmp_path):
    exe = tmp_path / "test_exp_tail"
    src = os.path.join(HERE, "cpp", "test_exp_tail.cpp")
    subprocess.run(["g++", "-O2", "-std=c++17", "-o", str(exe), src], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
