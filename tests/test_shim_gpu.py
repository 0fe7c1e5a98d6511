"""The reference's own sampling test (tests/test_sampling.cpp), as a C++
program linked against the drop-in shim with the c4::t2s::sampling
signatures, run on the GPU."""
import os
import subprocess

import pytest

from conftest import GOLDEN, REPO

pytestmark = pytest.mark.gpu
BIN = os.path.join(REPO, "tests", "cpp", "bin", "test_sampling_shim")


def test_reference_sampling_test_against_shim():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not os.path.exists(BIN):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "tests", "cpp")], check=True)
    r = subprocess.run([BIN, os.path.join(GOLDEN, "hf", "sampling")], capture_output=True, text=True,
                       timeout=120)
    print(r.stdout, r.stderr)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASSED" in r.stdout
