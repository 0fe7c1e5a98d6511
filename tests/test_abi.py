"""The C-ABI library loads and exports what include/*.h declares (no GPU use)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import REPO, load_c4s

HEADERS = [os.path.join(REPO, "include", "c4s_sampling.h")]


def _declared(path):
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(c4s_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol():
    c4s = load_c4s()
    lib = c4s.library()
    names = []
    for h in HEADERS:
        names += _declared(h)
    assert "c4s_sample" in names and "c4s_create" in names
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", c4s.sampling.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    for n in names:
        assert re.search(rf"\bT {n}$", out, flags=re.M), n
    # the C++ drop-in with the reference's mangled signatures (t2s.h:82-89)
    for sym in ["_ZN2c43t2s8sampling11temperatureERSt6vectorIfSaIfEEf",
                "_ZN2c43t2s8sampling18repetition_penaltyERSt6vectorIfSaIfEERKS2_IiSaIiEEf",
                "_ZN2c43t2s8sampling5top_kERSt6vectorIfSaIfEEi",
                "_ZN2c43t2s8sampling5top_pERSt6vectorIfSaIfEEfi",
                "_ZN2c43t2s8sampling6argmaxERKSt6vectorIfSaIfEE"]:
        assert sym in out, sym


def test_params_struct_layout():
    wl = load_c4s().workloads
    assert wl.ROW_PARAMS_DTYPE.itemsize == 24
    assert [wl.ROW_PARAMS_DTYPE.fields[n][1] for n in wl.ROW_PARAMS_DTYPE.names] == [0, 4, 8, 12, 16, 20]


def test_host_validation_without_device():
    lib = load_c4s().library()
    assert lib.c4s_version() == 1
    assert lib.c4s_status_string(-1) == b"invalid argument"
    # null context / bad arguments are rejected before any CUDA call
    assert lib.c4s_sample(None, None, 1, 8194, 8194, None, None, 0, None, 0, None, None, None, None, 0,
                          None) == -1
    assert lib.c4s_process(None, None, 1, 8194, 8194, None, None, 0, None, 0, 15, None) == -1
    assert lib.c4s_argmax(None, None, 1, 8194, 8194, None, None) == -1
    assert lib.c4s_destroy(None) == -1
    assert lib.c4s_set_debug(None, 0) == -1
    assert lib.c4s_seed_states(None, 4, 0, 0, None) == -1
    h = C.c_void_p()
    assert lib.c4s_create(C.byref(h), 10**6, 0) == -1      # above the shared-memory limit
    assert lib.c4s_create(C.byref(h), 0, 0) == -1
    assert lib.c4s_create(None, 8194, 0) == -1
    assert lib.c4s_create_sized(C.byref(h), 8194, 0, 0) == -1   # max_rows < 1
    assert lib.c4s_create_sized(C.byref(h), 0, 16, 0) == -1


def test_no_device_fails_loudly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    c4s = load_c4s()
    lib = c4s.library()
    h = C.c_void_p()
    assert lib.c4s_create(C.byref(h), 8194, 0) == -2
    with pytest.raises(Exception):
        c4s.top_k(np.zeros(16, np.float32), 3)
