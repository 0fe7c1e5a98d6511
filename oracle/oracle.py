"""ctypes bindings for the CPU checkers of the T2S sampling stage.

TEST INFRASTRUCTURE ONLY. Imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product library.

Two checkers:
  * ``Oracle()``    -- oracle/_build/libc4s_oracle.so, the plain-C restatement
                       (c4s_oracle.c), built on demand with ``make``.
  * ``RefOracle()`` -- oracle/_ref/libc4s_ref.so, the reference's own
                       src/t2s/sampling.cpp compiled from source (present only
                       where the reference tree was available at build time).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libc4s_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libc4s_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build(ref_tree: str | None = None) -> None:
    """Build the C oracle (and, given the reference source tree, the
    reference checker)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref_tree:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref_tree}"], check=True)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class _Base:
    prefix = ""

    def __init__(self, path):
        self.lib = C.CDLL(path)
        P = self.prefix
        L = self.lib
        for name, args, res in [
            ("temperature", [C.c_void_p, C.c_int32, C.c_float], None),
            ("repetition_penalty", [C.c_void_p, C.c_int32, C.c_void_p, C.c_int64, C.c_float], None),
            ("top_k", [C.c_void_p, C.c_int32, C.c_int32], None),
            ("top_p", [C.c_void_p, C.c_int32, C.c_float, C.c_int32], None),
            ("argmax", [C.c_void_p, C.c_int32], C.c_int32),
            ("sample_batch", [C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_void_p,
                              C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p,
                              C.c_void_p, C.c_void_p, C.c_int64, C.c_int32], None),
        ]:
            f = getattr(L, P + name)
            f.argtypes = args
            f.restype = res

    # -- single-row processors, in place on a float32 numpy vector ----------
    def temperature(self, x: np.ndarray, t: float) -> None:
        getattr(self.lib, self.prefix + "temperature")(_ptr(x), x.size, t)

    def repetition_penalty(self, x: np.ndarray, hist, pen: float) -> None:
        h = np.ascontiguousarray(hist, dtype=np.int32)
        getattr(self.lib, self.prefix + "repetition_penalty")(_ptr(x), x.size, _ptr(h), h.size, pen)

    def top_k(self, x: np.ndarray, k: int) -> None:
        getattr(self.lib, self.prefix + "top_k")(_ptr(x), x.size, k)

    def top_p(self, x: np.ndarray, p: float, min_keep: int = 1) -> None:
        getattr(self.lib, self.prefix + "top_p")(_ptr(x), x.size, p, min_keep)

    def argmax(self, x: np.ndarray) -> int:
        return getattr(self.lib, self.prefix + "argmax")(_ptr(x), x.size)

    # -- batched sample step ------------------------------------------------
    def sample_batch(self, logits, V, hist, hist_off, params, rng, active=None,
                     want_logits=False, nthreads=1, params_stride=1):
        """Runs one step; advances ``rng`` in place. Returns (ids, logits|None)."""
        assert logits.dtype == np.float32 and logits.flags.c_contiguous
        assert rng.dtype == np.uint64 and rng.flags.c_contiguous
        B, ld = logits.shape
        ids = np.empty(B, dtype=np.int32)
        out = np.empty((B, V), dtype=np.float32) if want_logits else None
        hist = np.ascontiguousarray(hist, dtype=np.int32) if hist is not None else None
        hist_off = np.ascontiguousarray(hist_off, dtype=np.int64) if hist_off is not None else None
        act = None if active is None else np.ascontiguousarray(active, dtype=np.uint8)
        getattr(self.lib, self.prefix + "sample_batch")(
            _ptr(logits), B, V, ld, _ptr(hist), _ptr(hist_off), _ptr(params), params_stride,
            _ptr(rng), _ptr(act), _ptr(ids), _ptr(out), V, nthreads)
        return ids, out


class Oracle(_Base):
    """The plain-C restatement (c4s_oracle.c)."""
    prefix = "c4o_"

    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build()
        super().__init__(ORACLE_SO)
        L = self.lib
        L.c4o_draw.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
        L.c4o_draw.restype = C.c_int32
        L.c4o_top_p_info.argtypes = [C.c_void_p, C.c_int32, C.c_float, C.c_int32,
                                     C.c_void_p, C.c_void_p]
        L.c4o_seed_states.argtypes = [C.c_void_p, C.c_int32, C.c_uint64, C.c_int64]
        L.c4o_process_batch.argtypes = [C.c_void_p, C.c_int32, C.c_int32, C.c_int64,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                        C.c_int32, C.c_int32]
        L.c4o_argmax_batch.argtypes = [C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_void_p]

    def draw(self, x: np.ndarray, state: np.ndarray) -> int:
        return self.lib.c4o_draw(_ptr(x), x.size, _ptr(state))

    def top_p_info(self, x: np.ndarray, p: float, min_keep: int = 1):
        tie = C.c_int32(0)
        margin = C.c_double(0)
        self.lib.c4o_top_p_info(_ptr(x), x.size, p, min_keep, C.byref(tie), C.byref(margin))
        return bool(tie.value), margin.value

    def seed_states(self, B, seed, row_offset=0):
        s = np.empty(B, dtype=np.uint64)
        self.lib.c4o_seed_states(_ptr(s), B, seed, row_offset)
        return s

    def process_batch(self, logits, V, hist, hist_off, params, stages, nthreads=1,
                      params_stride=1):
        B, ld = logits.shape
        self.lib.c4o_process_batch(_ptr(logits), B, V, ld, _ptr(hist), _ptr(hist_off),
                                   _ptr(params), params_stride, stages, nthreads)

    def argmax_batch(self, logits, V):
        B, ld = logits.shape
        out = np.empty(B, dtype=np.int32)
        self.lib.c4o_argmax_batch(_ptr(logits), B, V, ld, _ptr(out))
        return out


class RefOracle(_Base):
    """The reference's own sampling.cpp (compiled from source) + restated draw."""
    prefix = "ref_"

    def __init__(self):
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO)
        super().__init__(REF_SO)

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)
