"""c4s_sample_static: the entry point that allocates nothing (scratch in a
file-scope device array). Collected last; it must also pass on its own.

It is called through the C ABI and compared with c4s_sample (through a
context) on two sampling steps in a row: ids and advanced xorshift64 states
must be identical.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _bind(lib):
    f = lib.c4s_sample_static
    vp, i32, i64 = C.c_void_p, C.c_int32, C.c_int64
    f.argtypes = [vp, i32, i32, i64, vp, vp, i64, vp, i32, vp, vp, vp, vp]
    f.restype = C.c_int
    return f


def _static_step(f, b, rng_dev, dev):
    logits = torch.from_numpy(np.ascontiguousarray(b.logits)).to(dev)
    hist = torch.from_numpy(b.hist).to(dev)
    off = torch.from_numpy(b.hist_off).to(dev)
    params = torch.from_numpy(b.params.view(np.uint8).copy()).to(dev)
    ids = torch.empty(b.B, dtype=torch.int32, device=dev)
    rc = f(logits.data_ptr(), b.B, b.V, logits.stride(0), hist.data_ptr(), off.data_ptr(), int(hist.numel()),
           params.data_ptr(), 1, rng_dev.data_ptr(), None, ids.data_ptr(), None)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return ids.cpu().numpy()


@pytest.mark.gpu
def test_static_entry_matches_context_entry(c4s):
    wl = c4s.workloads
    dev = torch.device("cuda", 0)
    f = _bind(c4s.library())
    ctx = c4s.SamplingContext(max_vocab=8194, device=0)
    rng_s = torch.from_numpy(wl.config2(seed=21, B=256).rng.view(np.int64).copy()).to(dev)
    rng_c = rng_s.clone()
    for step in range(2):                       # two calls in a row, states carried over
        b = wl.config2(seed=21 + step, B=256)
        ids_s = _static_step(f, b, rng_s, dev)
        logits = torch.from_numpy(np.ascontiguousarray(b.logits)).to(dev)
        ids_c = ctx.sample(logits, torch.from_numpy(b.hist).to(dev), torch.from_numpy(b.hist_off).to(dev),
                           c4s.params_tensor(b.params, dev), rng_c)
        torch.cuda.synchronize()
        assert np.array_equal(ids_s, ids_c.cpu().numpy()), step
        assert torch.equal(rng_s, rng_c), step


@pytest.mark.gpu
def test_static_entry_matches_oracle(c4s, oracle):
    """Independently of the context path: the static entry point against the
    CPU oracle on two steps in a row (ids and states bit-exact)."""
    wl = c4s.workloads
    dev = torch.device("cuda", 0)
    f = _bind(c4s.library())
    rng_s = torch.from_numpy(wl.config2(seed=41, B=300).rng.view(np.int64).copy()).to(dev)
    ro = wl.config2(seed=41, B=300).rng.copy()
    for step in range(2):
        b = wl.config2(seed=41 + step, B=300)
        ids_s = _static_step(f, b, rng_s, dev)
        io, _ = oracle.sample_batch(np.ascontiguousarray(b.logits), b.V, b.hist, b.hist_off, b.params, ro,
                                    nthreads=8)
        assert np.array_equal(ids_s, io), step
        assert np.array_equal(rng_s.cpu().numpy().view(np.uint64), ro), step


@pytest.mark.gpu
def test_static_entry_rejects_oversized_rows(c4s):
    f = _bind(c4s.library())
    # V above the static scratch's capacity is refused before any launch
    assert f(None, 1, 16385, 16385, None, None, 0, None, 1, None, None, None, None) == -3
