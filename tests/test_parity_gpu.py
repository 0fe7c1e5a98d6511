"""Parity of the CUDA sampling path with the oracle and the reference goldens.

Every comparison here is bit-exact: processed logits as uint32 bit patterns,
token ids and xorshift64 states as integers. All calls go through the C ABI
(libc4s.so) via the Python mirror of the reference interface.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_c4s
from helpers import bits, gpu_sample, oracle_sample, to_dev

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def c4s():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return load_c4s()


@pytest.fixture(scope="module")
def ctx(c4s):
    return c4s.SamplingContext(max_vocab=32768, device=0)


@pytest.fixture(scope="module")
def wl(c4s):
    return c4s.workloads


# ---------------------------------------------------------------------------
# The reference's own goldens, through the reference-named API.
# ---------------------------------------------------------------------------
def test_hf_goldens_through_reference_api(c4s):
    H = os.path.join(GOLDEN, "hf", "sampling")
    g = lambda n: np.load(os.path.join(H, n + ".npy")).astype(np.float32).ravel()
    base = g("logits")
    ids = np.load(os.path.join(H, "ids.npy")).ravel().tolist()
    for name, fn in [("temp", lambda v: c4s.temperature(v, 0.8)),
                     ("rep", lambda v: c4s.repetition_penalty(v, ids, 1.3)),
                     ("topk", lambda v: c4s.top_k(v, 10)),
                     ("topp", lambda v: c4s.top_p(v, 0.9))]:
        v = torch.from_numpy(base.copy()).cuda()
        fn(v)
        got = v.cpu().numpy()
        # tests/test_sampling.cpp:24-38 criteria, then bit equality
        assert np.array_equal(np.isneginf(got), np.isneginf(g(name))), name
        assert np.array_equal(bits(got), bits(g(name))), name
    # host containers are modified in place like the reference's std::vector
    lst = base.tolist()
    c4s.temperature(lst, 0.8)
    assert np.array_equal(bits(np.array(lst, np.float32)), bits(g("temp")))
    arr = base.copy()
    c4s.top_k(arr, 10)
    assert np.array_equal(bits(arr), bits(g("topk")))
    assert c4s.argmax(base.copy()) == int(np.argmax(base))


def test_processors_vs_reference_fixtures(c4s, oracle, golden_proc):
    """Each processor alone and the full chain, on the compiled-reference fixtures."""
    G = golden_proc
    X, meta, H, OFF = G["x"], G["meta"], G["hist"], G["hist_off"]
    ctx = c4s.default_context()
    stage_of = {"rep": c4s.STAGE_PENALTY, "temp": c4s.STAGE_TEMPERATURE, "topk": c4s.STAGE_TOP_K,
                "topp": c4s.STAGE_TOP_P, "chain": c4s.STAGE_ALL}
    wl = c4s.workloads
    for i in range(X.shape[0]):
        V, T, k, p, pen, mk = meta[i]
        V = int(V)
        x = X[i, :V].copy()
        hist = H[OFF[i]:OFF[i + 1]].astype(np.int32)
        P = wl.make_params(1, temperature=T, top_k=int(k), top_p=p, repetition_penalty=pen,
                           min_tokens_to_keep=int(mk))
        for key, st in stage_of.items():
            d = torch.from_numpy(x.reshape(1, -1).copy()).cuda()
            ctx.process(d, torch.from_numpy(hist).cuda(),
                        torch.tensor([0, hist.size], dtype=torch.int64).cuda(),
                        c4s.params_tensor(P, d.device), st)
            got = d.cpu().numpy()[0]
            # oracle (canonical tie order) must match bit for bit
            o = x.reshape(1, -1).copy()
            oracle.process_batch(o, V, hist, np.array([0, hist.size], np.int64), P, st)
            assert np.array_equal(bits(got), bits(o[0])), (i, key)
            ref = G[key][i, :V]
            if not np.array_equal(bits(got), bits(ref)):
                # only a top-p boundary inside a run of equal logits may differ
                assert key in ("topp", "chain"), (i, key)
                v = x.copy()
                if key == "chain":
                    oracle.repetition_penalty(v, hist, pen); oracle.temperature(v, T); oracle.top_k(v, int(k))
                tie, _ = oracle.top_p_info(v, p, int(mk))
                assert tie, (i, key)
        am = ctx.argmax(torch.from_numpy(x.reshape(1, -1).copy()).cuda())
        assert int(am.cpu()[0]) == G["argmax"][i]


def test_reference_chain_fixture(ctx, golden_chain, wl):
    """The compiled reference's c0 draws (48 steps, both modes) and a c2 batch."""
    G = golden_chain
    pool = G["c0_pool"]
    for mode in ("sample", "greedy"):
        params = wl.make_params(1, greedy=int(mode == "greedy"))
        rng = wl.seed_states(1, 0)
        hist, off = G["c0_hist0"].copy(), np.array([0, 256], np.int64)
        ids = []
        for s in range(48):
            b = wl.Batch(np.ascontiguousarray(pool[s % 16:s % 16 + 1]), 8194, hist, off, params, rng)
            t, rng, _ = gpu_sample(ctx, b, torch)
            ids.append(int(t[0]))
            hist, off = wl.append_history(hist, off, t)
        assert np.array_equal(np.array(ids, np.int32), G[f"c0_{mode}_ids"]), mode
        assert np.array_equal(rng, G[f"c0_{mode}_rng"]), mode
    params = G["c2_params"].reshape(-1).view(wl.ROW_PARAMS_DTYPE)
    b = wl.Batch(G["c2_logits"], 8194, G["c2_hist"], G["c2_hist_off"], params, G["c2_rng0"].copy())
    ids, rng, lg = gpu_sample(ctx, b, torch, want_logits=True)
    assert np.array_equal(ids, G["c2_ids"])
    assert np.array_equal(rng, G["c2_rng1"])
    assert np.array_equal(bits(lg), bits(G["c2_out"]))


# ---------------------------------------------------------------------------
# BASELINE configurations.
# ---------------------------------------------------------------------------
def _ar_loop(ctx, oracle, wl, b0, steps, pool_rows=32, seed=5):
    """Emulate the AR loop: per step a fresh logits row from a pool, the
    history grows by the sampled ids (text2semantic.cpp:168/:334)."""
    g = np.random.default_rng(seed)
    pool = wl.normal_logits(g, pool_rows * b0.B, b0.V, spikes=5).reshape(pool_rows, b0.B, b0.V)
    hist, off = b0.hist.copy(), b0.hist_off.copy()
    rg, ro = b0.rng.copy(), b0.rng.copy()
    mism = 0
    for s in range(steps):
        x = np.ascontiguousarray(pool[s % pool_rows])
        bg = wl.Batch(x, b0.V, hist, off, b0.params, rg)
        tg, rg, _ = gpu_sample(ctx, bg, torch)
        bo = wl.Batch(x, b0.V, hist, off, b0.params, ro)
        to, ro, _ = oracle_sample(oracle, bo)
        mism += int(np.sum(tg != to))
        assert np.array_equal(tg, to), (s, np.nonzero(tg != to))
        assert np.array_equal(rg, ro), s
        hist, off = wl.append_history(hist, off, tg)
    return mism


def test_config0_1000_steps_sample_and_greedy(ctx, oracle, wl):
    for greedy in (False, True):
        b = wl.config0(greedy=greedy)
        assert _ar_loop(ctx, oracle, wl, b, 1000, pool_rows=64) == 0


def test_config1_500_steps(ctx, oracle, wl):
    b = wl.config1()
    assert _ar_loop(ctx, oracle, wl, b, 500, pool_rows=8) == 0


def test_config2_full_batch(ctx, oracle, wl):
    """B=4096 heterogeneous rows: ids, states and processed logits bit-exact."""
    b = wl.config2(seed=2)
    ig, rg, lg = gpu_sample(ctx, b, torch, want_logits=True)
    io, ro, lo = oracle_sample(oracle, b, want_logits=True)
    bad = np.nonzero(ig != io)[0]
    assert bad.size == 0, bad[:10]
    assert np.array_equal(rg, ro)
    assert np.array_equal(bits(lg), bits(lo))
    # and a second step from the advanced states
    b2 = wl.config2(seed=3)
    b2.rng = rg.copy()
    ig2, rg2, _ = gpu_sample(ctx, b2, torch)
    b2.rng = ro.copy()
    io2, ro2, _ = oracle_sample(oracle, b2)
    assert np.array_equal(ig2, io2)
    assert np.array_equal(rg2, ro2)


def test_fused_path_config2(c4s, oracle, wl):
    """The fused kernel (the small-batch path) forced on the full config-2
    batch: ids, states and processed logits bit-exact."""
    ctx = c4s.SamplingContext(max_vocab=8194, device=0)
    ctx.set_debug(c4s.sampling.DEBUG_FUSED_PATH)
    b = wl.config2(seed=2)
    ig, rg, lg = gpu_sample(ctx, b, torch, want_logits=True)
    io, ro, lo = oracle_sample(oracle, b, want_logits=True)
    assert np.array_equal(ig, io), np.nonzero(ig != io)[0][:10]
    assert np.array_equal(rg, ro)
    assert np.array_equal(bits(lg), bits(lo))


@pytest.mark.parametrize("fused", [False, True])
def test_batch_of_three_chunks(c4s, oracle, wl, fused):
    """B = 8192 + 37 rows with ragged histories: three 4096-row chunks on the
    split path (each chunk offsets logits, history offsets, states and ids),
    one launch on the fused path; ids, states and processed logits bit-exact."""
    ctx = c4s.SamplingContext(max_vocab=8194, device=0)
    if fused:
        ctx.set_debug(c4s.sampling.DEBUG_FUSED_PATH)
    b = wl.config2(seed=31, B=8192 + 37)
    ig, rg, lg = gpu_sample(ctx, b, torch, want_logits=True)
    io, ro, lo = oracle_sample(oracle, b, want_logits=True)
    assert np.array_equal(ig, io), np.nonzero(ig != io)[0][:10]
    assert np.array_equal(rg, ro)
    assert np.array_equal(bits(lg), bits(lo))


@pytest.mark.parametrize("max_rows,B,split", [(96, 1000, False), (96, 200, False), (96, 200, True), (1, 37, False)])
def test_sized_context(c4s, oracle, wl, max_rows, B, split):
    """A context sized for max_rows rows per call (c4s_create_sized) samples
    larger batches in chunks of max_rows (split path) or with fewer CTAs
    (fused kernel): ids, states and processed logits bit-exact."""
    free0 = torch.cuda.mem_get_info(0)[0]
    ctx = c4s.SamplingContext(max_vocab=8194, device=0, max_rows=max_rows)
    used = free0 - torch.cuda.mem_get_info(0)[0]
    # per row: two 72 KB candidate lists and two 128 KB scratch slabs; allocation granularity on top
    assert used <= (32 << 20) + max_rows * (420 << 10), used
    if split:
        ctx.set_debug(c4s.sampling.DEBUG_SPLIT_PATH)
    b = wl.config2(seed=37 + max_rows, B=B)
    ig, rg, lg = gpu_sample(ctx, b, torch, want_logits=True)
    io, ro, lo = oracle_sample(oracle, b, want_logits=True)
    assert np.array_equal(ig, io), np.nonzero(ig != io)[0][:10]
    assert np.array_equal(rg, ro)
    assert np.array_equal(bits(lg), bits(lo))
    # argmax on the general kernel, with fewer CTAs than rows
    x = torch.from_numpy(b.logits).cuda()
    assert np.array_equal(ctx.argmax(x).cpu().numpy(), np.argmax(b.logits, axis=1))
    ctx.close()


def test_split_path_recovers_after_failed_launch(c4s, oracle, wl):
    """A split-path call whose list-kernel launch fails on the host (no kernel
    faults: the launch is refused before it is made) returns an error; its
    row kernel has already taken queue tickets, and the next call must still
    sample every row bit-exactly."""
    ctx = c4s.SamplingContext(max_vocab=8194, device=0)
    ctx.set_debug(c4s.sampling.DEBUG_SPLIT_PATH | c4s.sampling.DEBUG_FAIL_AFTER_ROW)
    b = wl.config2(seed=33, B=1000)
    with pytest.raises(c4s.C4SError):
        gpu_sample(ctx, b, torch)
    torch.cuda.synchronize()
    ctx.set_debug(c4s.sampling.DEBUG_SPLIT_PATH)
    ig, rg, _ = gpu_sample(ctx, b, torch)
    io, ro, _ = oracle_sample(oracle, b)
    assert np.array_equal(ig, io)
    assert np.array_equal(rg, ro)


def _div_sweep(c4s, xbits, divisors):
    lib = c4s.library()
    x = torch.from_numpy(xbits.view(np.float32)).cuda()
    out = torch.empty_like(x)
    xh = xbits.view(np.float32)
    for d in divisors:
        rc = lib.c4s_test_div_rn(x.data_ptr(), float(np.float32(d)), out.data_ptr(), x.numel(), None)
        assert rc == 0
        torch.cuda.synchronize()
        want = (xh / np.float32(d)).astype(np.float32)          # IEEE round-to-nearest
        got = out.cpu().numpy()
        bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
        assert bad.size == 0, (d, xh[bad[:5]], got[bad[:5]], want[bad[:5]])


def test_div_rn_every_mantissa(c4s):
    """The inline exact division against IEEE division, bit for bit: every
    mantissa of x in the binades [1, 2) and [-2^-3, -2^-2), for temperatures,
    penalties, powers of two and divisors next to 1 (sampling.cpp:16, :26)."""
    m = np.arange(1 << 23, dtype=np.uint32)
    divisors = [0.5, 0.8, 1.2, 0.5000001, 0.99999994, 1.0000001, 3.0, 10.0, 2.0, 0.25, 1.7, 9.99]
    _div_sweep(c4s, m | np.uint32(127 << 23), divisors)                     # [1, 2)
    _div_sweep(c4s, m | np.uint32((1 << 31) | (124 << 23)), divisors)       # [-2^-3, -2^-2)


def test_div_rn_extreme_operands(c4s):
    """Quotients near the proof check's limits: tiny and huge dividends,
    subnormals, zeros of both signs, infinities."""
    g = np.random.default_rng(17)
    xs = [g.integers(0, 1 << 32, 1 << 20, dtype=np.uint64).astype(np.uint32)]   # every float class
    for e in (1, 2, 25, 26, 27, 100, 101, 126, 127, 226, 227, 228, 253, 254):
        xs.append(g.integers(0, 1 << 23, 4096).astype(np.uint32) | np.uint32(e << 23))
    xs.append(np.arange(1 << 16, dtype=np.uint32))                             # subnormals
    xs.append(np.array([0, 1 << 31, 0x7f800000, 0xff800000, 0x7f7fffff, 0x00800000], np.uint32))
    xb = np.concatenate(xs)
    xb = xb[~np.isnan(xb.view(np.float32))]
    _div_sweep(c4s, xb, [0.5, 0.8, 1.2, 10.0, 1e-30, 1e30, 3.0e-39, 1.0e38, 2.0 ** -100, 2.0 ** 100,
                         7.0, 0.1])


@pytest.mark.parametrize("flags", [1, 2, 3, 4, 1 | 32, 2 | 32, 4 | 32])
def test_forced_slow_paths(c4s, oracle, wl, flags):
    """The exact fallbacks, the binned paths and the exact-tail refinement of
    rows without top-k, forced on ordinary rows (split kernels at B = 384,
    and with flag 32 the fused kernel)."""
    ctx = c4s.SamplingContext(max_vocab=8194, device=0)
    ctx.set_debug(flags)
    b = wl.config2(seed=7, B=384)
    ctx.status(reset=True)
    ig, rg, lg = gpu_sample(ctx, b, torch, want_logits=True)
    err, cnt = ctx.status(reset=True)
    io, ro, lo = oracle_sample(oracle, b, want_logits=True)
    assert err == 0
    assert np.array_equal(ig, io)
    assert np.array_equal(rg, ro)
    assert np.array_equal(bits(lg), bits(lo))
    if flags & 2:
        assert cnt["topp_binned"] > 0 and cnt["draw_rowpass"] > 0
    if flags & 1:
        assert cnt["topk_radix"] > 0
    if flags & 4:
        assert cnt["exact_tail"] > 0


def test_path_counters_and_no_errors(ctx, wl):
    b = wl.config2(seed=9, B=1024)
    ctx.status(reset=True)
    gpu_sample(ctx, b, torch)
    err, cnt = ctx.status(reset=True)
    assert err == 0
    # rows handed to the general path are rare: rows without top-k whose
    # candidate list would exceed the list capacity (about 1% of config-2
    # rows), undecided double-precision bands, inputs outside the fast path
    assert cnt["deferred"] <= b.B // 50


# ---------------------------------------------------------------------------
# Edge cases the reference defines.
# ---------------------------------------------------------------------------
def _mk_batch(wl, rows, hists, params, seed=1):
    V = len(rows[0])
    B = len(rows)
    x = np.stack([np.asarray(r, np.float32) for r in rows])
    lens = np.array([len(h) for h in hists], np.int64)
    off = np.zeros(B + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    hist = np.concatenate([np.asarray(h, np.int32) for h in hists]) if off[-1] else np.zeros(0, np.int32)
    return wl.Batch(x, V, hist, off, params, wl.seed_states(B, seed))


def _check_same(ctx, oracle, b, active=None, ld_pad=0):
    ig, rg, lg = gpu_sample(ctx, b, torch, active=active, want_logits=True, ld_pad=ld_pad)
    io, ro, lo = oracle_sample(oracle, b, active=active, want_logits=True)
    assert np.array_equal(ig, io), (np.nonzero(ig != io), ig[ig != io], io[ig != io])
    assert np.array_equal(rg, ro)
    rows = np.ones(b.B, bool) if active is None else active.astype(bool)
    assert np.array_equal(bits(lg[rows]), bits(lo[rows]))
    return ig


def test_edge_parameters(ctx, oracle, wl):
    g = np.random.default_rng(3)
    V = 1000
    cases = [dict(top_k=1), dict(top_k=V - 1), dict(top_k=V), dict(top_k=-5), dict(top_k=0),
             dict(top_p=1.0), dict(top_p=0.0), dict(top_p=1.5), dict(top_p=-0.5), dict(top_p=1e-6),
             dict(temperature=1.0), dict(temperature=0.0), dict(temperature=-2.0), dict(temperature=3.0),
             dict(repetition_penalty=1.0), dict(repetition_penalty=0.5), dict(repetition_penalty=50.0),
             dict(min_tokens_to_keep=0), dict(min_tokens_to_keep=5), dict(min_tokens_to_keep=5000),
             dict(top_k=0, top_p=0.999), dict(top_k=0, top_p=1.0, min_tokens_to_keep=3),
             dict(greedy=1), dict(greedy=1, repetition_penalty=1.0)]
    rows, hists, plist = [], [], []
    for c in cases:
        for _ in range(3):
            rows.append(g.normal(0, 3, V).astype(np.float32))
            hists.append(g.integers(-5, V + 5, g.integers(0, 300)))
            kw = dict(temperature=0.8, top_k=30, top_p=0.8, repetition_penalty=10.0)
            kw.update(c)
            plist.append(wl.make_params(1, **kw))
    b = _mk_batch(wl, rows, hists, np.concatenate(plist))
    _check_same(ctx, oracle, b)


def test_edge_rows(ctx, oracle, wl):
    g = np.random.default_rng(4)
    V = 777
    rows = [
        np.full(V, -np.inf, np.float32),                        # all -inf
        np.zeros(V, np.float32),                                # constant (all ties)
        np.where(g.random(V) < 0.5, -np.inf, g.normal(0, 3, V)).astype(np.float32),
        np.round(g.normal(0, 1.5, V)).astype(np.float32),       # many ties
        np.where(g.random(V) < 0.3, -0.0, 0.0).astype(np.float32),  # signed zeros
        np.full(V, -1e31, np.float32),                          # below the draw's -1e30 floor
        np.r_[np.full(V - 1, -np.inf), 5.0].astype(np.float32),  # single survivor
        (g.normal(0, 3, V) * 40).astype(np.float32),            # very wide spread
        (g.normal(0, 1e-3, V)).astype(np.float32),              # very flat
    ]
    for kw in (dict(top_k=30, top_p=0.8), dict(top_k=0, top_p=0.9), dict(top_k=0, top_p=1.0),
               dict(top_k=5, top_p=0.5), dict(top_k=0, top_p=0.99999)):
        P = np.concatenate([wl.make_params(1, temperature=0.8, repetition_penalty=10.0, **kw)
                            for _ in rows])
        b = _mk_batch(wl, rows, [g.integers(0, V, 50) for _ in rows], P)
        _check_same(ctx, oracle, b)


@pytest.mark.parametrize("V,ld_pad", [(1, 0), (2, 3), (3, 1), (5, 0), (64, 0), (8194, 0), (8194, 2),
                                      (8195, 1), (8193, 0), (20000, 0), (32768, 0)])
def test_vocab_sizes_and_strides(ctx, oracle, wl, V, ld_pad):
    """Unaligned rows (odd ld), tiny and maximal vocabularies."""
    b = wl.config2(seed=V, B=24, V=V)
    _check_same(ctx, oracle, b, ld_pad=ld_pad)


def test_long_history_and_duplicates(ctx, oracle, wl):
    g = np.random.default_rng(5)
    V = 8194
    rows = [g.normal(0, 3, V).astype(np.float32) for _ in range(6)]
    hists = [g.integers(0, V, 5000), np.repeat(g.integers(0, V, 10), 300), np.arange(V),
             np.array([], np.int64), np.array([-1, V, V + 7, -100]), g.integers(0, 64, 3000)]
    P = wl.make_params(6, temperature=0.9, top_k=50, top_p=0.9, repetition_penalty=3.0)
    b = _mk_batch(wl, rows, hists, P)
    _check_same(ctx, oracle, b)


def test_inactive_rows_and_mixed_greedy(ctx, oracle, wl):
    b = wl.config2(seed=12, B=200)
    b.params["greedy"][::3] = 1
    active = np.ones(200, np.uint8)
    active[::7] = 0
    ids = _check_same(ctx, oracle, b, active=active)
    assert np.all(ids[active == 0] == -1)


def test_seed_states_kernel(ctx, wl):
    s = ctx.seed_states(1000, 0, row_offset=5).cpu().numpy().view(np.uint64)
    assert np.array_equal(s, wl.seed_states(1000, 0, 5))
    s = ctx.seed_states(3, 1234).cpu().numpy().view(np.uint64)
    assert np.array_equal(s, wl.seed_states(3, 1234))


def test_history_offsets_out_of_range_reported(c4s, wl):
    ctx = c4s.SamplingContext(max_vocab=8194, device=0)
    b = wl.config2(seed=13, B=4)
    d = to_dev(b, torch)
    bad_off = torch.tensor([0, 10, 5, 20, 10**9], dtype=torch.int64, device="cuda")  # non-monotone + past end
    ctx.status(reset=True)
    ctx.sample(d["logits"], d["hist"], bad_off, d["params"], d["rng"])
    err, _ = ctx.status(reset=True)
    assert err & 1


def test_invalid_arguments_rejected(c4s, ctx):
    x = torch.zeros((2, 16), device="cuda")
    p = c4s.params_tensor(c4s.workloads.make_params(2), x.device)
    r = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(c4s.C4SError):
        ctx.sample(x, None, None, p, r, V=17)          # V > ld
    with pytest.raises(c4s.C4SError):
        ctx.sample(x, None, None, p, r, params_stride=2)
    with pytest.raises(c4s.C4SError):
        ctx.process(x, None, None, p, 64)                # unknown stage bit
    with pytest.raises(c4s.C4SError):
        c4s.SamplingContext(max_vocab=10**6, device=0)
