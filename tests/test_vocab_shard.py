"""Vocab-sharded sampling (every row's vocabulary split into contiguous shards).

The product path is shard_candidates -> all-gather -> merge_candidates
(include/c4s_sampling.h, mlx-confucius4-tts_b200/vocab_shard.py). Its claim:
for 1 <= top_k <= 64 the ids and xorshift64 states equal those of sampling
the whole row, i.e. the oracle's restatement of text2semantic.cpp:303-331 of
the reference on the unsplit row.

CPU tests drive the host logic (shard bounds, gather layout, merge call)
over `gloo` with a stand-in context built from the oracle's processors; GPU
tests run the CUDA kernels through the C ABI against the oracle on whole rows.
"""
import os
import socket

import numpy as np
import pytest

from conftest import load_c4s
from helpers import NTHREADS, to_dev

C = 64


def _penalise_slice(x, voff, hist, pen):
    """sampling.cpp:19-28 on the columns [voff, voff + len(x)) of a row."""
    if pen == np.float32(1.0):
        return
    seen = set()
    for t in hist:
        t = int(t)
        if t in seen or not voff <= t < voff + len(x):
            continue
        seen.add(t)
        s = x[t - voff]
        x[t - voff] = s * pen if s < 0 else s / pen


class OracleShardContext:
    """Stand-in for SamplingContext's two sharded calls, from the oracle's
    processors (test infrastructure: lets the gloo test run without a GPU)."""

    def __init__(self, oracle):
        self.o = oracle

    def shard_candidates(self, logits, V, vocab_offset, hist, hist_off, params, active=None,
                         out=None, V_shard=None, params_stride=1, num_sub=1):
        if num_sub > 1:                             # sub-shard s of the shard's columns into out[s]
            c4s = load_c4s()
            for s in range(num_sub):
                so, sw = c4s.vocab_shard.shard_vocab(V_shard, s, num_sub)
                self.shard_candidates(logits[:, so:so + sw], V, vocab_offset + so, hist, hist_off, params,
                                      active, out[s], sw, params_stride)
            return out
        x_all = logits.numpy()
        P = np.frombuffer(params.numpy().tobytes(), dtype=load_c4s().workloads.ROW_PARAMS_DTYPE)
        h = hist.numpy()
        off = hist_off.numpy()
        res = out.numpy().view(np.uint32).reshape(out.shape[0], C, 2)
        for b in range(x_all.shape[0]):
            p = P[b * params_stride]
            x = x_all[b, :V_shard].astype(np.float32).copy()
            _penalise_slice(x, vocab_offset, h[off[b]:off[b + 1]], np.float32(p["repetition_penalty"]))
            if not p["greedy"]:
                self.o.temperature(x, float(p["temperature"]))
            order = np.lexsort((np.arange(len(x)), -x))
            top = order[:C]
            res[b, :, 0] = x[top].view(np.uint32)
            res[b, :, 1] = (top + vocab_offset).astype(np.uint32)
            if len(x) > C and x[order[C]] == x[order[C - 1]]:
                res[b, C - 1, 1] |= np.uint32(0x80000000)
        return out

    def merge_candidates(self, cand, V, params, rng, active=None, out_ids=None, params_stride=1):
        import torch
        G, B, _ = cand.shape
        raw = cand.numpy().view(np.uint32).reshape(G, B, C, 2)
        P = np.frombuffer(params.numpy().tobytes(), dtype=load_c4s().workloads.ROW_PARAMS_DTYPE)
        st = rng.numpy().view(np.uint64)
        ids = np.empty(B, np.int32)
        for b in range(B):
            p = P[b * params_stride]
            vals = raw[:, b, :, 0].ravel().view(np.float32)
            idx = (raw[:, b, :, 1].ravel() & np.uint32(0x7fffffff)).astype(np.int64)
            row = np.full(V, -np.inf, np.float32)
            row[idx] = vals
            if p["greedy"]:
                ids[b] = self.o.argmax(row)
                continue
            self.o.top_k(row, int(p["top_k"]))
            self.o.top_p(row, float(p["top_p"]), int(p["min_tokens_to_keep"]))
            s = st[b:b + 1].copy()
            ids[b] = self.o.draw(row, s)
            st[b] = s[0]
        out = torch.from_numpy(ids)
        if out_ids is not None:
            out_ids.copy_(out)
            return out_ids
        return out


def _gloo_rank(rank, world, port, V, B, q, sub_width):
    import torch
    import torch.distributed as dist
    sys_path_setup()
    c4s = load_c4s()
    import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b = c4s.workloads.config4(seed=7, B=B, V=V)
        voff, width = c4s.vocab_shard.shard_vocab(V, rank, world)
        logits = torch.from_numpy(np.ascontiguousarray(b.logits[:, voff:voff + width]))
        params = torch.from_numpy(np.ascontiguousarray(b.params).view(np.uint8).copy())
        rng = torch.from_numpy(b.rng.view(np.int64).copy())
        ids = c4s.vocab_shard.sample_vocab_sharded(
            OracleShardContext(orc.Oracle()), logits, V, torch.from_numpy(b.hist),
            torch.from_numpy(b.hist_off), params, rng, sub_width=sub_width)
        q.put((rank, ids.numpy().copy(), rng.numpy().view(np.uint64).copy()))
    finally:
        dist.destroy_process_group()


def sys_path_setup():
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (here, os.path.join(os.path.dirname(here), "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_vocab_bounds(c4s):
    for V, world in ((65536, 8), (8194, 3), (100, 1), (1000, 7)):
        spans = [c4s.vocab_shard.shard_vocab(V, r, world) for r in range(world)]
        assert spans[0][0] == 0
        assert sum(w for _, w in spans) == V
        for (o0, w0), (o1, _) in zip(spans, spans[1:]):
            assert o0 + w0 == o1
        assert max(w for _, w in spans) - min(w for _, w in spans) <= 1


def test_candidate_merge_is_exact_against_whole_rows(c4s, oracle):
    """The shard/merge decomposition restated with the oracle's processors
    gives the whole-row ids and states (including rounded logits with ties)."""
    import torch
    b = c4s.workloads.config4(seed=3, B=12, V=6000)
    b.logits[6:] = np.round(b.logits[6:])            # many ties below the threshold
    G = 5
    ctx = OracleShardContext(oracle)
    params = torch.from_numpy(np.ascontiguousarray(b.params).view(np.uint8).copy())
    cand = torch.empty((G, b.B, C), dtype=torch.int64)
    for s in range(G):
        voff, width = c4s.vocab_shard.shard_vocab(b.V, s, G)
        ctx.shard_candidates(torch.from_numpy(np.ascontiguousarray(b.logits[:, voff:voff + width])),
                             b.V, voff, torch.from_numpy(b.hist), torch.from_numpy(b.hist_off), params,
                             out=cand[s], V_shard=width)
    rng = torch.from_numpy(b.rng.view(np.int64).copy())
    ids = ctx.merge_candidates(cand, b.V, params, rng).numpy()
    ro = b.rng.copy()
    oid, _ = oracle.sample_batch(b.logits, b.V, b.hist, b.hist_off, b.params, ro, nthreads=NTHREADS)
    assert np.array_equal(ids, oid)
    assert np.array_equal(rng.numpy().view(np.uint64), ro)


@pytest.mark.parametrize("sub_width", [8192, 700])
def test_gloo_two_ranks_match_whole_rows(oracle, sub_width):
    """world_size 2 over gloo: sample_vocab_sharded's shard bounds, gather
    layout and merge give every rank the whole-row ids and states, each rank's
    shard in one block or (sub_width 700) as three sub-shards, six blocks."""
    import torch.multiprocessing as mp
    c4s = load_c4s()
    V, B, world = 4096 + 3, 8, 2
    assert c4s.vocab_shard.sub_shards(c4s.vocab_shard.shard_vocab(V, 0, world)[1], world, sub_width) == \
        (1 if sub_width == 8192 else 3)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, V, B, q, sub_width)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    b = c4s.workloads.config4(seed=7, B=B, V=V)
    ro = b.rng.copy()
    oid, _ = oracle.sample_batch(b.logits, b.V, b.hist, b.hist_off, b.params, ro, nthreads=NTHREADS)
    for _, ids, st in got:
        assert np.array_equal(ids, oid)
        assert np.array_equal(st, ro)


# ---------------------------------------------------------------------------
# GPU: the CUDA kernels through the C ABI
# ---------------------------------------------------------------------------
def _inv_xorshift_state(out: int) -> int:
    """State whose xorshift64 (13, 7, 17) successor is `out`."""
    M = (1 << 64) - 1

    def inv_shl(y, s):
        x = y
        for _ in range(64 // s + 1):
            x = y ^ ((x << s) & M)
        return x

    def inv_shr(y, s):
        x = y
        for _ in range(64 // s + 1):
            x = y ^ (x >> s)
        return x

    return inv_shl(inv_shr(inv_shl(out, 17), 7), 13)


def _gpu_split(ctx, b, G, torch, active=None, ld_pad=0):
    c4s = load_c4s()
    d = to_dev(b, torch, ld_pad)
    act = None if active is None else torch.from_numpy(active.astype(np.uint8)).cuda()
    ids = c4s.vocab_shard.sample_vocab_split(ctx, d["logits"], G, d["hist"], d["hist_off"], d["params"],
                                             d["rng"], active=act, V=b.V)
    torch.cuda.synchronize()
    err, _ = ctx.status(reset=True)
    return ids.cpu().numpy(), d["rng"].cpu().numpy().view(np.uint64), err


def _oracle(oracle, b, active=None):
    ro = b.rng.copy()
    oid, _ = oracle.sample_batch(np.ascontiguousarray(b.logits), b.V, b.hist, b.hist_off, b.params, ro,
                                 active=active, nthreads=NTHREADS)
    return oid, ro


@pytest.fixture(scope="module")
def sctx():
    c4s = load_c4s()
    ctx = c4s.SamplingContext(max_vocab=c4s.workloads.SEMANTIC_VOCAB, device=0)
    yield ctx
    ctx.close()


def _check_xorshift_inverse():
    s = 0x0123456789ABCDEF
    x = s
    x ^= (x << 13) & ((1 << 64) - 1)
    x ^= x >> 7
    x ^= (x << 17) & ((1 << 64) - 1)
    assert _inv_xorshift_state(x) == s


def test_xorshift_inverse():
    _check_xorshift_inverse()


@pytest.mark.gpu
def test_config4_eight_shards_one_gpu(sctx, oracle):
    """Config 4 (B=512, V=65536, 8 shards of 8192, top_k 50, top_p 0.9): ids
    and states equal the oracle's on the whole rows; greedy too."""
    import torch
    c4s = load_c4s()
    b = c4s.workloads.config4()
    ids, st, err = _gpu_split(sctx, b, 8, torch)
    oid, ro = _oracle(oracle, b)
    assert err == 0
    assert np.array_equal(ids, oid)
    assert np.array_equal(st, ro)
    b.params["greedy"] = 1
    ids, st, err = _gpu_split(sctx, b, 8, torch)
    oid, ro = _oracle(oracle, b)
    assert err == 0
    assert np.array_equal(ids, oid)
    assert np.array_equal(st, b.rng)


@pytest.mark.gpu
@pytest.mark.parametrize("V,G,ld_pad,k", [(8194, 3, 0, 30), (1000, 7, 3, 64), (20000, 16, 1, 1),
                                          (65536, 2, 0, 20)])
def test_ragged_shards_strides_and_topk(sctx, oracle, V, G, ld_pad, k):
    import torch
    c4s = load_c4s()
    b = c4s.workloads.config4(seed=V + G, B=64, V=V, top_k=k, top_p=0.8)
    b.params["top_p"] = np.random.default_rng(V).uniform(0.3, 1.0, size=b.B).astype(np.float32)
    b.params["temperature"][::5] = 1.0
    b.params["repetition_penalty"][::7] = 1.0
    ids, st, err = _gpu_split(sctx, b, G, torch, ld_pad=ld_pad)
    oid, ro = _oracle(oracle, b)
    assert err == 0
    assert np.array_equal(ids, oid)
    assert np.array_equal(st, ro)


@pytest.mark.gpu
def test_history_lengths_and_repeats(sctx, oracle):
    """The shard kernel penalises histories of up to 1024 ids by
    read-then-write and longer ones through a de-duplication bitmap: rows of
    0 to 6000 ids, many repeated (ids drawn from a narrow range that falls in
    one or two shards), out-of-range ids, penalties above and below 1."""
    import torch
    c4s = load_c4s()
    V, G, B = 65536, 8, 48
    b = c4s.workloads.config4(seed=77, B=B, V=V, top_k=40, top_p=0.85)
    g = np.random.default_rng(77)
    lens = np.array([0, 1, 2, 31, 255, 256, 1023, 1024, 1025, 2048, 4000, 6000] * 4)
    off = np.zeros(B + 1, dtype=np.int64)
    np.cumsum(lens, out=off[1:])
    hist = np.empty(int(off[-1]), dtype=np.int32)
    for r in range(B):
        n = int(lens[r])
        if r % 4 == 0:
            ids = g.integers(0, V, size=n)                 # uniform: few repeats
        elif r % 4 == 1:
            ids = g.integers(8000, 8400, size=n)           # narrow: many repeats across a shard edge
        elif r % 4 == 2:
            ids = g.integers(-50, V + 50, size=n)          # some out of range (ignored)
        else:
            ids = np.argsort(b.logits[r])[-64:][g.integers(0, 64, size=n)]  # the row's largest values
        hist[off[r]:off[r + 1]] = ids.astype(np.int32)
    b.hist, b.hist_off = hist, off
    b.params["repetition_penalty"][::3] = 0.5
    b.params["temperature"][1::5] = 1.0
    ids, st, err = _gpu_split(sctx, b, G, torch)
    oid, ro = _oracle(oracle, b)
    assert err == 0
    assert np.array_equal(ids, oid)
    assert np.array_equal(st, ro)


@pytest.mark.gpu
def test_ties_fallback_and_refusals(sctx, oracle):
    """Rounded logits (ties below the threshold), a shard with more than 1024
    values above the fast path's bound (exact radix fallback), a draw with
    r == 0, inactive rows; rows the candidates cannot decide come back -1
    with the error bit."""
    import torch
    c4s = load_c4s()
    V, G, B = 16384, 4, 24
    b = c4s.workloads.config4(seed=11, B=B, V=V, top_k=30)
    g = np.random.default_rng(11)
    b.logits[:6] = np.round(b.logits[:6])
    for r in range(6, 12):                          # 2000 copies of 5.0 and 40 larger values per shard
        row = np.clip(g.normal(0, 1, V), -8, 4.5).astype(np.float32)
        for s in range(G):
            voff, width = c4s.vocab_shard.shard_vocab(V, s, G)
            pos = g.permutation(width)
            row[voff + pos[:2000]] = 5.0
            row[voff + pos[2000:2040]] = g.uniform(10, 20, 40).astype(np.float32)
        b.logits[r] = row
    b.hist_off[:] = 0                               # no history: the planted values stay as they are
    b.hist = b.hist[:0]
    b.rng[12] = np.uint64(_inv_xorshift_state(5))   # x >> 11 == 0: the reference returns index 0
    active = np.ones(B, bool)
    active[13] = False
    ids, st, err = _gpu_split(sctx, b, G, torch, active=active)
    oid, ro = _oracle(oracle, b, active=active)
    assert err == 0
    assert ids[12] == 0 and oid[12] == 0
    assert ids[13] == -1
    assert np.array_equal(ids, oid)
    assert np.array_equal(st, ro)
    # refusals: constant rows (ties across > 64 values at the threshold), top_k 0 and 65
    b.logits[0] = 1.0
    b.params["top_k"][1] = 0
    b.params["top_k"][2] = 65
    ids, st, err = _gpu_split(sctx, b, G, torch, active=active)
    assert err & c4s.sampling.DEVERR_SHARD
    assert list(ids[:3]) == [-1, -1, -1]
    oid, ro = _oracle(oracle, b, active=active)
    assert np.array_equal(ids[3:], oid[3:])


def test_host_params_checked_before_launch():
    """Host params with a sampled row outside 1 <= top_k <= 64 (the reference's
    T2S default top_k 0 among them) are refused on the host, before any
    device call; greedy and inactive rows are exempt."""
    c4s = load_c4s()
    vs = c4s.vocab_shard
    P = c4s.workloads.make_params(4, top_k=30)
    vs.check_shardable(P)
    P["top_k"][1] = 0
    with pytest.raises(ValueError, match=r"rows \[1\]"):
        vs.check_shardable(P)
    with pytest.raises(ValueError):
        vs.sample_vocab_split(None, None, 2, None, None, P, None)    # raises before touching ctx / logits
    P["greedy"][1] = 1
    vs.check_shardable(P)
    P["greedy"][1] = 0
    P["top_k"][2] = 65
    vs.check_shardable(P, active=np.array([1, 0, 0, 1], bool))
    with pytest.raises(ValueError):
        vs.check_shardable(P[2])                                       # one broadcast struct


@pytest.mark.gpu
def test_invalid_shard_arguments(sctx):
    import torch
    c4s = load_c4s()
    x = torch.zeros((4, 100), device="cuda")
    p = c4s.params_tensor(c4s.workloads.make_params(4), "cuda")
    with pytest.raises(c4s.C4SError):
        sctx.shard_candidates(x, 100, 0, None, None, p, V_shard=63)        # narrower than 64
    with pytest.raises(c4s.C4SError):
        sctx.shard_candidates(x, 150, 60, None, None, p, V_shard=100)      # past the vocabulary
    cand = torch.zeros((17, 4, 64), dtype=torch.int64, device="cuda")
    rng = torch.zeros(4, dtype=torch.int64, device="cuda")
    with pytest.raises(c4s.C4SError):
        sctx.merge_candidates(cand, 1000, p, rng)                          # more than 16 shards


def _nccl_rank(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist
    sys_path_setup()
    c4s = load_c4s()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        ctx = c4s.SamplingContext(max_vocab=c4s.workloads.SEMANTIC_VOCAB, device=rank)
        b = c4s.workloads.config4(seed=9)
        voff, width = c4s.vocab_shard.shard_vocab(b.V, rank, world)
        d = dict(logits=torch.from_numpy(np.ascontiguousarray(b.logits[:, voff:voff + width])).to(dev),
                 hist=torch.from_numpy(b.hist).to(dev), hist_off=torch.from_numpy(b.hist_off).to(dev),
                 params=c4s.params_tensor(b.params, dev),
                 rng=torch.from_numpy(b.rng.view(np.int64).copy()).to(dev))
        all_ids, all_st = [], []
        for _ in range(3):                           # three AR steps on the same logits
            ids = c4s.vocab_shard.sample_vocab_sharded(ctx, d["logits"], b.V, d["hist"], d["hist_off"],
                                                       d["params"], d["rng"])
            all_ids.append(ids.cpu().numpy())
            all_st.append(d["rng"].cpu().numpy().view(np.uint64).copy())
        torch.cuda.synchronize()
        err, _ = ctx.status(reset=True)
        ctx.close()
        q.put((rank, err, all_ids, all_st))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_two_ranks_match_whole_rows(oracle):
    """Config 4 on 2 GPUs: shard r on rank r, candidates all-gathered over
    NCCL; both ranks return the whole-row ids and states for 3 steps."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    c4s = load_c4s()
    world = 2
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_nccl_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    b = c4s.workloads.config4(seed=9)
    ro = b.rng.copy()
    for step in range(3):
        oid, _ = oracle.sample_batch(b.logits, b.V, b.hist, b.hist_off, b.params, ro, nthreads=NTHREADS)
        for _, err, ids, st in got:
            assert err == 0
            assert np.array_equal(ids[step], oid)
            assert np.array_equal(st[step], ro)


@pytest.mark.gpu
def test_split_launch_matches_per_shard_calls(sctx):
    """The one-launch form (all shards of whole rows) writes the same
    candidate blocks as one c4s_shard_candidates call per shard."""
    import torch
    c4s = load_c4s()
    b = c4s.workloads.config4(seed=5, B=96, V=20011)
    b.params["greedy"][::9] = 1
    d = to_dev(b, torch)
    G = 6
    split = sctx.shard_candidates_split(d["logits"], G, d["hist"], d["hist_off"], d["params"], V=b.V)
    per = torch.empty_like(split)
    for s in range(G):
        voff, width = c4s.vocab_shard.shard_vocab(b.V, s, G)
        sctx.shard_candidates(d["logits"][:, voff:], b.V, voff, d["hist"], d["hist_off"], d["params"],
                              out=per[s], V_shard=width)
    torch.cuda.synchronize()
    assert torch.equal(split, per)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_sub_shards_of_a_rank_match_whole_rows(sctx, oracle, world):
    """Config 4 as world ranks would run it, on one GPU: each rank's shard as
    sub-shards of at most 8192 columns (c4s_shard_candidates_sub), the blocks
    concatenated rank-major as the all-gather lays them out, then the merge:
    ids and states equal whole-row sampling; each rank's blocks equal one
    c4s_shard_candidates call per sub-shard."""
    import torch
    c4s = load_c4s()
    vs = c4s.vocab_shard
    b = c4s.workloads.config4(seed=40 + world, B=128)
    d = to_dev(b, torch)
    nsub = vs.sub_shards(vs.shard_vocab(b.V, 0, world)[1], world)
    assert world * nsub == 8
    blocks = []
    for r in range(world):
        voff, width = vs.shard_vocab(b.V, r, world)
        x = d["logits"][:, voff:voff + width]
        sub = sctx.shard_candidates(x, b.V, voff, d["hist"], d["hist_off"], d["params"], V_shard=width,
                                    num_sub=nsub)
        for s in range(nsub):
            so, sw = vs.shard_vocab(width, s, nsub)
            one = sctx.shard_candidates(d["logits"][:, voff + so:], b.V, voff + so, d["hist"], d["hist_off"],
                                        d["params"], V_shard=sw)
            assert torch.equal(sub[s], one)
        blocks.append(sub)
    cand = torch.cat(blocks, 0)
    ids = sctx.merge_candidates(cand, b.V, d["params"], d["rng"])
    torch.cuda.synchronize()
    err, _ = sctx.status(reset=True)
    oid, ro = _oracle(oracle, b)
    assert err == 0
    assert np.array_equal(ids.cpu().numpy(), oid)
    assert np.array_equal(d["rng"].cpu().numpy().view(np.uint64), ro)
