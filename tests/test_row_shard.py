"""Row sharding (configs 0-2 on N GPUs): every rank owns a contiguous block of
rows and needs no collective on the data path.

The rule checked here: a rank that takes rows [start, start + n) of a batch
(``sharding.shard_rows``) and seeds their xorshift64 states with the block's
global row offset (text2semantic.cpp:292-295 of the reference, ``row_offset``
of c4s_seed_states) produces, row for row, the ids and states of the
unsharded batch. The per-rank step is the oracle here (CPU test
infrastructure standing in for the kernel); two `gloo` ranks gather their
blocks and compare with one process sampling the whole batch.
"""
import os
import socket

import numpy as np
import pytest

from conftest import load_c4s
from helpers import NTHREADS


def test_shard_rows_partition(c4s):
    for total, world in ((4096, 8), (13, 4), (3, 5), (0, 2), (1, 1)):
        spans = [c4s.sharding.shard_rows(total, r, world) for r in range(world)]
        assert spans[0][0] == 0
        assert sum(n for _, n in spans) == total
        for (s0, n0), (s1, _) in zip(spans, spans[1:]):
            assert s0 + n0 == s1
        assert max(n for _, n in spans) - min(n for _, n in spans) <= 1
    with pytest.raises(ValueError):
        c4s.sharding.shard_rows(10, 2, 2)
    with pytest.raises(ValueError):
        c4s.sharding.shard_rows(-1, 0, 1)


def _batch(c4s):
    b = c4s.workloads.config2(seed=31, B=13)
    b.rng[:] = c4s.workloads.seed_states(b.B, 1234)
    return b


def _rank_block(c4s, oracle, b, rank, world):
    start, n = c4s.sharding.shard_rows(b.B, rank, world)
    off = b.hist_off[start:start + n + 1]
    hist = b.hist[off[0]:off[-1]]
    rng = c4s.workloads.seed_states(n, 1234, row_offset=start)
    ids, _ = oracle.sample_batch(np.ascontiguousarray(b.logits[start:start + n]), b.V, hist, off - off[0],
                                 b.params[start:start + n], rng, nthreads=1)
    return ids, rng


def _gloo_rank(rank, world, port, q):
    import sys
    import torch
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (here, os.path.join(os.path.dirname(here), "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import oracle as orc
    c4s = load_c4s()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        b = _batch(c4s)
        ids, rng = _rank_block(c4s, orc.Oracle(), b, rank, world)
        cap = -(-b.B // world)                      # pad blocks to the largest
        t = torch.full((cap, 3), -1, dtype=torch.int64)
        t[:len(ids), 0] = torch.from_numpy(ids.astype(np.int64))
        t[:len(ids), 1] = torch.from_numpy((rng & np.uint64(0xFFFFFFFF)).astype(np.int64))
        t[:len(ids), 2] = torch.from_numpy((rng >> np.uint64(32)).astype(np.int64))
        out = torch.empty((world * cap, 3), dtype=torch.int64)
        dist.all_gather_into_tensor(out, t)
        if rank == 0:
            q.put(out.numpy().copy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gloo_two_ranks_match_whole_batch(oracle):
    import torch.multiprocessing as mp
    c4s = load_c4s()
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    b = _batch(c4s)
    ro = b.rng.copy()
    oid, _ = oracle.sample_batch(b.logits, b.V, b.hist, b.hist_off, b.params, ro, nthreads=NTHREADS)
    cap = -(-b.B // world)
    rows = []
    for r in range(world):
        _, n = c4s.sharding.shard_rows(b.B, r, world)
        rows.append(got[r * cap:r * cap + n])
    g = np.concatenate(rows)
    assert np.array_equal(g[:, 0].astype(np.int32), oid)
    st = g[:, 1].astype(np.uint64) | (g[:, 2].astype(np.uint64) << np.uint64(32))
    assert np.array_equal(st, ro)
