"""Vocab-sharded sampling: every row's vocabulary split across GPUs.

No GPU holds a whole row, so one step is three parts (include/c4s_sampling.h):
each rank computes the 64 largest penalised, tempered values of its shard
(``SamplingContext.shard_candidates``), the ranks all-gather those [B, 64]
blocks over NCCL, and every rank merges them into the same token ids with the
same xorshift64 state updates (``SamplingContext.merge_candidates``). For
rows with 1 <= top_k <= 64 the ids equal those of sampling the whole row
(text2semantic.cpp:303-331 of the reference); other sampled rows come back
as -1 with the C4S_DEVERR_SHARD error bit.
"""
from __future__ import annotations

import numpy as np

from . import workloads
from .sampling import MAX_SHARDS, SHARD_CANDIDATES, params_tensor
from .sharding import shard_rows


def check_shardable(params, active=None) -> None:
    """Raise ValueError if a sampled row's top_k is outside [1, 64]: the merge
    is exact only there and refuses such rows (id -1, C4S_DEVERR_SHARD).
    The reference's own T2S entry points default to top_k = 0 (t2s.h:156,169
    of the reference); sample those rows with SamplingContext.sample on whole
    rows instead. ``params`` is a host ROW_PARAMS_DTYPE array (one struct or
    one per row), ``active`` an optional host mask."""
    p = np.atleast_1d(np.asarray(params, dtype=workloads.ROW_PARAMS_DTYPE))
    bad = (p["greedy"] == 0) & ((p["top_k"] < 1) | (p["top_k"] > SHARD_CANDIDATES))
    if active is not None and p.size > 1:
        bad &= np.asarray(active, dtype=bool).reshape(-1)
    if bad.any():
        rows = np.nonzero(bad)[0]
        raise ValueError(f"vocab-sharded sampling needs 1 <= top_k <= {SHARD_CANDIDATES} on every sampled "
                         f"row; rows {rows[:8].tolist()}{' ...' if rows.size > 8 else ''} have top_k "
                         f"{p['top_k'][rows[:8]].tolist()}")


def _device_params(params, active, tensor):
    """Host params are checked (check_shardable) and uploaded to the device of
    `tensor`; a device tensor is taken as is (refused rows then come back -1)."""
    if isinstance(params, np.ndarray):
        check_shardable(params, active if isinstance(active, np.ndarray) else None)
        return params_tensor(np.atleast_1d(params), tensor.device)
    return params


SUB_WIDTH = 8192              # widest sub-shard a rank's candidate launch works


def shard_vocab(V: int, rank: int, world: int) -> tuple[int, int]:
    """(first column, width) of `rank`'s contiguous vocabulary shard."""
    return shard_rows(V, rank, world)


def sub_shards(width: int, world: int, sub_width: int = SUB_WIDTH) -> int:
    """Sub-shards of a rank's `width` columns: blocks of at most `sub_width`
    (so that a wide shard keeps several CTAs per SM), at most
    C4S_MAX_SHARDS blocks over all ranks, at least 64 columns each."""
    n = max(1, -(-width // sub_width))
    n = min(n, max(1, MAX_SHARDS // world), max(1, width // SHARD_CANDIDATES))
    return n


def sample_vocab_sharded(ctx, logits_shard, V: int, hist, hist_off, params, rng, group=None,
                         active=None, out_ids=None, params_stride: int = 1, cand_out=None,
                         sub_width: int = SUB_WIDTH):
    """One sampling step on this rank's shard of every row.

    ``logits_shard`` [B, ld] holds the columns ``shard_vocab(V, rank, world)``
    of each row (rank and world of ``group``, the default process group if
    None). ``hist``/``hist_off`` carry global ids. Returns int32 ids [B],
    identical on every rank; ``rng`` is advanced identically on every rank.
    ``params`` as a host ROW_PARAMS_DTYPE array is checked first
    (check_shardable: ValueError for a sampled row with top_k outside
    [1, 64]); as a device tensor it is used unchecked. Each rank computes
    its shard as ``sub_shards(width, world)`` sub-shards of at most
    ``sub_width`` columns; the gathered blocks ([world * sub, B, 64],
    rank-major) are in vocabulary order.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    voff, width = shard_vocab(V, rank, world)
    B = logits_shard.shape[0]
    dev = logits_shard.device
    params = _device_params(params, active, logits_shard)
    # every rank's width gives the same sub-shard count (widths differ by at most one)
    nsub = sub_shards(shard_vocab(V, 0, world)[1], world, sub_width)
    local = torch.empty((nsub, B, SHARD_CANDIDATES), dtype=torch.int64, device=dev)
    if nsub == 1:
        ctx.shard_candidates(logits_shard, V, voff, hist, hist_off, params, active=active,
                             out=local[0], V_shard=width, params_stride=params_stride)
    else:
        ctx.shard_candidates(logits_shard, V, voff, hist, hist_off, params, active=active,
                             out=local, V_shard=width, params_stride=params_stride, num_sub=nsub)
    if world > 1:
        if cand_out is None:
            cand_out = torch.empty((world * nsub, B, SHARD_CANDIDATES), dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(cand_out.view(world * nsub * B, SHARD_CANDIDATES),
                                    local.view(nsub * B, SHARD_CANDIDATES), group=group)
    else:
        cand_out = local
    return ctx.merge_candidates(cand_out, V, params, rng, active=active, out_ids=out_ids,
                                params_stride=params_stride)


def sample_vocab_split(ctx, logits, num_shards: int, hist, hist_off, params, rng, active=None,
                       out_ids=None, params_stride: int = 1, cand_out=None, V: int | None = None):
    """The same step with all shards on one GPU: ``logits`` [B, ld] holds whole
    rows; shard s is the column block ``shard_vocab(V, s, num_shards)``, and
    one launch writes the candidate blocks straight into the gathered layout
    [G, B, 64]. Also the way to sample rows wider than ``SamplingContext.sample``
    takes (32768) on one GPU, for 1 <= top_k <= 64 (host ``params`` are
    checked as in sample_vocab_sharded)."""
    import torch

    params = _device_params(params, active, logits)
    B, ld = logits.shape
    V = ld if V is None else V
    if cand_out is None:
        cand_out = torch.empty((num_shards, B, SHARD_CANDIDATES), dtype=torch.int64,
                               device=logits.device)
    ctx.shard_candidates_split(logits, num_shards, hist, hist_off, params, active=active,
                               out=cand_out, V=V, params_stride=params_stride)
    return ctx.merge_candidates(cand_out, V, params, rng, active=active, out_ids=out_ids,
                                params_stride=params_stride)
