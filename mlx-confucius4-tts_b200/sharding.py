"""Row sharding of a sampling batch across GPUs (one process per GPU).

Rows of a batch are independent: each carries its own logits, history,
parameters and xorshift64 state (text2semantic.cpp:292-331 of the reference
loops over them one by one). A rank therefore owns a contiguous block of rows
and needs no collective on the data path; seeding with the block's global row
offset gives every row the state it would have in a single-device batch.
"""
from __future__ import annotations


def shard_rows(total_rows: int, rank: int, world: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s contiguous block; sizes differ by <= 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if total_rows < 0:
        raise ValueError("total_rows < 0")
    base, extra = divmod(total_rows, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)
