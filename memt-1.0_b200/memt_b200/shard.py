"""Head and session sharding for one process per GPU.

GDN-2 memory heads never interact: the update, the snapshot read and the gated RMSNorm
(per head, over the value dimension) each touch one head at a time, and sessions only
share the kernels. A rank therefore owns a contiguous slice of heads (tensor parallel)
or of sessions (data parallel) and runs the same kernels on that slice, with no
collective on the data path.

The head slice is the one the reference's tensor-parallel hook keeps after computing all
heads on every rank (``inference/memt_sglang/models/qwen/integration.py:52-57``: rank r
keeps heads ``[r * H / P, (r + 1) * H / P)``); here each rank computes only that slice.
"""

from __future__ import annotations

__all__ = ["head_range", "shard_heads", "session_ranges", "shard_sessions"]


def head_range(rank: int, world: int, num_heads: int) -> tuple[int, int]:
    """Heads ``[start, stop)`` owned by ``rank`` of ``world`` tensor-parallel ranks.

    The reference slices ``num_heads / tp_size`` heads per rank, so the head count must
    divide evenly; anything else is a configuration error.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if num_heads % world:
        raise ValueError(f"{num_heads} memory heads do not split over {world} ranks")
    per = num_heads // world
    return rank * per, (rank + 1) * per


def shard_heads(x, rank: int, world: int, dim: int):
    """View of ``x`` restricted to this rank's heads along ``dim`` (no copy)."""
    start, stop = head_range(rank, world, x.shape[dim])
    return x.narrow(dim, start, stop - start)


def session_ranges(lengths, world: int) -> list[tuple[int, int]]:
    """Split packed sessions into ``world`` contiguous ranges with balanced token counts.

    Range r ends at the session boundary nearest to ``r + 1`` world-ths of the total
    tokens, keeping every range non-empty (there must be at least ``world`` sessions).
    Work per range is proportional to its tokens (64-token tiles), so this balances the
    ranks.
    """
    lengths = [int(n) for n in lengths]
    if world < 1:
        raise ValueError("world must be positive")
    if len(lengths) < world:
        raise ValueError(f"{len(lengths)} sessions cannot fill {world} ranks")
    if any(n <= 0 for n in lengths):
        raise ValueError("session lengths must be positive")
    total = sum(lengths)
    ranges, start, acc = [], 0, 0
    for r in range(world):
        if r == world - 1:
            stop = len(lengths)
        else:
            target = total * (r + 1) / world
            limit = len(lengths) - (world - 1 - r)  # leave one session per later range
            stop = start
            while stop < limit and (stop == start or acc + lengths[stop] <= target):
                acc += lengths[stop]
                stop += 1
            if stop < limit and target - acc > acc + lengths[stop] - target:
                acc += lengths[stop]
                stop += 1
        ranges.append((start, stop))
        start = stop
    return ranges


def shard_sessions(lengths, rank: int, world: int):
    """(session range, token range, this rank's lengths) for ``rank``."""
    ranges = session_ranges(lengths, world)
    s0, s1 = ranges[rank]
    lengths = [int(n) for n in lengths]
    t0 = sum(lengths[:s0])
    t1 = t0 + sum(lengths[s0:s1])
    return (s0, s1), (t0, t1), lengths[s0:s1]
