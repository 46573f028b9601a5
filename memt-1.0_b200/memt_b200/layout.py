"""Host-side tiling plan with the fields of the reference ``ChunkPlan``.

The field list of ``ChunkPlan`` is the reference's interface (``models/qwen/ops/layout.py:18-44``
of ``inference/memt_sglang``) so callers holding a plan object keep working; the tables are
built here by one forward walk over the offsets, the same walk the device plan kernel
(``csrc/plan.cuh``) and ``memt_gdn2_count_chunks`` make: write events every ``chunk_tokens``
inside each sample (``models/qwen/ops/packed.py:16-31``), 64-token tiles inside each event,
the read block that holds each tile's first token and the first tile of every sample.

The update kernels do not consume this object (they build their chunk table on the device
from ``cu_seqlens``); ``memt_gdn2_read_fwd`` uses its read-block boundaries.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

WY_TILE_TOKENS = 64

__all__ = ["WY_TILE_TOKENS", "ChunkPlan", "boundaries", "build_chunk_plan", "packed_plan", "read_segments"]


def _offsets(lengths):
    out = [0]
    for n in lengths:
        out.append(out[-1] + int(n))
    return out


def boundaries(lengths, device):
    """int32 [N+1] sample offsets (the reference's ``boundaries``, models/common/packed.py:8-9)."""
    return torch.tensor(_offsets(lengths), device=device, dtype=torch.int32)


@dataclass(frozen=True, slots=True)
class ChunkPlan:
    wy_tile_tokens: int
    num_event: int
    num_block: int
    num_sample: int
    num_chunk: int
    total_tokens: int
    event_slice: torch.Tensor
    chunk_indices: torch.Tensor
    sample_chunk_offsets: torch.Tensor
    chunk_block_ids: torch.Tensor
    chunk_is_block_start: torch.Tensor
    chunk_tok0: torch.Tensor
    chunk_len: torch.Tensor
    chunk_commits: torch.Tensor
    read_slice: torch.Tensor  # [num_block + 1] token offsets of the read blocks
    max_block_tokens: int


def _host_list(x):
    if isinstance(x, torch.Tensor):
        return [int(v) for v in x.detach().to("cpu", torch.int64).tolist()]
    return [int(v) for v in x]


def _tables(read, sample, event, tile, commits):
    """One walk over the event offsets. Every argument is a host list; returns host lists."""
    tok0, length, ev_of, sub_of, block_of, block_start, commit_of = [], [], [], [], [], [], []
    first_chunk_of_event = []
    block = 0
    last_read = len(read) - 1
    for e in range(len(event) - 1):
        lo, hi = event[e], event[e + 1]
        first_chunk_of_event.append(len(tok0))
        for sub, t in enumerate(range(lo, hi, tile)):
            # read block holding token t: the last read offset <= t (t never decreases)
            while block < last_read and read[block + 1] <= t:
                block += 1
            tok0.append(t)
            length.append(min(tile, hi - t))
            ev_of.append(e)
            sub_of.append(sub)
            block_of.append(block)
            block_start.append(t == read[block])
            commit_of.append(commits[e] if commits is not None else True)
    first_chunk_of_event.append(len(tok0))
    # first tile of each sample: the tiles of the first event starting at or after its offset
    sample_first, e = [], 0
    for s in sample:
        while e < len(event) - 1 and event[e] < s:
            e += 1
        sample_first.append(first_chunk_of_event[e])
    return tok0, length, ev_of, sub_of, block_of, block_start, commit_of, sample_first


def _plan_from_lists(read, sample, event, tile, commits, device) -> ChunkPlan:
    tok0, length, ev_of, sub_of, block_of, block_start, commit_of, sample_first = _tables(
        read, sample, event, tile, commits)

    def dev(values, dtype=torch.int32):
        return torch.tensor(values, dtype=torch.int64).to(device=device, dtype=dtype).contiguous()

    pairs = torch.tensor(list(zip(ev_of, sub_of)), dtype=torch.int64).reshape(-1, 2)
    block_len = [b - a for a, b in zip(read[:-1], read[1:])]
    return ChunkPlan(
        wy_tile_tokens=tile, num_event=len(event) - 1, num_block=len(read) - 1, num_sample=len(sample) - 1,
        num_chunk=len(tok0), total_tokens=event[-1], event_slice=dev(event),
        chunk_indices=pairs.to(device=device, dtype=torch.int32).contiguous(),
        sample_chunk_offsets=dev(sample_first), chunk_block_ids=dev(block_of),
        chunk_is_block_start=dev(block_start), chunk_tok0=dev(tok0), chunk_len=dev(length),
        chunk_commits=dev(commit_of), read_slice=dev(read),
        max_block_tokens=max(block_len) if block_len else 0,
    )


def build_chunk_plan(turn_slice, sample_slice, wy_tile_tokens=WY_TILE_TOKENS, *, event_slice=None,
                     commit_mask=None) -> ChunkPlan:
    """Plan for read blocks ``turn_slice``, samples ``sample_slice`` and write events
    ``event_slice`` (default: the read blocks), all offset tensors; the same tables as the
    reference builder (models/qwen/ops/layout.py:47-149)."""
    device = turn_slice.device
    read = _host_list(turn_slice)
    sample = _host_list(sample_slice)
    event = _host_list(turn_slice if event_slice is None else event_slice)
    commits = None if commit_mask is None else [bool(c) for c in commit_mask.detach().to("cpu").tolist()]
    return _plan_from_lists(read, sample, event, wy_tile_tokens, commits, device)


def packed_plan(lengths, device, *, chunk_tokens) -> ChunkPlan:
    """Commit plan: write events every ``chunk_tokens`` inside each sample, all committed
    (the reference's packed_plan, models/qwen/ops/packed.py:16-31)."""
    samples = _offsets(lengths)
    events = []
    for lo, hi in zip(samples[:-1], samples[1:]):
        events.extend(range(lo, hi, chunk_tokens))
    events.append(samples[-1])
    return _plan_from_lists(samples, samples, events, WY_TILE_TOKENS, [True] * (len(events) - 1), device)


def read_segments(plan):
    """(cu [M+1], block ids [M], longest segment) of the token runs that read one snapshot.

    Works on this module's plans and on the reference's own ``ChunkPlan`` (which has no
    ``read_slice``): each chunk reads the snapshot ``chunk_block_ids`` names
    (models/qwen/ops/_triton/read.py:40-50), so consecutive chunks of one block form one
    segment. Offsets and ids are host lists; this copies the plan's small tables to the host.
    """
    tok0 = _host_list(plan.chunk_tok0)
    ids = _host_list(plan.chunk_block_ids)
    cu, seg_ids = [], []
    for t, b in zip(tok0, ids):
        if not seg_ids or b != seg_ids[-1]:
            cu.append(t)
            seg_ids.append(b)
    cu.append(int(plan.total_tokens))
    longest = max((b - a for a, b in zip(cu[:-1], cu[1:])), default=0)
    return cu, seg_ids, longest
