"""Host-side tiling plan with the fields of the reference ``ChunkPlan``.

Mirrors ``models/qwen/ops/layout.py:18-216`` and ``models/qwen/ops/packed.py:16-31``
of the reference package (``inference/memt_sglang``) so that callers holding a plan
object keep working: write events every ``chunk_tokens`` inside each sample, 64-token
tiles inside each event, the read block of each tile and the per-sample tile offsets.
The update kernels do not consume this object (they build the same table on the
device from ``cu_seqlens``); ``memt_gdn2_read_fwd`` uses its read-block boundaries.
"""

from __future__ import annotations

from dataclasses import dataclass
from itertools import accumulate

import torch

WY_TILE_TOKENS = 64

__all__ = ["WY_TILE_TOKENS", "ChunkPlan", "boundaries", "build_chunk_plan", "packed_plan"]


def boundaries(lengths, device):
    """int32 [N+1] sample offsets (models/common/packed.py:8-9)."""
    return torch.tensor([0, *accumulate(lengths)], device=device, dtype=torch.int32)


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


def build_chunk_plan(turn_slice, sample_slice, wy_tile_tokens=WY_TILE_TOKENS, *, event_slice=None,
                     commit_mask=None) -> ChunkPlan:
    """Same tables as the reference builder (models/qwen/ops/layout.py:128-189)."""
    device = turn_slice.device
    read = turn_slice.detach().to("cpu", torch.int64)
    sample = sample_slice.detach().to("cpu", torch.int64)
    event = (turn_slice if event_slice is None else event_slice).detach().to("cpu", torch.int64)
    total = int(event[-1])
    event_len = event[1:] - event[:-1]
    n_chunk_per_event = (event_len + wy_tile_tokens - 1) // wy_tile_tokens
    n_event = int(event_len.numel())
    event_chunk_offsets = torch.cat((torch.zeros(1, dtype=torch.int64), torch.cumsum(n_chunk_per_event, 0)))
    num_chunk = int(event_chunk_offsets[-1])
    chunk_event = torch.repeat_interleave(torch.arange(n_event, dtype=torch.int64), n_chunk_per_event)
    chunk_sub = torch.arange(num_chunk, dtype=torch.int64) - event_chunk_offsets[chunk_event]
    chunk_tok0 = event[chunk_event] + chunk_sub * wy_tile_tokens
    chunk_len = torch.clamp(event[chunk_event + 1] - chunk_tok0, max=wy_tile_tokens)
    sample_chunk_offsets = event_chunk_offsets[torch.searchsorted(event, sample)]
    chunk_block_ids = torch.searchsorted(read, chunk_tok0, right=True) - 1
    chunk_is_block_start = chunk_tok0 == read[chunk_block_ids]
    if commit_mask is None:
        chunk_commits = torch.ones(num_chunk, dtype=torch.bool)
    else:
        chunk_commits = commit_mask.detach().to("cpu", torch.bool)[chunk_event]
    block_len = read[1:] - read[:-1]

    def dev(t, dtype=torch.int32):
        return t.to(device=device, dtype=dtype).contiguous()

    return ChunkPlan(
        wy_tile_tokens=wy_tile_tokens, num_event=n_event, num_block=int(read.numel()) - 1,
        num_sample=int(sample.numel()) - 1, num_chunk=num_chunk, total_tokens=total,
        event_slice=dev(event), chunk_indices=dev(torch.stack((chunk_event, chunk_sub), dim=-1)),
        sample_chunk_offsets=dev(sample_chunk_offsets), chunk_block_ids=dev(chunk_block_ids),
        chunk_is_block_start=dev(chunk_is_block_start), chunk_tok0=dev(chunk_tok0), chunk_len=dev(chunk_len),
        chunk_commits=dev(chunk_commits), read_slice=dev(read),
        max_block_tokens=int(block_len.max()) if block_len.numel() else 0,
    )


def packed_plan(lengths, device, *, chunk_tokens) -> ChunkPlan:
    """Write events every chunk_tokens inside each sample (models/qwen/ops/packed.py:16-31)."""
    samples = boundaries(lengths, device)
    events = [0]
    offset = 0
    for length in lengths:
        events.extend(offset + t for t in range(chunk_tokens, length, chunk_tokens))
        offset += length
        events.append(offset)
    event_slice = torch.tensor(events, device=device, dtype=torch.int32)
    commit_mask = torch.ones(len(events) - 1, device=device, dtype=torch.bool)
    return build_chunk_plan(samples, samples, event_slice=event_slice, commit_mask=commit_mask)
