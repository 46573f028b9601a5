"""B200 (sm_100a) GDN-2 memory hot path for MemT-1.0.

Drop-in operators for the reference plugin's operator layer (``token_memory_packed``,
``memt_gdn2_read_fwd``, ``snapshot_read``), the Qwen memory-block prologue, the fused decode
readout and the BASELINE-style ``gdn2_chunked`` entry, all over the C ABI in ``include/memt_gdn2.h``.
"""

from . import flash, shard, snapshots
from .layout import ChunkPlan, boundaries, build_chunk_plan, packed_plan
from .ops import (Workspace, gdn2_chunked, gdn2_update, memory_readout, memt_gdn2_read_fwd, qwen_prologue,
                  snapshot_read, token_memory_packed)

__all__ = [
    "ChunkPlan", "boundaries", "build_chunk_plan", "flash", "packed_plan", "Workspace", "gdn2_chunked", "gdn2_update",
    "memory_readout", "memt_gdn2_read_fwd", "qwen_prologue", "shard", "snapshot_read", "snapshots",
    "token_memory_packed",
]
