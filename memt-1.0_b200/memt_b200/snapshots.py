"""Memory snapshots of head-sharded states in the reference's ``memt-memory-v1`` file.

The reference replicates every memory head on every tensor-parallel rank and saves one
session's slot of its state pool as a safetensors file (``runtime/snapshots.py:34-103`` of
``inference/memt_sglang``): one fp32 tensor ``memory.<layer>`` of shape ``[1, H, K, V]`` per
memory layer, metadata ``{"format": "memt-memory-v1", "identity": <identity>}``, written to a
temporary file in the target directory, fsynced, then linked (or, with ``overwrite``, moved)
into place and the directory fsynced. Loading checks the metadata, the layer set, the dtype,
the shapes and that every value is finite before it changes any state; a file without tensors
means "no memory" and zeroes the slot.

Here each rank holds only its contiguous slice of heads (``memt_b200.shard.head_range``), so:

* ``save_memory_sharded`` gathers the slices of all ranks on rank 0 (``torch.distributed``
  gather, in rank order, which is head order), rank 0 writes the unchanged file, and every rank
  returns rank 0's result or raises its error;
* ``load_memory_sharded`` needs no collective: every rank reads the shared file, checks it
  whole, and keeps its own heads.

Files written here load in the reference and the reference's files load here.
"""

from __future__ import annotations

import os
import tempfile
from pathlib import Path

import torch

SNAPSHOT_FORMAT = "memt-memory-v1"

__all__ = ["SNAPSHOT_FORMAT", "save_memory_sharded", "load_memory_sharded", "load_into_pool"]


def _dist():
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist, dist.get_rank(), dist.get_world_size()
    return None, 0, 1


def _write_atomic(tensors, path: Path, metadata, overwrite):
    """The reference's atomic write: temporary file in the same directory, fsync, link or
    replace, fsync of the directory."""
    from safetensors.torch import save_file

    descriptor, temporary = tempfile.mkstemp(dir=path.parent, prefix=".memt-state-")
    os.close(descriptor)
    try:
        save_file(tensors, temporary, metadata=metadata)
        with open(temporary, "rb") as stream:
            os.fsync(stream.fileno())
        if overwrite:
            os.replace(temporary, path)
        else:
            os.link(temporary, path)  # never replace an existing file
        descriptor = os.open(path.parent, os.O_RDONLY)
        try:
            os.fsync(descriptor)
        finally:
            os.close(descriptor)
    finally:
        Path(temporary).unlink(missing_ok=True)


def save_memory_sharded(layers, path, *, identity, num_heads, head_range, overwrite=False, has_memory=True):
    """Save one session's memory, held as head slices across the ranks, as one snapshot file.

    layers: {layer id: this rank's fp32 state slice [1, h1 - h0, K, V] (or [h1 - h0, K, V])}, the
    same layer ids on every rank; head_range: (h0, h1) of this rank; num_heads: H of the layer.
    Collective over the default process group when one is initialised (every rank must call it);
    returns ``{"file", "format", "has_memory"}`` on every rank, as the reference's save_memory.
    """
    dist, rank, world = _dist()
    path = Path(path)
    h0, h1 = (int(x) for x in head_range)
    error = None
    gathered = {}
    names = sorted(layers)
    spans = [None] * world
    if dist is not None:
        dist.all_gather_object(spans, (h0, h1, names, bool(has_memory)))
    else:
        spans = [(h0, h1, names, bool(has_memory))]
    if any(s[2] != names or s[3] != bool(has_memory) for s in spans):
        error = "ranks hold different memory layer sets"
    elif sorted((s[0], s[1]) for s in spans) != [(s[0], s[1]) for s in spans] or spans[0][0] != 0 or \
            spans[-1][1] != num_heads or any(a[1] != b[0] for a, b in zip(spans, spans[1:])):
        error = "rank head ranges do not tile the heads in rank order"
    if error is None and has_memory:
        for layer in names:
            x = layers[layer].detach()
            x = x.reshape(1, h1 - h0, *x.shape[-2:]).float().contiguous()
            if dist is not None:
                parts = None
                if rank == 0:
                    parts = [torch.empty((1, s[1] - s[0], *x.shape[-2:]), dtype=x.dtype, device=x.device)
                             for s in spans]
                dist.gather(x, parts, dst=0)
                if rank == 0:
                    gathered[f"memory.{layer}"] = torch.cat(parts, dim=1).cpu().contiguous()
            else:
                gathered[f"memory.{layer}"] = x.cpu().contiguous()
    result = None
    if rank == 0 and error is None:
        try:
            _write_atomic(gathered if has_memory else {}, path, {"format": SNAPSHOT_FORMAT, "identity": identity},
                          overwrite)
            result = {"file": path.name, "format": SNAPSHOT_FORMAT, "has_memory": bool(has_memory)}
        except (OSError, ValueError) as e:  # a failed write is reported on every rank
            error = f"{type(e).__name__}: {e}"
    if dist is not None:
        box = [(result, error)]
        dist.broadcast_object_list(box, src=0)
        result, error = box[0]
    if error is not None:
        raise ValueError(f"memory snapshot not saved: {error}")
    return result


def load_memory_sharded(path, *, identity, layer_shapes, head_range):
    """Read and check a snapshot file; return ({layer: this rank's slice [1, h1 - h0, K, V]
    fp32 on the CPU}, has_memory). layer_shapes: {layer id: full shape (1, H, K, V)}.

    Raises ValueError, before anything is returned, on a wrong format or identity, a different
    layer set, a tensor that is not fp32 of the exact shape, or a non-finite value
    (the reference's checks, runtime/snapshots.py:67-97). A file without tensors means no
    memory: the slices are zeros.
    """
    from safetensors import SafetensorError, safe_open

    h0, h1 = (int(x) for x in head_range)
    try:
        with safe_open(str(path), framework="pt", device="cpu") as handle:
            if handle.metadata() != {"format": SNAPSHOT_FORMAT, "identity": identity}:
                raise ValueError("Snapshot model/encoding/format identity mismatch")
            names = {f"memory.{layer}": layer for layer in layer_shapes}
            keys = set(handle.keys())
            if keys and keys != names.keys():
                raise ValueError("Snapshot memory layer set mismatch")
            full = {layer: handle.get_tensor(name) for name, layer in names.items()} if keys else {}
    except SafetensorError as error:
        raise ValueError("Invalid memory snapshot") from error
    for layer, tensor in full.items():
        if (tensor.dtype != torch.float32 or tuple(tensor.shape) != tuple(layer_shapes[layer])
                or not torch.isfinite(tensor).all()):
            raise ValueError("Snapshot requires finite FP32 tensors with exact layer shapes")
    out = {}
    for layer, shape in layer_shapes.items():
        if not 0 <= h0 < h1 <= shape[1]:
            raise ValueError(f"head range {(h0, h1)} outside {shape[1]} heads")
        out[layer] = (full[layer][:, h0:h1].contiguous() if full
                      else torch.zeros((1, h1 - h0, *shape[2:]), dtype=torch.float32))
    return out, bool(full)


def load_into_pool(pool, slot, path, *, identity, num_heads, head_range):
    """Load a snapshot into slot ``slot`` of this rank's sharded state pool.

    pool: {layer id: fp32 [S, h1 - h0, K, V] or [S, 1, h1 - h0, K, V] device tensor}. The file
    is checked whole before any slot changes; returns has_memory like the reference's
    load_memory (runtime/snapshots.py:67-103).
    """
    h0, h1 = (int(x) for x in head_range)
    shapes = {layer: (1, num_heads, *t.shape[-2:]) for layer, t in pool.items()}
    slices, has_memory = load_memory_sharded(path, identity=identity, layer_shapes=shapes, head_range=(h0, h1))
    for layer, storage in pool.items():
        storage[slot].copy_(slices[layer].reshape(storage[slot].shape))
    return has_memory
