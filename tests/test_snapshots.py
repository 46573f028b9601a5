"""Snapshot export / import of head-sharded states in the reference's memt-memory-v1 file.

The reference saves a slot of its (head-replicated) state pool as safetensors with one fp32
``memory.<layer>`` tensor [1, H, K, V] per layer and {"format", "identity"} metadata
(runtime/snapshots.py:34-103 of inference/memt_sglang). Two gloo ranks on CPU each hold half
of the heads: the file they save together must be the one the reference would write for the
full state, and loading it back must give every rank its own heads. Invalid files are rejected
before any slot changes.
"""

import os
import socket

import numpy as np
import pytest
import torch

from memt_b200 import shard, snapshots

IDENTITY = '{"model": "test", "encoding": "x"}'
LAYERS = {3: (1, 4, 8, 8), 7: (1, 4, 8, 8)}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_states(seed=0):
    g = torch.Generator().manual_seed(seed)
    return {layer: torch.randn(*shape, generator=g) for layer, shape in LAYERS.items()}


def _rank_main(rank, world, port, directory, queue):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _full_states()
        h0, h1 = shard.head_range(rank, world, 4)
        mine = {layer: t[:, h0:h1].clone() for layer, t in full.items()}
        path = os.path.join(directory, "s1.safetensors")
        res = snapshots.save_memory_sharded(mine, path, identity=IDENTITY, num_heads=4, head_range=(h0, h1))
        # saving again without overwrite fails on every rank (the reference never replaces a key)
        try:
            snapshots.save_memory_sharded(mine, path, identity=IDENTITY, num_heads=4, head_range=(h0, h1))
            again = "saved"
        except ValueError:
            again = "refused"
        # a sharded pool [S, heads of this rank, K, V]: load into slot 2
        pool = {layer: torch.zeros(5, h1 - h0, 8, 8) for layer in LAYERS}
        has = snapshots.load_into_pool(pool, 2, path, identity=IDENTITY, num_heads=4, head_range=(h0, h1))
        ok = all(torch.equal(pool[layer][2], full[layer][0, h0:h1]) for layer in LAYERS)
        untouched = all(not pool[layer][[0, 1, 3, 4]].any() for layer in LAYERS)
        queue.put((rank, res, again, has, ok, untouched))
    finally:
        dist.destroy_process_group()


def test_two_ranks_save_the_reference_file_and_load_their_heads(tmp_path):
    import torch.multiprocessing as mp

    from safetensors import safe_open

    ctx = mp.get_context("spawn")
    queue = ctx.SimpleQueue()
    procs = mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path), queue), nprocs=2, join=False,
                               start_method="spawn")
    procs.join(timeout=120)
    results = sorted(queue.get() for _ in range(2))
    for rank, res, again, has, ok, untouched in results:
        assert res == {"file": "s1.safetensors", "format": "memt-memory-v1", "has_memory": True}
        assert again == "refused" and has and ok and untouched
    full = _full_states()
    with safe_open(str(tmp_path / "s1.safetensors"), framework="pt", device="cpu") as f:
        assert f.metadata() == {"format": "memt-memory-v1", "identity": IDENTITY}
        assert set(f.keys()) == {"memory.3", "memory.7"}
        for layer in LAYERS:
            t = f.get_tensor(f"memory.{layer}")
            assert t.dtype == torch.float32 and torch.equal(t, full[layer])
    assert not [p for p in os.listdir(tmp_path) if p.startswith(".memt-state-")]  # no temporary left


def _reference_style_file(path, tensors, metadata):
    """A file as the reference's save_memory writes it (safetensors save_file)."""
    from safetensors.torch import save_file

    save_file(tensors, str(path), metadata=metadata)


def test_load_checks_the_file_before_changing_state(tmp_path):
    full = _full_states(1)
    good = {f"memory.{layer}": t for layer, t in full.items()}
    meta = {"format": "memt-memory-v1", "identity": IDENTITY}
    _reference_style_file(tmp_path / "ok.safetensors", good, meta)
    pool = {layer: torch.full((3, 2, 8, 8), 7.0) for layer in LAYERS}
    assert snapshots.load_into_pool(pool, 1, tmp_path / "ok.safetensors", identity=IDENTITY, num_heads=4,
                                    head_range=(2, 4))
    assert torch.equal(pool[3][1], full[3][0, 2:4])
    before = {layer: t.clone() for layer, t in pool.items()}
    bad_cases = {
        "identity": (good, {"format": "memt-memory-v1", "identity": "other"}),
        "format": (good, {"format": "memt-memory-v2", "identity": IDENTITY}),
        "layers": ({"memory.3": full[3]}, meta),
        "dtype": ({k: v.double() for k, v in good.items()}, meta),
        "shape": ({k: v[:, :3].contiguous() for k, v in good.items()}, meta),
        "finite": ({k: (v.clone().index_fill_(1, torch.tensor([0]), float("nan"))) for k, v in good.items()}, meta),
    }
    for name, (tensors, metadata) in bad_cases.items():
        p = tmp_path / f"{name}.safetensors"
        _reference_style_file(p, tensors, metadata)
        with pytest.raises(ValueError):
            snapshots.load_into_pool(pool, 0, p, identity=IDENTITY, num_heads=4, head_range=(2, 4))
        assert all(torch.equal(pool[layer], before[layer]) for layer in LAYERS), name
    (tmp_path / "junk.safetensors").write_bytes(b"not a safetensors file")
    with pytest.raises(ValueError):
        snapshots.load_into_pool(pool, 0, tmp_path / "junk.safetensors", identity=IDENTITY, num_heads=4,
                                 head_range=(2, 4))


def test_a_file_without_memory_zeroes_the_slot(tmp_path):
    res = snapshots.save_memory_sharded({layer: torch.ones(1, 4, 8, 8) for layer in LAYERS},
                                        tmp_path / "empty.safetensors", identity=IDENTITY, num_heads=4,
                                        head_range=(0, 4), has_memory=False)
    assert res["has_memory"] is False
    pool = {layer: torch.ones(2, 4, 8, 8) for layer in LAYERS}
    assert not snapshots.load_into_pool(pool, 1, tmp_path / "empty.safetensors", identity=IDENTITY, num_heads=4,
                                        head_range=(0, 4))
    assert all(not pool[layer][1].any() and pool[layer][0].all() for layer in LAYERS)


def test_single_process_save_matches_full_state(tmp_path):
    full = _full_states(2)
    snapshots.save_memory_sharded(full, tmp_path / "one.safetensors", identity=IDENTITY, num_heads=4,
                                  head_range=(0, 4))
    slices, has = snapshots.load_memory_sharded(tmp_path / "one.safetensors", identity=IDENTITY,
                                                layer_shapes=LAYERS, head_range=(1, 3))
    assert has and all(torch.equal(slices[layer], full[layer][:, 1:3]) for layer in LAYERS)
    with pytest.raises(ValueError):  # ranges that do not tile the heads
        snapshots.save_memory_sharded(full, tmp_path / "two.safetensors", identity=IDENTITY, num_heads=8,
                                      head_range=(0, 4))
    assert np.all([not (tmp_path / "two.safetensors").exists()])
