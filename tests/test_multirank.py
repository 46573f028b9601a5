"""Multi-rank sharding: heads (tensor parallel) and sessions (data parallel).

The GDN-2 path has no exchange step, so a sharded run must reproduce the unsharded one
exactly. CPU tests run two gloo ranks, each computing its shard with the oracle, gather
the shards and compare them with the full oracle run; they also check the bench's
max-over-ranks timing reduction. GPU tests run the shards through the C ABI on one
device and compare bit for bit with the unsharded call.
"""

import os
import socket

import numpy as np
import pytest
import torch

from memt_b200 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seed, lengths, H, D):
    rng = np.random.default_rng(seed)
    L = sum(lengths)
    q = rng.standard_normal((L, H, D))
    k = rng.standard_normal((L, H, D))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((L, H, D))
    g = np.broadcast_to(-np.logaddexp(0.0, -rng.normal(2.0, 0.5, (L, H, 1))), (L, H, D)).copy()
    b = np.broadcast_to(1 / (1 + np.exp(-rng.standard_normal((L, H, 1)))), (L, H, D)).copy()
    w = 1 / (1 + np.exp(-rng.standard_normal((L, H, D))))
    h0 = 0.02 * rng.standard_normal((len(lengths), H, D, D))
    r0 = 0.05 * rng.standard_normal((len(lengths), H, D, D))
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    return dict(q=q, k=k, v=v, g=g, b=b, w=w, h0=h0, r0=r0, cu=cu)


def _oracle(x, chunk_tokens=128):
    from oracle import gdn2 as O

    return O.chunked(x["q"], x["k"], x["v"], x["g"], x["h0"], x["r0"], x["cu"], 0.25, b=x["b"], w=x["w"],
                     chunk_tokens=chunk_tokens, mode="bf16")


LENGTHS, H, D = [70, 130, 33, 96], 4, 16


def _rank_main(rank, world, port, queue):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = _inputs(7, LENGTHS, H, D)

        # heads: this rank's slice of every per-head tensor
        h0, h1 = shard.head_range(rank, world, H)
        xs = {n: (a[:, h0:h1] if n != "cu" else a) for n, a in x.items()}
        o, s = _oracle(xs)
        parts = [None] * world
        dist.all_gather_object(parts, (o, s))
        heads = (np.concatenate([p[0] for p in parts], axis=1), np.concatenate([p[1] for p in parts], axis=1))

        # sessions: this rank's contiguous sessions, offsets rebased to its token range
        (s0, s1), (t0, t1), mine = shard.shard_sessions(LENGTHS, rank, world)
        xt = {n: x[n][t0:t1] for n in ("q", "k", "v", "g", "b", "w")}
        xt.update(h0=x["h0"][s0:s1], r0=x["r0"][s0:s1], cu=np.concatenate([[0], np.cumsum(mine)]))
        o, s = _oracle(xt)
        parts = [None] * world
        dist.all_gather_object(parts, (o, s))
        sessions = (np.concatenate([p[0] for p in parts], axis=0), np.concatenate([p[1] for p in parts], axis=0))

        # bench timing: every rank contributes its device time, rank 0 reports the max
        t = torch.tensor([1.0 + rank, 5.0 - rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            o, s = _oracle(x)
            err = [float(np.abs(a - b).max()) for a, b in ((heads[0], o), (heads[1], s), (sessions[0], o),
                                                           (sessions[1], s))]
            queue.put((err, t.tolist()))
    finally:
        dist.destroy_process_group()


def test_head_range_partitions_heads():
    for H_, world in [(16, 1), (16, 2), (16, 4), (16, 8), (128, 8), (4, 4)]:
        ranges = [shard.head_range(r, world, H_) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == H_
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert len({b - a for a, b in ranges}) == 1
    with pytest.raises(ValueError):
        shard.head_range(0, 3, 16)
    with pytest.raises(ValueError):
        shard.head_range(2, 2, 16)


def test_shard_heads_is_a_view():
    x = torch.arange(2 * 8 * 3).reshape(2, 8, 3)
    v = shard.shard_heads(x, 1, 4, 1)
    assert v.shape == (2, 2, 3) and v.data_ptr() == x[:, 2:4].data_ptr()


def test_session_ranges_balance_and_cover():
    rng = np.random.default_rng(3)
    for world in (1, 2, 4, 8):
        lengths = rng.integers(1024, 32768, 32).tolist()  # varlen long-history config
        ranges = shard.session_ranges(lengths, world)
        assert ranges[0][0] == 0 and ranges[-1][1] == len(lengths)
        assert all(a[1] == b[0] and a[0] < a[1] for a, b in zip(ranges, ranges[1:]))
        loads = [sum(lengths[a:b]) for a, b in ranges]
        assert max(loads) - sum(lengths) / world <= max(lengths)
    assert shard.session_ranges([5, 1, 1], 3) == [(0, 1), (1, 2), (2, 3)]
    with pytest.raises(ValueError):
        shard.session_ranges([5, 1], 3)
    with pytest.raises(ValueError):
        shard.session_ranges([5, 0, 2], 2)


def test_gloo_two_ranks_match_unsharded():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.SimpleQueue()
    procs = mp.start_processes(_rank_main, args=(2, _free_port(), queue), nprocs=2, join=False,
                               start_method="spawn")
    while not procs.join(timeout=1):
        pass
    err, t = queue.get()
    assert max(err) < 1e-12, err
    assert t == [2.0, 5.0]


# ---------------------------------------------------------------------------
# GPU: sharded calls through the C ABI reproduce the unsharded call bit for bit
# ---------------------------------------------------------------------------

def _gpu_inputs(dev, lengths, H_, D_):
    gen = torch.Generator(device=dev).manual_seed(11)
    L = sum(lengths)
    bf = torch.bfloat16

    def nrm(t):
        return (t / t.norm(dim=-1, keepdim=True)).to(bf)

    return dict(
        q=nrm(torch.randn(L, H_, D_, device=dev, generator=gen)),
        k=nrm(torch.randn(L, H_, D_, device=dev, generator=gen)),
        v=torch.randn(L, H_, D_, device=dev, generator=gen).to(bf),
        g=torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L, H_, device=dev, generator=gen)),
        beta=torch.sigmoid(torch.randn(L, H_, device=dev, generator=gen)).to(bf),
        w=torch.sigmoid(torch.randn(L, H_, D_, device=dev, generator=gen)).to(bf),
        h0=0.02 * torch.randn(len(lengths), H_, D_, D_, device=dev, generator=gen),
        cu=torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev),
    )


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_gpu_head_shards_equal_full(cuda, world):
    import memt_b200 as M

    lengths, H_, D_ = [300, 1000, 64, 2100], 8, 128
    x = _gpu_inputs(cuda, lengths, H_, D_)
    o, s = M.gdn2_chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["h0"], x["cu"], w=x["w"],
                          max_seqlen=max(lengths), chunk_tokens=512)
    for r in range(world):
        h0, h1 = shard.head_range(r, world, H_)
        xs = {n: (shard.shard_heads(t, r, world, 1) if n != "cu" else t) for n, t in x.items()}
        o_r, s_r = M.gdn2_chunked(xs["q"], xs["k"], xs["v"], xs["g"], xs["beta"], xs["h0"], xs["cu"], w=xs["w"],
                                  max_seqlen=max(lengths), chunk_tokens=512)
        torch.cuda.synchronize()
        assert torch.equal(o_r, o[:, h0:h1]), r
        assert torch.equal(s_r, s[:, h0:h1]), r


@pytest.mark.gpu
def test_gpu_session_shards_equal_full(cuda):
    import memt_b200 as M

    lengths, H_, D_, world = [700, 130, 2048, 64, 999, 1500], 4, 128, 3
    x = _gpu_inputs(cuda, lengths, H_, D_)
    o, s = M.gdn2_chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["h0"], x["cu"], w=x["w"],
                          max_seqlen=max(lengths), chunk_tokens=256)
    for r in range(world):
        (s0, s1), (t0, t1), mine = shard.shard_sessions(lengths, r, world)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(mine)]), dtype=torch.int32, device=cuda)
        tok = {n: x[n][t0:t1] for n in ("q", "k", "v", "g", "beta", "w")}
        o_r, s_r = M.gdn2_chunked(tok["q"], tok["k"], tok["v"], tok["g"], tok["beta"], x["h0"][s0:s1], cu,
                                  w=tok["w"], max_seqlen=max(mine), chunk_tokens=256)
        torch.cuda.synchronize()
        assert torch.equal(o_r, o[t0:t1]), r
        assert torch.equal(s_r, s[s0:s1]), r


@pytest.mark.gpu
def test_gpu_readout_head_offset_shards(cuda):
    """Each tensor-parallel rank writes its heads' gated readout into its own columns of
    the attention output (head_offset); the union equals the unsharded readout."""
    import memt_b200 as M

    gen = torch.Generator(device=cuda).manual_seed(5)
    bf = torch.bfloat16
    lengths, H_, D_, world = [1, 3, 1, 40, 2], 8, 128, 4
    L = sum(lengths)
    q = torch.randn(L, H_, D_, device=cuda, generator=gen).to(bf)
    gate = torch.randn(L, H_, D_, device=cuda, generator=gen).to(bf)
    states = 0.05 * torch.randn(len(lengths), H_, D_, D_, device=cuda, generator=gen)
    wt = (1.0 + 0.1 * torch.randn(D_, device=cuda, generator=gen)).to(bf)
    attn = torch.randn(L, H_ * D_, device=cuda, generator=gen).to(bf)
    full = M.memory_readout(q, states, lengths, D_ ** -0.5, gate, wt, softcap=10.0, residual=attn,
                            out=torch.empty_like(attn))
    out = attn.clone()
    for r in range(world):
        h0, _ = shard.head_range(r, world, H_)
        M.memory_readout(shard.shard_heads(q, r, world, 1), shard.shard_heads(states, r, world, 1), lengths,
                         D_ ** -0.5, shard.shard_heads(gate, r, world, 1), wt, softcap=10.0, residual=out, out=out,
                         head_offset=h0)
    torch.cuda.synchronize()
    assert torch.equal(out, full)
