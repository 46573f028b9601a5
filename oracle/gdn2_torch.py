"""fp32 PyTorch CPU restatement of the GDN-2 chunked update and snapshot read.

TEST AND BASELINE INFRASTRUCTURE ONLY. Nothing in the product imports this module: only
``tests/`` and ``bench.py``'s CPU legs (the timed CPU baseline and ``--impl reference``) do.

The reference has no CPU implementation of its memory update (its kernels are Triton only),
so this is the CPU baseline: the same chunked WY algorithm, in the reference kernel order,
vectorised with PyTorch over all (sample, chunk, head) tiles and run on every host thread.
Paths are relative to the reference package ``inference/memt_sglang``:

* cumulative log2 decay inside each 64-token tile          _vendor/fla/ops/utils/cumsum.py:116-133
* key-key scores A[i,j] = sum_c k_ic k_jc 2^(G_ic - G_jc), j < i, with the decay taken
  relative to a reference point (the tile's middle token) so that both factors stay finite
                                                           _vendor/fla/ops/gdn2/chunk_intra.py:233-299
* (I + A)^-1 by a batched triangular solve                 _vendor/fla/ops/gdn2/chunk_intra.py:326-395
* u = A^-1 (w * v), w_wy = A^-1 (k * 2^G), kg = k * 2^(G_last - G)
                                                           _vendor/fla/ops/gdn2/wy_fast.py:92-142
* sequential inter-chunk scan  v_new = u - w_wy S,  S <- 2^G_last * S + kg^T v_new
                                                           models/qwen/ops/_triton/state.py:76-115
* read  o = scale * q S_in                                 models/qwen/ops/_triton/read.py:40-71

All arithmetic is fp32 (no bf16 rounding points). Samples are padded to whole tiles with zero
keys, values and log-decay, which leaves the state unchanged; write events of ``chunk_tokens``
tokens restart the tiling only where they are not tile multiples, so ``chunk_tokens`` must be a
multiple of 64 here.
"""

from __future__ import annotations

import torch

RCP_LN2 = 1.4426950216  # _vendor/fla/ops/utils/constant.py:10
TILE = 64


def _pad_tiles(x, cu, nt):
    """[L, H, ...] -> [N, nt*64, H, ...] zero-padded per sample."""
    N = len(cu) - 1
    out = x.new_zeros((N, nt * TILE) + tuple(x.shape[1:]))
    for n in range(N):
        a, b = int(cu[n]), int(cu[n + 1])
        out[n, :b - a] = x[a:b]
    return out


@torch.no_grad()
def chunked_update(k, v, g, h0, cu, *, w=None, chunk_tokens=2048):
    """Final states [N, H, K, V] of the GDN-2 update (k already carries sqrt(beta) and erase).

    k, v: [L, H, D]; g: natural-log decay [L, H] or [L, H, D]; w: write gate [L, H, D] or None;
    h0: [N, H, D, D]; cu: host sequence of N + 1 offsets. fp32 throughout.
    """
    if chunk_tokens % TILE:
        raise ValueError("the CPU restatement needs chunk_tokens to be a multiple of 64")
    f = torch.float32
    L, H, D = k.shape
    N = len(cu) - 1
    nt = max((int(cu[n + 1]) - int(cu[n]) + TILE - 1) // TILE for n in range(N))
    if g.dim() == 2:
        g = g[:, :, None].expand(L, H, D)
    vv = v.to(f) * (w.to(f) if w is not None else 1.0)
    # [N, nt, 64, H, D] -> [N, nt, H, 64, D]
    kt = _pad_tiles(k.to(f), cu, nt).view(N, nt, TILE, H, D).transpose(2, 3)
    vt = _pad_tiles(vv, cu, nt).view(N, nt, TILE, H, D).transpose(2, 3)
    gt = _pad_tiles(g.to(f), cu, nt).view(N, nt, TILE, H, D).transpose(2, 3)
    G = torch.cumsum(gt * RCP_LN2, dim=3)                      # log2 cumulative decay in the tile
    Gm = G[:, :, :, TILE // 2 - 1:TILE // 2]                    # reference point
    kp = kt * torch.exp2(G - Gm)
    km = kt * torch.exp2(Gm - G)
    A = torch.tril(kp @ km.transpose(-1, -2), diagonal=-1)      # [N, nt, H, 64, 64]
    eye = torch.eye(TILE, dtype=f)
    T = torch.linalg.solve_triangular(A + eye, eye.expand_as(A), upper=False, unitriangular=True)
    u = T @ vt                                                  # [N, nt, H, 64, D]
    ww = T @ (kt * torch.exp2(G))
    Glast = G[:, :, :, -1:]
    kg = kt * torch.exp2(Glast - G)
    decay = torch.exp2(Glast[:, :, :, 0, :])                    # [N, nt, H, D]
    S = h0.to(f).clone()                                        # [N, H, D, D]
    for c in range(nt):
        vn = u[:, c] - ww[:, c] @ S
        S = decay[:, c, :, :, None] * S + kg[:, c].transpose(-1, -2) @ vn
    return S


@torch.no_grad()
def read(q, states, cu, scale):
    """o[t] = scale * q[t] . S_in[block(t)] in fp32: [L, H, D]."""
    out = torch.empty(q.shape[0], q.shape[1], states.shape[-1], dtype=torch.float32)
    for n in range(len(cu) - 1):
        a, b = int(cu[n]), int(cu[n + 1])
        out[a:b] = torch.einsum("thk,hkv->thv", q[a:b].float(), states[n].float()) * scale
    return out
