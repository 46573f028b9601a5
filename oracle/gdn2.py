"""CPU oracle for the MemT-1.0 GDN-2 memory hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product imports this module: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg do,
and there only as the checker (or, for the CPU baseline, as the timed restatement).

It restates, in numpy, the reference's algorithm for the memory path:

* ``recurrence``      exact token-by-token gated delta rule in float64 (ground truth).
* ``chunked``         the chunked WY algorithm in the reference kernel order:
    - per-64-token tile cumulative log2 decay       R/.../_vendor/fla/ops/utils/cumsum.py:116-133
    - diagonal 16x16 key-key blocks, exact exponents  .../gdn2/chunk_intra_token_parallel.py:106-132
    - off-diagonal blocks with a per-sub-chunk reference point (tf32 dots on GPU)
                                                      .../gdn2/chunk_intra.py:233-299
    - blocked unit-lower-triangular inverse           .../gdn2/chunk_intra.py:326-395
    - WY operands u, w and the tail-decayed key kg    .../gdn2/wy_fast.py:92-142
    - sequential inter-chunk fp32 state scan          models/qwen/ops/_triton/state.py:76-115
  ``mode="exact"`` evaluates it in float64 with no rounding (mathematically equal to
  the recurrence). ``mode="bf16"`` rounds at every point where the reference's GPU
  path rounds: bf16 storage of A^-1, u, w, kg, the bf16 casts of the state and of
  v_new before the tensor-core products, tf32 inputs of the solve and of the
  off-diagonal score dots, fp32 storage of the cumulative decay and of the state.
* ``read``            o = scale * q . S_in, reading the incoming snapshot of the sample
                      (models/qwen/ops/_triton/read.py:40-71; models/deepseek/ops/read.py:6-31).
* ``gated_rms_norm``  w * bf16(x rsqrt(mean x^2 + eps)) * L tanh(SiLU(gate)/L)
                      (models/qwen/layer.py:15-31).
* ``l2norm``          x / sqrt(sum x^2 + eps)   (_vendor/fla/modules/l2norm.py:95-109).
* ``qwen_gates``, ``qwen_prologue``  gates, decay and the symmetric q/k inputs of the Qwen
                      memory block (models/qwen/layer.py:71-97).
* ``latent_rms_norm``, ``expand_grouped_qkv``, ``memory_inject``  the DeepSeek block's grouped
                      low-rank q/k/v expansion and wo_a injection
                      (models/deepseek/ops/compiled_tensor_ops.py:12-41, integration.py:56-72).
* ``plan_chunks``     write events every ``chunk_tokens`` inside each sample, 64-token tiles
                      inside each event (models/qwen/ops/packed.py:16-31, ops/layout.py:128-189).

Paths are relative to the reference package ``inference/memt_sglang``. The oracle is
pinned against the reference's own outputs by the fixtures in ``tests/golden``.
"""

from __future__ import annotations

import numpy as np

RCP_LN2 = np.float32(1.4426950216)  # _vendor/fla/ops/utils/constant.py:10
TILE = 64  # models/common/constants.py:3 (WY_TILE_TOKENS)
SUB = 16  # sub-chunk of the blocked solve, gdn2/chunk_intra.py:710


# ---------------------------------------------------------------------------
# rounding helpers
# ---------------------------------------------------------------------------

def r32(x):
    """Round to float32 (kept as float64 for further exact arithmetic)."""
    return np.asarray(x, np.float64).astype(np.float32).astype(np.float64)


def bf16(x):
    """Round to bfloat16, nearest-even, via float32 (as the GPU casts an fp32 value)."""
    f = np.ascontiguousarray(np.asarray(x, np.float64).astype(np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


def tf32(x):
    """Round to tf32 (10-bit mantissa), nearest with ties away from zero (cvt.rna.tf32.f32)."""
    f = np.ascontiguousarray(np.asarray(x, np.float64).astype(np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x1000) & 0xFFFFE000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


def _id(x):
    return np.asarray(x, np.float64)


def rel_fro(a, b):
    """Relative Frobenius error ||a-b|| / ||b||."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (nb if nb > 0 else 1.0))


# ---------------------------------------------------------------------------
# plan
# ---------------------------------------------------------------------------

def plan_chunks(cu_seqlens, chunk_tokens, tile=TILE):
    """Chunk table [(sample, tok0, len)] in scan order.

    Each sample is cut into write events of at most ``chunk_tokens`` tokens
    (models/qwen/ops/packed.py:16-31) and each event into ``tile``-token chunks, the
    last one partial (models/qwen/ops/layout.py:142-158).
    """
    cu = [int(x) for x in cu_seqlens]
    out = []
    for n in range(len(cu) - 1):
        bos, eos = cu[n], cu[n + 1]
        events = list(range(bos, eos, chunk_tokens)) + [eos]
        for e0, e1 in zip(events[:-1], events[1:]):
            for t0 in range(e0, e1, tile):
                out.append((n, t0, min(tile, e1 - t0)))
    return out


# ---------------------------------------------------------------------------
# ground truth: token recurrence
# ---------------------------------------------------------------------------

def recurrence(k, v, g, h0, cu_seqlens, *, b=None, w=None):
    """Exact gated delta rule, float64. Shapes: k,g,b [L,H,K]; v,w [L,H,V]; h0 [N,H,K,V].

    S~ = diag(exp g_t) S;  delta = w*v - S~^T (b*k);  S = S~ + k delta^T.
    Returns the final state [N,H,K,V] (float64).
    """
    k = _id(k)
    v = _id(v)
    a = np.exp(_id(g))
    kb = k if b is None else k * _id(b)
    wv = v if w is None else v * _id(w)
    out = _id(h0).copy()
    cu = [int(x) for x in cu_seqlens]
    for n in range(len(cu) - 1):
        S = out[n]
        for t in range(cu[n], cu[n + 1]):
            S = a[t][:, :, None] * S
            delta = wv[t] - np.einsum("hkv,hk->hv", S, kb[t])
            S = S + k[t][:, :, None] * delta[:, None, :]
        out[n] = S
    return out


# ---------------------------------------------------------------------------
# chunked WY algorithm in the reference kernel order
# ---------------------------------------------------------------------------

def _gather_chunks(x, chunks, tile=TILE):
    """[L,H,D] -> [NC,H,tile,D], zero padded beyond each chunk's length."""
    L, H, D = x.shape
    NC = len(chunks)
    out = np.zeros((NC, tile, H, D), np.float64)
    for c, (_, t0, ln) in enumerate(chunks):
        out[c, :ln] = x[t0:t0 + ln]
    return out.transpose(0, 2, 1, 3)


def intra(k, g, v, chunks, *, b=None, w=None, mode="exact", exact_scores=False):
    """Per-chunk WY operands. Returns dict with G, Ainv, u, w_wy, kg, g_last (all [NC,H,...]).

    Follows the reference's GPU algorithm; ``mode`` selects exact float64 or the
    GPU rounding points (see module docstring). ``exact_scores`` drops the tf32 rounding of
    the off-diagonal score operands (the sm_100a kernel's evaluation for a per-head decay:
    exact products scaled by 2^(G_i - G_j)); the default is the reference's.
    """
    emu = mode == "bf16"
    rb = bf16 if emu else _id
    rt = tf32 if emu else _id
    rf = r32 if emu else _id
    L, H, K = k.shape
    kc = _gather_chunks(_id(k), chunks)  # [NC,H,T,K]
    gc = _gather_chunks(_id(g), chunks)
    bc = None if b is None else _gather_chunks(_id(b), chunks)
    vc = _gather_chunks(_id(v), chunks)
    wc = None if w is None else _gather_chunks(_id(w), chunks)
    NC = kc.shape[0]
    T = TILE
    lens = np.array([ln for (_, _, ln) in chunks])
    valid = (np.arange(T)[None, :] < lens[:, None])  # [NC,T]
    vmask = valid[:, None, :, None]

    # cumulative log2 decay inside the tile: cumsum then * 1/ln2 (cumsum.py:126-133)
    G = rf(np.cumsum(gc, axis=2) * np.float64(RCP_LN2))
    kb = kc if bc is None else kc * bc  # fp32 product in the score kernels

    # --- key-key scores Akk (strictly lower) ---
    A = np.zeros((NC, H, T, T), np.float64)
    for r in range(T // SUB):
        rows = slice(r * SUB, (r + 1) * SUB)
        # diagonal block: exact per-pair exponents (token_parallel.py:114-123)
        Gi = G[:, :, rows, None, :]
        Gj = G[:, :, None, rows, :]
        blk = np.einsum("nhic,nhjc,nhijc->nhij", kb[:, :, rows], kc[:, :, rows], np.exp2(Gi - Gj))
        blk = np.tril(blk, -1)
        A[:, :, rows, rows] = rf(blk)
        if r == 0:
            continue
        # off-diagonal blocks: reference point = first token of the row sub-chunk
        # (chunk_intra.py:251-253, 267-271, 287-297)
        gn = G[:, :, r * SUB, :][:, :, None, :]  # [NC,H,1,K]
        rs = _id if exact_scores else rt
        left = rs(kb[:, :, rows] * np.exp2(G[:, :, rows] - gn)) * vmask[:, :, rows]
        cols = slice(0, r * SUB)
        right = rs(kc[:, :, cols] * np.exp2(gn - G[:, :, cols]))
        A[:, :, rows, cols] = rf(np.einsum("nhic,nhjc->nhij", left, right))
    # rows of sub-chunks that start beyond the chunk length are skipped by the kernel
    A *= valid[:, None, :, None]

    # --- blocked inverse of (I + A) (chunk_intra.py:326-395) ---
    nb = T // SUB
    Ai = [[None] * nb for _ in range(nb)]
    eye = np.eye(SUB)
    for r in range(nb):
        blk = A[:, :, r * SUB:(r + 1) * SUB, r * SUB:(r + 1) * SUB]
        X = -np.tril(blk, -1)
        for i in range(2, SUB):
            a = -blk[:, :, i, :].copy()
            a[:, :, i:] = 0.0
            a = a + np.einsum("nhj,nhjc->nhc", a, X)
            X[:, :, i, :] = a
        Ai[r][r] = rf(X + eye)

    def dot(x, y):  # tf32 tensor-core dot with fp32 accumulation
        return rf(np.einsum("nhij,nhjk->nhik", rt(x), rt(y)))

    def blkA(r, s):
        return A[:, :, r * SUB:(r + 1) * SUB, s * SUB:(s + 1) * SUB]

    Ai[1][0] = -dot(dot(Ai[1][1], blkA(1, 0)), Ai[0][0])
    Ai[2][1] = -dot(dot(Ai[2][2], blkA(2, 1)), Ai[1][1])
    Ai[3][2] = -dot(dot(Ai[3][3], blkA(3, 2)), Ai[2][2])
    Ai[2][0] = -dot(Ai[2][2], rf(dot(blkA(2, 0), Ai[0][0]) + dot(blkA(2, 1), Ai[1][0])))
    Ai[3][1] = -dot(Ai[3][3], rf(dot(blkA(3, 1), Ai[1][1]) + dot(blkA(3, 2), Ai[2][1])))
    Ai[3][0] = -dot(Ai[3][3], rf(dot(blkA(3, 0), Ai[0][0]) + dot(blkA(3, 1), Ai[1][0])
                                 + dot(blkA(3, 2), Ai[2][0])))
    Ainv = np.zeros((NC, H, T, T), np.float64)
    for r in range(nb):
        for s in range(r + 1):
            Ainv[:, :, r * SUB:(r + 1) * SUB, s * SUB:(s + 1) * SUB] = Ai[r][s]
    Ainv = rb(Ainv * valid[:, None, :, None])  # stored in the key dtype (chunk_intra.py:408-417)

    # --- WY operands (wy_fast.py:92-142) ---
    wv = rb(vc if wc is None else vc * wc)
    u = rb(np.einsum("nhij,nhjv->nhiv", Ainv, wv))
    kbb = rb(kc if bc is None else kc * bc)  # bf16 x bf16 -> bf16 in the WY kernel
    w_wy = rb(np.einsum("nhij,nhjc->nhic", Ainv, rb(kbb * np.exp2(G))))
    last = np.maximum(lens - 1, 0)
    g_last = G[np.arange(NC), :, last, :]  # [NC,H,K]
    kg = rb(kc * np.where(vmask, np.exp2(g_last[:, :, None, :] - G), 0.0))
    return dict(G=G, A=A, Ainv=Ainv, u=u, w_wy=w_wy, kg=kg, g_last=g_last)


def scan(ops, chunks, h0, *, mode="exact"):
    """Sequential inter-chunk state scan (models/qwen/ops/_triton/state.py:76-115).

    v_new = u - w_wy . S ;  S <- diag(2^g_last) S + kg^T . v_new
    with the state cast to bf16 before the first product and v_new cast to bf16
    before the second in ``mode="bf16"``.
    """
    emu = mode == "bf16"
    rb = bf16 if emu else _id
    rf = r32 if emu else _id
    out = rf(_id(h0)).copy()
    for c, (n, _, _) in enumerate(chunks):
        S = out[n]
        vn = rf(ops["u"][c] - rf(np.einsum("htk,hkv->htv", ops["w_wy"][c], rb(S))))
        S = rf(rf(S * np.exp2(ops["g_last"][c])[:, :, None])
               + np.einsum("htk,htv->hkv", ops["kg"][c], rb(vn)))
        out[n] = S
    return out


def read(q, states, cu_seqlens, scale, *, mode="exact"):
    """o[t] = scale * q[t] . S[sample(t)] (read.py:51-71: state cast to q's dtype, fp32
    accumulation, scale, cast to the output dtype)."""
    emu = mode == "bf16"
    rb = bf16 if emu else _id
    rf = r32 if emu else _id
    q = _id(q)
    L, H, K = q.shape
    V = states.shape[-1]
    o = np.zeros((L, H, V), np.float64)
    cu = [int(x) for x in cu_seqlens]
    for n in range(len(cu) - 1):
        s = rb(_id(states[n]))
        acc = rf(np.einsum("thk,hkv->thv", q[cu[n]:cu[n + 1]], s))
        o[cu[n]:cu[n + 1]] = rb(rf(acc * np.float64(np.float32(scale))))
    return o


def chunked(q, k, v, g, h0, r0, cu_seqlens, scale, *, b=None, w=None, chunk_tokens=2048, mode="exact",
            exact_scores=False):
    """token_memory_packed: (read of the incoming snapshot r0, final state from h0)."""
    chunks = plan_chunks(cu_seqlens, chunk_tokens)
    ops = intra(k, g, v, chunks, b=b, w=w, mode=mode, exact_scores=exact_scores)
    final = scan(ops, chunks, h0, mode=mode)
    o = read(q, r0, cu_seqlens, scale, mode=mode)
    return o, final


# ---------------------------------------------------------------------------
# readout epilogue
# ---------------------------------------------------------------------------

def l2norm(x, eps=1e-6, *, mode="exact"):
    """x / sqrt(sum x^2 + eps) per last-dim row (l2norm.py:104-108); bf16 output in bf16 mode."""
    x = _id(x)
    y = x / np.sqrt((x * x).sum(-1, keepdims=True) + eps)
    return bf16(y) if mode == "bf16" else y


def qwen_gates(erase_gate, write_gate, decay_latent, decay_bias, decay_scale_log, *, mode="exact"):
    """QwenMemoryBlock._write_gates / _log_decay (models/qwen/layer.py:71-88): (erase_sqrt,
    write, log_decay) from the [L, H, D] pre-activations, decay_bias [H*D], decay_scale_log [H].

    erase_sqrt = exp(0.5 * logsigmoid(e)) with logsigmoid = min(0, x) - log1p(exp(-|x|));
    write = sigmoid(w); log_decay = -exp(decay_scale_log) * softplus(d + bias), softplus
    threshold 20. ``mode="bf16"`` evaluates in float32 and rounds erase_sqrt and write to bf16
    as the reference does (log_decay stays fp32); ``mode="exact"`` is float64 without rounding.
    """
    L, H, D = np.shape(erase_gate)
    f = np.float32 if mode == "bf16" else np.float64
    e = np.asarray(erase_gate, f)
    es = np.exp(f(0.5) * (np.minimum(f(0), e) - np.log1p(np.exp(-np.abs(e)))))
    w = f(1) / (f(1) + np.exp(-np.asarray(write_gate, f)))
    x = np.asarray(decay_latent, f) + np.asarray(decay_bias, f).reshape(1, H, D)
    sp = np.where(x > f(20), x, np.log1p(np.exp(np.minimum(x, f(20)))))
    g = -np.exp(np.asarray(decay_scale_log, f)).reshape(1, H, 1) * sp
    if mode == "bf16":
        return bf16(es.astype(f)), bf16(w.astype(f)), g.astype(f).astype(np.float64)
    return es, w, g


def qwen_prologue(q, k, erase_gate, write_gate, decay_latent, decay_bias, decay_scale_log, eps=1e-6, *,
                  mode="exact"):
    """The Qwen memory block's inputs to the update: (q_hat, k_scaled, write, log_decay).

    _symmetric_inputs (models/qwen/layer.py:90-97): q_hat = l2norm(q), k_scaled =
    erase_sqrt * l2norm(k), with the gates of ``qwen_gates``. ``mode="bf16"`` follows the
    eager rounding points in float32: l2norm in fp32 with a bf16 result (l2norm.py:104-108) and
    k_scaled = bf16(erase_sqrt * k_hat) (layer.py:94).
    """
    es, w, g = qwen_gates(erase_gate, write_gate, decay_latent, decay_bias, decay_scale_log, mode=mode)
    if mode == "bf16":
        f = np.float32

        def l2(x):
            x = np.asarray(x, f)
            rstd = f(1) / np.sqrt((x * x).sum(-1, keepdims=True, dtype=f) + f(eps))
            return bf16(x * rstd)

        return l2(q), bf16(es.astype(f) * l2(k).astype(f)), w, g
    return l2norm(q, eps), es * l2norm(k, eps), w, g


def latent_rms_norm(x, weight, eps):
    """_latent_norm (models/deepseek/ops/compiled_tensor_ops.py:12-20) on bf16 latents
    [T, G, R] in float32: bf16((x * rsqrt(mean(x^2) + eps[g])) * weight[g])."""
    f = np.float32
    x = np.asarray(x, f)
    w = np.asarray(weight, f).reshape(1, x.shape[1], x.shape[2])
    e = np.broadcast_to(np.asarray(eps, f).reshape(-1), (x.shape[1],)).reshape(1, -1, 1)
    ms = (x * x).sum(-1, keepdims=True, dtype=f) / f(x.shape[-1])
    return bf16((x * (f(1) / np.sqrt(ms + e))) * w)


def expand_grouped_qkv(q, k, v, q_norm, q_up, q_eps, k_up, v_up, k_norm, v_norm, k_eps, v_eps):
    """expand_grouped_qkv (models/deepseek/ops/compiled_tensor_ops.py:23-41): q [T, q_rank],
    k, v [T, G * rank], q_up [Vd, q_rank], k_up, v_up [G, width, rank]; bf16 outputs of float64
    products of the bf16 normalised latents."""
    T = q.shape[0]
    qn = latent_rms_norm(np.asarray(q).reshape(T, 1, -1), np.asarray(q_norm).reshape(1, -1), q_eps)[:, 0]
    qo = bf16(qn @ _id(q_up).T)

    def expand(lat, up, gain, eps):
        G, W, R = up.shape
        n = latent_rms_norm(np.asarray(lat).reshape(T, G, R), gain, eps)
        return bf16(np.einsum("tgr,gwr->tgw", n, _id(up))).reshape(T, G * W)

    return qo, expand(k, k_up, k_norm, k_eps), expand(v, v_up, v_norm, v_eps)


def memory_inject(memory, wo_a, groups, residual):
    """residual + einsum("tgd,grd->tgr") of the memory output and wo_a
    (models/deepseek/integration.py:56-61,66-72), exact (float64)."""
    T = memory.shape[0]
    m = _id(memory).reshape(T, groups, -1)
    w = _id(wo_a).reshape(groups, -1, m.shape[-1])
    return _id(residual) + np.einsum("tgd,grd->tgr", m, w).reshape(T, -1)


def gated_rms_norm(x, gate, weight, eps, softcap, *, mode="exact"):
    """MemTRMSNormGated.forward (models/qwen/layer.py:22-31).

    bf16 mode follows the eager rounding points: x fp32 -> normalise -> bf16 ->
    weight * (bf16 product) -> times the fp32 softcapped SiLU gate -> bf16.
    """
    emu = mode == "bf16"
    rb = bf16 if emu else _id
    x = _id(x)
    var = (x * x).mean(-1, keepdims=True)
    xn = rb(x / np.sqrt(var + eps))
    hs = rb(_id(weight) * xn)
    gt = _id(gate)
    sg = gt / (1.0 + np.exp(-gt))
    gv = softcap * np.tanh(sg / softcap)
    return rb(hs * gv)


def readout_fused(q, states, cu_seqlens, scale, gate, weight, eps, softcap, attn=None, *,
                  normalize_q=False, mode="exact"):
    """Decode-time memory readout: (l2norm q) -> read -> gated RMSNorm -> + attention row."""
    qh = l2norm(q, mode=mode) if normalize_q else _id(q)
    o = read(qh, states, cu_seqlens, scale, mode=mode)
    L, H, V = o.shape
    y = gated_rms_norm(o.reshape(-1, V), _id(gate).reshape(-1, V), weight, eps, softcap, mode=mode)
    y = y.reshape(L, H * V)
    if attn is None:
        return y
    out = _id(attn) + y
    return bf16(out) if mode == "bf16" else out
