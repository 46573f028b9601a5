"""GPU parity of the path as the reference serves it.

The Qwen memory block (models/qwen/layer.py:71-152) commits with channel-wise fp32 log-decay,
the sqrt-erase factor folded into the key and a write gate; the DeepSeek writer the same
without erase at d = 256. These tests run that shape end to end through the library (the
prologue kernel, then the update) at the BASELINE sizes, against the oracle. Tolerances
(relative Frobenius): bf16 inputs with fp32 state <= 1e-3 against the oracle's emulation of the
reference's rounding; prologue outputs within two bf16 units of the last place.
"""

import ctypes
import zlib
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import memt_b200 as M
from memt_b200 import _lib, ops
from oracle import gdn2 as O

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-3


def _np(t):
    return t.detach().float().cpu().numpy()


def _bf16_ulps(a, b):
    ia = np.asarray(a, np.float32).view(np.int32) >> 16
    ib = np.asarray(b, np.float32).view(np.int32) >> 16
    return np.abs(ia.astype(np.int64) - ib.astype(np.int64))


def _latents(dev, L, H, D, seed):
    """Projection outputs of a Qwen memory block: q/k/v as split views of one [L, 3HD] GEMM
    output and the erase/write pre-activations as views of the gate GEMM output (the layout
    QwenMemoryBlock.packed hands to its prologue), plus f_down of the decay rows and the decay
    parameters. Distributions follow the BASELINE configs: q, k, v ~ N(0, 1); erase and write
    pre-activations ~ N(0, 1) (sqrt(sigmoid) and sigmoid gates); decay latent ~ N(-2, 0.5) with
    zero bias and scale, i.e. log_decay = logsigmoid(N(2, 0.5)) per channel."""
    gen = torch.Generator(device=dev).manual_seed(seed)
    bf = torch.bfloat16
    qkv = torch.randn(L, 3 * H * D, device=dev, generator=gen).to(bf)
    gates = torch.randn(L, 2 * H * D + D, device=dev, generator=gen).to(bf)
    q, k, v = (qkv[:, i * H * D:(i + 1) * H * D].view(L, H, D) for i in range(3))
    erase_gate, write_gate = gates[:, :H * D], gates[:, H * D:2 * H * D]
    decay = (-2.0 + 0.5 * torch.randn(L, H * D, device=dev, generator=gen)).to(bf)
    bias = torch.zeros(H * D, device=dev, dtype=bf)
    scale_log = torch.zeros(H, device=dev, dtype=bf)
    return SimpleNamespace(q=q, k=k, v=v, erase_gate=erase_gate, write_gate=write_gate, decay=decay, bias=bias,
                           scale_log=scale_log)


# ---------------------------------------------------------------------------
# the prologue kernel
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("L,H,D", [(1, 1, 64), (37, 3, 64), (300, 2, 128), (129, 4, 256), (4096, 16, 128)])
def test_qwen_prologue_matches_oracle(cuda, L, H, D):
    """q_hat, k_scaled, write (bf16) on at most 1 % of the elements off the oracle's float32
    restatement, by at most two units of the last place (libm exp/log1p and the summation order
    of the norms may differ by an ulp; k_scaled is the rounded product of two such values), and
    log-decay (fp32) within 1e-6 relative."""
    x = _latents(cuda, L, H, D, zlib.crc32(f"{L},{H},{D}".encode()))
    gen = torch.Generator(device=cuda).manual_seed(L)
    x.bias = (0.5 * torch.randn(H * D, device=cuda, generator=gen)).to(torch.bfloat16)
    x.scale_log = (0.3 * torch.randn(H, device=cuda, generator=gen)).to(torch.bfloat16)
    q_hat, k_s, w, g = M.qwen_prologue(x.q, x.k, x.erase_gate, x.write_gate, x.decay, x.bias, x.scale_log)
    torch.cuda.synchronize()
    assert q_hat.shape == (1, L, H, D) and g.dtype == torch.float32
    ref = O.qwen_prologue(_np(x.q), _np(x.k), _np(x.erase_gate).reshape(L, H, D),
                          _np(x.write_gate).reshape(L, H, D), _np(x.decay).reshape(L, H, D), _np(x.bias),
                          _np(x.scale_log), 1e-6, mode="bf16")
    for got, want in zip((q_hat, k_s, w), ref[:3]):
        d = _bf16_ulps(_np(got[0]), want)
        assert d.max() <= 2 and np.mean(d > 0) <= 0.01, (d.max(), np.mean(d > 0))
    assert O.rel_fro(_np(g[0]), ref[3]) <= 1e-6


def test_qwen_prologue_matches_the_reference_eager_ops(cuda):
    """The gate math against the reference's own eager PyTorch expressions
    (models/qwen/layer.py:71-88) evaluated by torch on the same GPU: erase and write within one
    bf16 ulp, log-decay within fp32 rounding; l2norm against the FLA formula in fp32."""
    L, H, D = 2048, 4, 128
    x = _latents(cuda, L, H, D, 11)
    gen = torch.Generator(device=cuda).manual_seed(5)
    x.bias = (0.5 * torch.randn(H * D, device=cuda, generator=gen)).to(torch.bfloat16)
    x.scale_log = (0.3 * torch.randn(H, device=cuda, generator=gen)).to(torch.bfloat16)
    q_hat, k_s, w, g = M.qwen_prologue(x.q, x.k, x.erase_gate, x.write_gate, x.decay, x.bias, x.scale_log)
    F = torch.nn.functional
    gate = F.softplus(x.decay.float() + x.bias)
    log_decay = -x.scale_log.float().exp().view(H, 1) * gate.view(L, H, -1)
    erase = torch.exp(0.5 * F.logsigmoid(x.erase_gate.float())).to(torch.bfloat16).view(L, H, D)
    write = x.write_gate.sigmoid().view(L, H, D)

    def l2(t):
        t = t.float()
        return (t * (1 / torch.sqrt((t * t).sum(-1, keepdim=True) + 1e-6))).to(torch.bfloat16)

    k_ref = (erase.float() * l2(x.k).float()).to(torch.bfloat16)
    torch.cuda.synchronize()
    assert _bf16_ulps(_np(w[0]), _np(write)).max() <= 1
    assert _bf16_ulps(_np(q_hat[0]), _np(l2(x.q))).max() <= 1
    assert _bf16_ulps(_np(k_s[0]), _np(k_ref)).max() <= 2
    assert torch.allclose(g[0], log_decay, rtol=2e-7, atol=0)


# ---------------------------------------------------------------------------
# BASELINE config 1 as the reference serves it: channel-wise decay, erase folded into the key
# ---------------------------------------------------------------------------

def _oracle_state(k, v, g, w, h0, t0, t1, n, h, ct=2048):
    x = dict(cu=np.array([0, t1 - t0]), k=_np(k[t0:t1, h:h + 1]), v=_np(v[t0:t1, h:h + 1]),
             g=_np(g[t0:t1, h:h + 1]), w=_np(w[t0:t1, h:h + 1]), h0=_np(h0[n:n + 1, h:h + 1]))
    chunks = O.plan_chunks(x["cu"], ct)
    ops_ = O.intra(x["k"], x["g"], x["v"], chunks, w=x["w"], mode="bf16")
    return O.scan(ops_, chunks, x["h0"], mode="bf16")


def test_config1_qwen_commit_channel_decay(cuda):
    """8 sessions x 8192 tokens, H = 16, d = 128: prologue -> token_memory_packed (erase None,
    per-channel fp32 log-decay, write gate) as the Qwen block commits. Four (session, head)
    slices against the oracle; one session run alone reproduces its pack result bit for bit;
    passing the reference's all-ones erase tensor gives the same states within tolerance."""
    lengths, H, D = [8192] * 8, 16, 128
    L = sum(lengths)
    x = _latents(cuda, L, H, D, 21)
    q_hat, k_s, w, g = M.qwen_prologue(x.q, x.k, x.erase_gate, x.write_gate, x.decay, x.bias, x.scale_log)
    gen = torch.Generator(device=cuda).manual_seed(22)
    h0 = 0.02 * torch.randn(8, H, D, D, device=cuda, generator=gen)
    args = dict(lengths=lengths, scale=D ** -0.5, chunk_tokens=2048)
    read, final = M.token_memory_packed(q_hat, k_s, x.v[None], g, w, h0, h0, erase=None, **args)
    n = 6
    sl = slice(n * 8192, (n + 1) * 8192)
    _, one = M.token_memory_packed(q_hat[:, sl], k_s[:, sl], x.v[None, sl], g[:, sl], w[:, sl],
                                   h0[n:n + 1].contiguous(), h0[n:n + 1].contiguous(), erase=None,
                                   lengths=[8192], scale=D ** -0.5, chunk_tokens=2048)
    ones = torch.ones_like(k_s)
    _, final_ones = M.token_memory_packed(q_hat, k_s, x.v[None], g, w, h0, h0, erase=ones, **args)
    torch.cuda.synchronize()
    assert torch.isfinite(final).all()
    assert torch.equal(final[n], one[0])
    assert O.rel_fro(_np(final_ones), _np(final)) <= 1e-4
    k2, v2, g2, w2 = k_s[0], x.v, g[0], w[0]
    for s, h in ((0, 0), (3, 7), (6, 12), (7, 15)):
        ref = _oracle_state(k2, v2, g2, w2, h0, s * 8192, (s + 1) * 8192, s, h)
        err = O.rel_fro(_np(final[s, h:h + 1])[None], ref)
        assert err <= TOL_BF16, (s, h, err)
    # the commit read of the incoming snapshot for one slice
    s, h = 2, 5
    o_ref = O.read(_np(q_hat[0, s * 8192:(s + 1) * 8192, h:h + 1]), _np(h0[s:s + 1, h:h + 1]),
                   np.array([0, 8192]), D ** -0.5, mode="bf16")
    assert O.rel_fro(_np(read[0, s * 8192:(s + 1) * 8192, h:h + 1]), o_ref) <= TOL_BF16


@pytest.mark.parametrize("D", [64, 128])
def test_channel_decay_with_many_units_per_cta(cuda, D):
    """Channel-wise decay without erase, ragged sessions and enough (chunk, head) units that
    every CTA of the persistent intra grid walks several of them (each unit's decay table is
    loaded while the previous unit finishes). Three (session, head) slices against the oracle,
    and one session run alone reproduces its pack result bit for bit."""
    lengths, H = [2000, 1500, 3000, 64, 1, 900], 16
    L = sum(lengths)
    x = _latents(cuda, L, H, D, 31 + D)
    q_hat, k_s, w, g = M.qwen_prologue(x.q, x.k, x.erase_gate, x.write_gate, x.decay, x.bias, x.scale_log)
    gen = torch.Generator(device=cuda).manual_seed(32)
    N = len(lengths)
    h0 = 0.02 * torch.randn(N, H, D, D, device=cuda, generator=gen)
    args = dict(scale=D ** -0.5, chunk_tokens=2048)
    _, final = M.token_memory_packed(q_hat, k_s, x.v[None], g, w, h0, h0, erase=None, lengths=lengths, **args)
    cu = np.concatenate([[0], np.cumsum(lengths)])
    n = 2
    sl = slice(int(cu[n]), int(cu[n + 1]))
    _, one = M.token_memory_packed(q_hat[:, sl], k_s[:, sl], x.v[None, sl], g[:, sl], w[:, sl],
                                   h0[n:n + 1].contiguous(), h0[n:n + 1].contiguous(), erase=None,
                                   lengths=[lengths[n]], **args)
    torch.cuda.synchronize()
    assert torch.isfinite(final).all()
    assert torch.equal(final[n], one[0])
    for s_, h in ((0, 3), (2, 15), (5, 0)):
        ref = _oracle_state(k_s[0], x.v, g[0], w[0], h0, int(cu[s_]), int(cu[s_ + 1]), s_, h)
        err = O.rel_fro(_np(final[s_, h:h + 1])[None], ref)
        assert err <= TOL_BF16, (s_, h, err)


def test_config4_flash_full_length(cuda):
    """BASELINE config 4 at its real length: 4 sessions x 16384 tokens, d = 256, the 16 heads
    one of eight tensor-parallel ranks owns (128 heads / TP8), channel-wise decay, write gate,
    no erase (the DeepSeek writer). Three (session, head) slices against the oracle."""
    lengths, H, D = [16384] * 4, 16, 256
    L = sum(lengths)
    gen = torch.Generator(device=cuda).manual_seed(44)
    bf = torch.bfloat16

    def nrm(t):
        return (t / torch.sqrt((t.float() ** 2).sum(-1, keepdim=True) + 1e-6)).to(bf)

    q = nrm(torch.randn(L, H, D, device=cuda, generator=gen))
    k = nrm(torch.randn(L, H, D, device=cuda, generator=gen))
    v = torch.randn(L, H, D, device=cuda, generator=gen).to(bf)
    g = torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L, H, D, device=cuda, generator=gen))
    w = torch.sigmoid(torch.randn(L, H, D, device=cuda, generator=gen)).to(bf)
    h0 = 0.02 * torch.randn(4, H, D, D, device=cuda, generator=gen)
    read, final = M.token_memory_packed(q[None], k[None], v[None], g[None], w[None], h0, h0, lengths=lengths,
                                        scale=D ** -0.5, chunk_tokens=2048)
    torch.cuda.synchronize()
    assert torch.isfinite(final).all()
    for s, h in ((0, 3), (2, 9), (3, 15)):
        ref = _oracle_state(k, v, g, w, h0, s * 16384, (s + 1) * 16384, s, h)
        err = O.rel_fro(_np(final[s, h:h + 1])[None], ref)
        assert err <= TOL_BF16, (s, h, err)
    # the commit read of the incoming snapshot (d = 256 tensor-core tile read) for two slices
    for s, h in ((1, 0), (3, 14)):
        t0, t1 = s * 16384, (s + 1) * 16384
        o_ref = O.read(_np(q[t0:t1, h:h + 1]), _np(h0[s:s + 1, h:h + 1]), np.array([0, 16384]), D ** -0.5,
                       mode="bf16")
        assert O.rel_fro(_np(read[0, t0:t1, h:h + 1]), o_ref) <= TOL_BF16


# ---------------------------------------------------------------------------
# state pools against the oracle
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("gate", ["head", "channel"])
def test_state_pool_update_against_oracle(cuda, gate):
    """The update reading and writing a state pool by slot index matches the oracle run on the
    gathered states (not only the gathered CUDA call)."""
    rng = np.random.default_rng(31 if gate == "head" else 32)
    lengths, H, D, S = [300, 64, 129], 3, 128, 7
    L, N = sum(lengths), len(lengths)
    cu = np.concatenate([[0], np.cumsum(lengths)])
    k = O.bf16(rng.standard_normal((L, H, D)) / np.sqrt(D))
    v = O.bf16(rng.standard_normal((L, H, D)))
    gshape = (L, H, D) if gate == "channel" else (L, H)
    g = (-np.logaddexp(0.0, -rng.normal(2.0, 0.5, gshape))).astype(np.float32)
    w = O.bf16(1 / (1 + np.exp(-rng.standard_normal((L, H, D)))))
    pool = (0.05 * rng.standard_normal((S, H, D, D))).astype(np.float32)
    slots = np.array([5, 0, 3], np.int32)
    bf = torch.bfloat16

    def t(a, dtype=torch.float32):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda).to(dtype)

    pool_t = t(pool)
    slot_t = torch.from_numpy(slots).to(cuda)
    ops.gdn2_update(t(k, bf), t(v, bf), t(g), pool_t, torch.from_numpy(cu.astype(np.int32)).to(cuda),
                    num_samples=N, total_tokens=L, write=t(w, bf), final_state=pool_t, initial_slots=slot_t,
                    final_slots=slot_t)
    torch.cuda.synchronize()
    g3 = g if g.ndim == 3 else np.broadcast_to(g[:, :, None], (L, H, D))
    chunks = O.plan_chunks(cu, 2048)
    ref = O.scan(O.intra(k, g3, v, chunks, w=w, mode="bf16"), chunks, pool[slots], mode="bf16")
    got = pool_t.cpu().numpy()
    assert O.rel_fro(got[slots], ref) <= TOL_BF16
    others = [i for i in range(S) if i not in slots]
    assert np.array_equal(got[others], pool[others])


# ---------------------------------------------------------------------------
# reads: grid bound below the longest block, the reference's own ChunkPlan
# ---------------------------------------------------------------------------

def _read_call(q, states, cu, n_blocks, bound, D, cuda):
    _, args, out, keep = ops._read_args(q, states, cu, n_blocks, bound, D ** -0.5, torch.bfloat16)
    return _lib.load().memt_gdn2_read(ctypes.byref(args), ops._stream(cuda)), out, keep


def _readout_call(q, states, cu, n_blocks, bound, gate, nw, cuda):
    L, H, D = q.shape
    out = torch.zeros(L, H * D, device=cuda, dtype=torch.bfloat16)
    args = _lib.ReadoutArgs(num_blocks=n_blocks, num_heads=H, head_dim=D, total_tokens=L, max_block_tokens=bound,
                            cu_seqlens=cu.data_ptr(), q=q.data_ptr(), normalize_q=1, q_eps=1e-6,
                            states=states.data_ptr(), scale=D ** -0.5, gate=gate.data_ptr(), norm_weight=nw.data_ptr(),
                            norm_eps=1e-6, softcap=10.0, residual=None, out=out.data_ptr(), row_stride=H * D,
                            head_offset=0)
    return _lib.load().memt_memory_readout(ctypes.byref(args), ops._stream(cuda)), out


@pytest.mark.parametrize("D", [64, 128, 256])
def test_read_with_a_short_block_bound_reads_every_token(cuda, D):
    """max_block_tokens sizes the grid and picks the kernel. A bound the blocks cannot satisfy
    (bound * blocks < tokens) is rejected before launch; any other bound below the longest block
    still reads every token, on the tile kernels (bounds > 16) and on the multi-token GEMV
    (bounds 2..16), for the plain read and the fused readout."""
    rng = np.random.default_rng(D)
    bf = torch.bfloat16
    for lengths, bounds in (([1500, 3, 700], (800, 1000)), ([40] + [1] * 9, (5, 16))):
        L, N, H = sum(lengths), len(lengths), 2
        q = torch.from_numpy(rng.standard_normal((L, H, D)).astype(np.float32)).to(cuda).to(bf)
        states = torch.from_numpy((0.05 * rng.standard_normal((N, H, D, D))).astype(np.float32)).to(cuda)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=cuda)
        gate = torch.from_numpy(rng.standard_normal((L, H, D)).astype(np.float32)).to(cuda).to(bf)
        nw = torch.ones(D, device=cuda, dtype=bf)
        st, _, _ = _read_call(q, states, cu, N, 1, D, cuda)
        assert st == _lib.MEMT_ERR_INVALID_ARGUMENT
        st, _ = _readout_call(q, states, cu, N, 1, gate, nw, cuda)
        assert st == _lib.MEMT_ERR_INVALID_ARGUMENT
        ref = O.read(_np(q), states.cpu().numpy(), cu.cpu().numpy(), D ** -0.5, mode="bf16")
        st, full_fused = _readout_call(q, states, cu, N, max(lengths), gate, nw, cuda)
        assert st == 0
        for bound in bounds:
            st, out, keep = _read_call(q, states, cu, N, bound, D, cuda)
            assert st == 0
            st, fused = _readout_call(q, states, cu, N, bound, gate, nw, cuda)
            assert st == 0
            torch.cuda.synchronize()
            assert O.rel_fro(_np(out), ref) <= TOL_BF16, (lengths, bound)
            assert bool((fused.float().abs().sum(-1) > 0).all()), (lengths, bound)  # every token row written
            assert O.rel_fro(_np(fused), _np(full_fused)) <= 4e-3, (lengths, bound)


def test_decode_read_records_a_block_longer_than_its_bound(cuda):
    """With an empty block beside it, a block of two tokens passes the host's bound check for
    bound 1: the one-token decode kernel reads its first token and sets bit 0 of the read
    status, which memt_read_status reports once and clears."""
    lib = _lib.load()
    bf = torch.bfloat16
    H, D = 2, 128
    rng = np.random.default_rng(4)
    q = torch.from_numpy(rng.standard_normal((2, H, D)).astype(np.float32)).to(cuda).to(bf)
    states = torch.from_numpy((0.05 * rng.standard_normal((2, H, D, D))).astype(np.float32)).to(cuda)
    stream = ops._stream(cuda)
    status = ctypes.c_int32(-1)
    assert lib.memt_read_status(stream, ctypes.byref(status)) == 0  # clear what earlier tests left
    good = torch.tensor([0, 1, 2], dtype=torch.int32, device=cuda)
    st, ref, _ = _read_call(q, states, good, 2, 1, D, cuda)
    assert st == 0
    assert lib.memt_read_status(stream, ctypes.byref(status)) == 0 and status.value == 0
    cu = torch.tensor([0, 0, 2], dtype=torch.int32, device=cuda)  # block 0 empty, block 1 two tokens
    st, out, _ = _read_call(q, states, cu, 2, 1, D, cuda)
    assert st == 0
    assert lib.memt_read_status(stream, ctypes.byref(status)) == 0 and status.value == 1
    assert lib.memt_read_status(stream, ctypes.byref(status)) == 0 and status.value == 0
    want = O.read(_np(q[:1]), states[1:].cpu().numpy(), np.array([0, 1]), D ** -0.5, mode="bf16")
    assert O.rel_fro(_np(out[:1]), want) <= TOL_BF16


def test_read_fwd_takes_the_reference_chunk_plan(cuda):
    """memt_gdn2_read_fwd with a plan object that carries only the reference ChunkPlan's fields
    (no read_slice) reads the same snapshots as with this library's plan."""
    rng = np.random.default_rng(8)
    lengths, H, D = [70, 1, 300, 64], 2, 128
    L = sum(lengths)
    q = torch.from_numpy(rng.standard_normal((1, L, H, D)).astype(np.float32)).to(cuda).to(torch.bfloat16)
    snaps = torch.from_numpy((0.05 * rng.standard_normal((4, H, D, D))).astype(np.float32)).to(cuda)
    plan = M.packed_plan(lengths, cuda, chunk_tokens=2048)
    ref_like = SimpleNamespace(**{f: getattr(plan, f) for f in plan.__slots__ if f not in ("read_slice",
                                                                                            "max_block_tokens")})
    a = M.memt_gdn2_read_fwd(q, snaps, plan, D ** -0.5, torch.bfloat16)
    b = M.memt_gdn2_read_fwd(q, snaps, ref_like, D ** -0.5, torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("gate", ["head", "channel"])
def test_update_reads_split_projection_views_in_place(cuda, gate):
    """k, v and the write gate as split views of one wider projection output (token rows of
    3 H D elements) give the same states, bit for bit, as their contiguous copies: the kernels
    read the rows in place (TMA maps and cp.async with the views' row strides)."""
    L, H, D = 700, 2, 128
    x = _latents(cuda, L, H, D, 77)
    gen = torch.Generator(device=cuda).manual_seed(78)
    w_all = torch.sigmoid(torch.randn(L, 2 * H * D, device=cuda, generator=gen)).to(torch.bfloat16)
    w = w_all[:, H * D:].view(L, H, D)
    gshape = (L, H, D) if gate == "channel" else (L, H)
    g = torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(*gshape, device=cuda, generator=gen))
    h0 = 0.02 * torch.randn(2, H, D, D, device=cuda, generator=gen)
    cu = torch.tensor([0, 300, L], dtype=torch.int32, device=cuda)
    k = (x.k.float() / x.k.float().norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    kv = torch.cat([k.reshape(L, -1), x.v.reshape(L, -1)], dim=1)  # one [L, 2HD] buffer
    k_view, v_view = kv[:, :H * D].view(L, H, D), kv[:, H * D:].view(L, H, D)
    assert not k_view.is_contiguous() and not v_view.is_contiguous()
    a = ops.gdn2_update(k_view, v_view, g, h0, cu, num_samples=2, total_tokens=L, write=w)
    b = ops.gdn2_update(k_view.contiguous(), v_view.contiguous(), g, h0, cu, num_samples=2, total_tokens=L,
                        write=w.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(a, b)
