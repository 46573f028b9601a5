"""GPU parity of the sm_100a kernels against the CPU oracle and the reference's goldens.

Tolerances (relative Frobenius):
  * bf16 inputs / fp32 state: <= 1e-3 against the oracle's emulation of the reference's
    GPU rounding points (BASELINE tolerance);
  * fp32 mode: <= 1e-5 against float64 exact math and the reference's fp32 outputs.
"""

import ctypes
import zlib

import numpy as np
import pytest
import torch

import memt_b200 as M
from memt_b200 import _lib, ops
from oracle import gdn2 as O

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-3
TOL_F32 = 1e-5
# per-head decay: the kernel evaluates the key-key scores from exact products; against the
# oracle's model of that evaluation the differences are accumulation orders and the bf16
# rounding flips they cause
TOL_KERNEL = 5e-4


def _t(x, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(x, np.float32))).to(dev).to(dtype)


def make_inputs(seed, lengths, H, D, *, gate="channel", beta="head", erase=False, write=True, state=True,
                decay_mean=2.0):
    """BASELINE distributions: q,k ~N(0,1) then L2-normalised, v ~N(0,1), g = logsigmoid(N(2,.5)),
    beta = sigmoid(N(0,1)), write = sigmoid(N(0,1)), states ~N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    L, N = int(sum(lengths)), len(lengths)

    def nrm(x):
        return x / np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)

    x = dict(lengths=list(lengths), cu=np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32))
    x["q"] = nrm(rng.standard_normal((L, H, D))).astype(np.float32)
    x["k"] = nrm(rng.standard_normal((L, H, D))).astype(np.float32)
    x["v"] = rng.standard_normal((L, H, D)).astype(np.float32)
    gshape = (L, H, D) if gate == "channel" else (L, H)
    x["g"] = (-np.logaddexp(0.0, -rng.normal(decay_mean, 0.5, gshape))).astype(np.float32)
    bshape = {"head": (L, H), "channel": (L, H, D), None: None}[beta]
    x["beta"] = None if bshape is None else (1 / (1 + np.exp(-rng.standard_normal(bshape)))).astype(np.float32)
    x["erase"] = (1 / (1 + np.exp(-rng.standard_normal((L, H, D))))).astype(np.float32) if erase else None
    x["w"] = (1 / (1 + np.exp(-rng.standard_normal((L, H, D))))).astype(np.float32) if write else None
    sd = 0.02 if state else 0.0
    x["h0"] = (sd * rng.standard_normal((N, H, D, D))).astype(np.float32)
    x["r0"] = (sd * rng.standard_normal((N, H, D, D))).astype(np.float32)
    return x


def to_bf16(x):
    out = dict(x)
    for key in ("q", "k", "v", "beta", "erase", "w"):
        if out[key] is not None:
            out[key] = O.bf16(out[key]).astype(np.float32)
    return out


def oracle_key(x, mode):
    """k' = sqrt(beta) * k, with the reference's bf16 rounding of sqrt(beta) and of the product."""
    k = x["k"].astype(np.float64)
    if x["beta"] is None:
        return k
    b = x["beta"].astype(np.float64)
    if b.ndim == 2:
        b = b[:, :, None]
    s = np.sqrt(b)
    return O.bf16(O.bf16(s) * k) if mode == "bf16" else s * k


def oracle_update(x, chunk_tokens, mode, exact_scores=False):
    kk = oracle_key(x, mode)
    g = x["g"] if x["g"].ndim == 3 else np.broadcast_to(x["g"][:, :, None], x["k"].shape)
    if mode == "bf16":
        ops_ = O.intra(kk, g, x["v"], O.plan_chunks(x["cu"], chunk_tokens), b=x["erase"], w=x["w"], mode="bf16",
                       exact_scores=exact_scores)
        return O.scan(ops_, O.plan_chunks(x["cu"], chunk_tokens), x["h0"], mode="bf16")
    return O.recurrence(kk, x["v"], g, x["h0"], x["cu"], b=x["erase"], w=x["w"])


def gpu_update(x, dev, dtype, chunk_tokens, final_state=None, h0=None):
    cu = torch.from_numpy(x["cu"]).to(dev)
    h0 = _t(x["h0"], dev) if h0 is None else h0
    return ops.gdn2_update(
        _t(x["k"], dev, dtype), _t(x["v"], dev, dtype), _t(x["g"], dev), h0, cu,
        num_samples=len(x["lengths"]), total_tokens=int(x["cu"][-1]),
        beta=None if x["beta"] is None else _t(x["beta"], dev, dtype),
        erase=None if x["erase"] is None else _t(x["erase"], dev, dtype),
        write=None if x["w"] is None else _t(x["w"], dev, dtype), chunk_tokens=chunk_tokens,
        final_state=final_state)


# ---------------------------------------------------------------------------
# reference goldens
# ---------------------------------------------------------------------------

PACKED = ["cfg0_qwen", "varlen_qwen", "d128_qwen", "varlen_flash"]


@pytest.mark.parametrize("name", PACKED)
def test_golden_fp32(golden, cuda, name):
    """fp32 mode against the reference's own fp32 outputs."""
    z = golden(name)
    erase = _t(z["b"], cuda)[None] if str(z["flavour"]) == "qwen" else None
    read, final = M.token_memory_packed(
        _t(z["q"], cuda)[None], _t(z["k"], cuda)[None], _t(z["v"], cuda)[None], _t(z["g"], cuda)[None],
        _t(z["w"], cuda)[None], _t(z["r0"], cuda), _t(z["h0"], cuda), erase=erase,
        lengths=[int(n) for n in z["lengths"]], scale=float(z["scale"]), chunk_tokens=int(z["chunk_tokens"]))
    torch.cuda.synchronize()
    assert read.shape == (1, *z["read"].shape) and read.dtype == torch.float32
    assert O.rel_fro(final.cpu().numpy(), z["final_state"]) <= TOL_F32
    if np.abs(z["read"]).sum() > 0:
        assert O.rel_fro(read[0].cpu().numpy(), z["read"]) <= TOL_F32


@pytest.mark.parametrize("name", PACKED)
def test_golden_bf16(golden, cuda, name):
    """bf16 inputs through token_memory_packed against the oracle's GPU-rounding emulation."""
    z = golden(name)
    qwen = str(z["flavour"]) == "qwen"
    rb = {key: O.bf16(z[key]).astype(np.float32) for key in ("q", "k", "v", "w", "b")}
    bf = torch.bfloat16
    read, final = M.token_memory_packed(
        _t(rb["q"], cuda, bf)[None], _t(rb["k"], cuda, bf)[None], _t(rb["v"], cuda, bf)[None],
        _t(z["g"], cuda)[None], _t(rb["w"], cuda, bf)[None], _t(z["r0"], cuda), _t(z["h0"], cuda),
        erase=_t(rb["b"], cuda, bf)[None] if qwen else None, lengths=[int(n) for n in z["lengths"]],
        scale=float(z["scale"]), chunk_tokens=int(z["chunk_tokens"]))
    torch.cuda.synchronize()
    assert read.dtype == torch.bfloat16
    o_ref, s_ref = O.chunked(rb["q"], rb["k"], rb["v"], z["g"], z["h0"], z["r0"], z["cu_seqlens"],
                             float(z["scale"]), b=rb["b"] if qwen else None, w=rb["w"],
                             chunk_tokens=int(z["chunk_tokens"]), mode="bf16")
    err_s = O.rel_fro(final.cpu().numpy(), s_ref)
    assert err_s <= TOL_BF16, err_s
    if np.abs(o_ref).sum() > 0:
        assert O.rel_fro(read[0].float().cpu().numpy(), o_ref) <= TOL_BF16


# ---------------------------------------------------------------------------
# update parity sweep
# ---------------------------------------------------------------------------

CASES = [
    # lengths, H, D, gate, beta, erase, write, chunk_tokens
    ([512], 4, 64, "head", "head", False, True, 2048),           # BASELINE config 0 shape
    ([1], 2, 128, "channel", None, False, True, 2048),
    ([63, 64, 65], 2, 128, "channel", "head", True, True, 2048),
    ([130, 1, 200], 3, 128, "head", "channel", False, False, 128),
    ([300, 7], 2, 128, "channel", "head", False, True, 100),     # events not a multiple of 64
    ([150, 64], 2, 256, "channel", "head", True, True, 2048),
    ([257], 1, 256, "head", None, False, True, 2048),
    ([33, 97, 64, 1], 4, 64, "channel", "channel", True, False, 64),
    # per-head decay without erase (the TMA-fed intra path): ragged chunks whose tile rows past
    # the sample hold the next sample's tokens, no beta, per-channel beta, d = 64
    ([100, 37, 64, 200], 2, 128, "head", "head", False, True, 2048),
    ([70, 5], 2, 128, "head", None, False, True, 2048),
    ([90, 40], 2, 64, "head", "channel", False, True, 64),
    # d = 256 (the tcgen05 scan over two 128-value blocks): ragged, a single-token sample, odd H,
    # per-head decay through the TMA-fed intra path; per-channel decay with 64-token events
    ([1, 130, 64, 200], 3, 256, "head", "head", False, True, 2048),
    ([65, 1, 129], 2, 256, "channel", None, False, False, 64),
]


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_update_bf16_parity(cuda, case):
    lengths, H, D, gate, beta, erase, write, ct = case
    x = to_bf16(make_inputs(zlib.crc32(str(case).encode()), lengths, H, D, gate=gate, beta=beta, erase=erase,
                            write=write))
    out = gpu_update(x, cuda, torch.bfloat16, ct)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    err = O.rel_fro(got, oracle_update(x, ct, "bf16"))  # the reference's rounding
    assert err <= TOL_BF16, err
    if gate == "head":
        err_k = O.rel_fro(got, oracle_update(x, ct, "bf16", exact_scores=True))
        assert err_k <= TOL_KERNEL, (err_k, err)


@pytest.mark.parametrize("case", CASES[:5], ids=[f"c{i}" for i in range(5)])
def test_update_fp32_exact(cuda, case):
    lengths, H, D, gate, beta, erase, write, ct = case
    x = make_inputs(1 + zlib.crc32(str(case).encode()), lengths, H, D, gate=gate, beta=beta, erase=erase, write=write)
    out = gpu_update(x, cuda, torch.float32, ct)
    torch.cuda.synchronize()
    ref = oracle_update(x, ct, "exact")
    assert O.rel_fro(out.cpu().numpy(), ref) <= TOL_F32


def test_update_read_matches_separate_calls(cuda):
    """memt_gdn2_update_read (the read overlapping the update's state scan on a second stream)
    gives exactly the results of memt_gdn2_update followed by memt_gdn2_read, also when the
    read states are the update's own output (then the two run in order)."""
    x = to_bf16(make_inputs(5, [300, 64, 129], 4, 128, gate="head", beta="head", erase=False, write=True))
    bf = torch.bfloat16
    q, k, v = (_t(x[n], cuda, bf) for n in ("q", "k", "v"))
    g, beta, w = _t(x["g"], cuda), _t(x["beta"], cuda, bf), _t(x["w"], cuda, bf)
    h0 = _t(x["h0"], cuda)
    rs = h0 + 0.01
    cu = torch.from_numpy(x["cu"]).to(cuda)
    N, L = len(x["lengths"]), int(x["cu"][-1])
    o_ref_fin = ops.gdn2_update(k, v, g, h0, cu, num_samples=N, total_tokens=L, beta=beta, write=w)
    o_ref = ops._read(q, rs, cu, N, 300, 128 ** -0.5, bf)
    o, fin = ops.gdn2_chunked(q, k, v, g, beta, h0, cu, w=w, read_states=rs, max_seqlen=300)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(fin, o_ref_fin)
    # read of the states the update writes (an in-place update): in order, the read first
    lib = _lib.load()
    final = rs.clone()
    uargs_lib, uargs, ws, out, keep_u = ops._update_args(k, v, g, h0, cu, N, L, beta, None, w, 2048, final)
    _, rargs, o2, keep_r = ops._read_args(q, final, cu, N, 300, 128 ** -0.5, bf)
    st = lib.memt_gdn2_update_read(ctypes.byref(uargs), ops._ptr(ws), ws.numel(), ctypes.byref(rargs),
                                   ops._stream(cuda))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(final, o_ref_fin)
    assert torch.equal(o2, o_ref)  # the incoming snapshot rs, not the updated state


def test_reads_from_a_state_pool(cuda):
    """Slot indices into a state pool (instead of gathering the step's states into a new
    tensor) give bit-identical readouts and commit reads; a slot outside the pool leaves its
    block's output untouched."""
    gen = torch.Generator(device=cuda).manual_seed(3)
    bf = torch.bfloat16
    H, D, S = 4, 128, 11
    pool = 0.05 * torch.randn(S, H, D, D, device=cuda, generator=gen)
    slots = torch.tensor([7, 2, 9], dtype=torch.int32, device=cuda)
    gathered = pool[slots.long()].contiguous()
    # decode readout: one token per session
    n = 3
    q = torch.randn(n, H, D, device=cuda, generator=gen).to(bf)
    gate = torch.randn(n, H, D, device=cuda, generator=gen).to(bf)
    w = (1 + 0.1 * torch.randn(D, device=cuda, generator=gen)).to(bf)
    res = torch.randn(n, H * D, device=cuda, generator=gen).to(bf)
    ref = M.memory_readout(q, gathered, [1] * n, D ** -0.5, gate, w, softcap=10.0, residual=res)
    got = M.memory_readout(q, pool, [1] * n, D ** -0.5, gate, w, softcap=10.0, residual=res, state_slots=slots)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    # commit read inside token_memory_packed: ragged samples long enough for the tile kernels
    x = to_bf16(make_inputs(9, [700, 64, 1100], H, D, gate="channel", beta=None, erase=False, write=True))
    args = dict(lengths=x["lengths"], scale=D ** -0.5, chunk_tokens=2048)
    kk = _t(x["k"], cuda, bf)
    tens = [_t(x[name], cuda, bf)[None] for name in ("q",)] + [kk[None], _t(x["v"], cuda, bf)[None],
                                                              _t(x["g"], cuda)[None], _t(x["w"], cuda, bf)[None]]
    h0 = _t(x["h0"], cuda)
    r_ref, f_ref = M.token_memory_packed(*tens, gathered, h0, **args)
    r_got, f_got = M.token_memory_packed(*tens, pool, h0, read_slots=slots, **args)
    torch.cuda.synchronize()
    assert torch.equal(r_got, r_ref) and torch.equal(f_got, f_ref)
    # a slot outside the pool: that session's output is not written
    bad = torch.tensor([7, S + 3, 9], dtype=torch.int32, device=cuda)
    out = torch.full((n, H * D), 7.0, device=cuda, dtype=bf)
    M.memory_readout(q, pool, [1] * n, D ** -0.5, gate, w, softcap=10.0, residual=res, out=out, state_slots=bad)
    torch.cuda.synchronize()
    assert torch.equal(out[1], torch.full_like(out[1], 7.0))
    assert torch.equal(out[0], ref[0]) and torch.equal(out[2], ref[2])


@pytest.mark.parametrize("D", [128, 256])
def test_update_in_a_state_pool(cuda, D):
    """The update reading its initial states from and writing its final states into a state
    pool by slot index (in place, no gather and no index_copy_) equals the gathered update;
    slots not named stay untouched, and the read of the same pool sees the incoming states."""
    bf = torch.bfloat16
    H, S = 4, 9
    x = to_bf16(make_inputs(13, [500, 64, 333], H, D, gate="channel", beta=None, erase=False, write=True))
    gen = torch.Generator(device=cuda).manual_seed(4)
    pool = 0.05 * torch.randn(S, H, D, D, device=cuda, generator=gen)
    slots = torch.tensor([6, 0, 3], dtype=torch.int32, device=cuda)
    before = pool.clone()
    gathered = pool[slots.long()].contiguous()
    q, k, v = (_t(x[n], cuda, bf)[None] for n in ("q", "k", "v"))
    g, w = _t(x["g"], cuda)[None], _t(x["w"], cuda, bf)[None]
    args = dict(lengths=x["lengths"], scale=D ** -0.5, chunk_tokens=2048)
    r_ref, f_ref = M.token_memory_packed(q, k, v, g, w, gathered, gathered.clone(), **args)
    r_got, pool_out = M.token_memory_packed(q, k, v, g, w, pool, pool, read_slots=slots, write_slots=slots, **args)
    torch.cuda.synchronize()
    assert pool_out.data_ptr() == pool.data_ptr()
    assert torch.equal(r_got, r_ref)
    assert torch.equal(pool[slots.long()], f_ref)
    others = [i for i in range(S) if i not in (6, 0, 3)]
    assert torch.equal(pool[others], before[others])


@pytest.mark.parametrize("D", [128, 256])
def test_update_partial_chunk_ignores_next_sample(cuda, D):
    """The last chunk of a sample is a 64-row tile whose rows past the sample are the next
    sample's tokens (the tile loads do not stop at the sample end). Non-finite values there
    must not reach the sample's result."""
    x = to_bf16(make_inputs(11, [100, 60], 2, D, gate="head", beta="head", erase=False, write=True))
    first = {k_: (v_[:100] if k_ in ("q", "k", "v", "g", "beta", "w") and v_ is not None else v_) for k_, v_ in x.items()}
    first.update(lengths=[100], cu=np.array([0, 100], np.int32), h0=x["h0"][:1])
    for key in ("k", "v", "w", "beta"):
        x[key] = x[key].copy()
        x[key][100:] = np.nan
    out = gpu_update(x, cuda, torch.bfloat16, 2048)
    torch.cuda.synchronize()
    got = out[0:1].cpu().numpy()
    assert np.isfinite(got).all()
    assert O.rel_fro(got, oracle_update(first, 2048, "bf16")) <= TOL_BF16


def test_update_extreme_decay_slow_path(cuda):
    """Channels that decay by ~2^-40 per token overflow any factorised exponent; the kernel
    must switch to exact per-pair exponents (as the reference's diagonal kernel does)."""
    x = make_inputs(7, [200, 64], 2, 128, gate="channel", beta="head", erase=False, write=True)
    x["g"][:, :, ::5] = -28.0
    x = to_bf16(x)
    out = gpu_update(x, cuda, torch.bfloat16, 2048)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert O.rel_fro(got, oracle_update(x, 2048, "bf16")) <= TOL_BF16


@pytest.mark.parametrize("D", [128, 256])
def test_update_in_place(cuda, D):
    x = to_bf16(make_inputs(11, [100, 37], 2, D))
    state = _t(x["h0"], cuda)
    out = gpu_update(x, cuda, torch.bfloat16, 2048, final_state=state, h0=state)
    torch.cuda.synchronize()
    assert out.data_ptr() == state.data_ptr()
    assert O.rel_fro(state.cpu().numpy(), oracle_update(x, 2048, "bf16")) <= TOL_BF16


@pytest.mark.parametrize("D", [64, 256])
def test_update_zero_state_and_single_token_samples(cuda, D):
    x = to_bf16(make_inputs(12, [1, 1, 1, 2], 2, D, state=False))
    out = gpu_update(x, cuda, torch.bfloat16, 2048)
    torch.cuda.synchronize()
    assert O.rel_fro(out.cpu().numpy(), oracle_update(x, 2048, "bf16")) <= TOL_BF16


@pytest.mark.parametrize("D", [128, 256])
def test_update_empty_sample_keeps_its_state(cuda, D):
    """A sample with no tokens (equal offsets) has no chunks: its final state is its initial
    state, and its neighbours are unaffected."""
    x = to_bf16(make_inputs(14, [100, 0, 70], 2, D))
    out = gpu_update(x, cuda, torch.bfloat16, 2048)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.array_equal(got[1], x["h0"][1].astype(np.float32))
    assert O.rel_fro(got, oracle_update(x, 2048, "bf16")) <= TOL_BF16


def test_update_workspace_status_clean(cuda):
    x = to_bf16(make_inputs(13, [70, 3], 2, 128))
    gpu_update(x, cuda, torch.bfloat16, 2048)
    from memt_b200 import _lib
    import ctypes
    lib = _lib.load()
    ws = ops.Workspace.get(cuda, 0)
    st = ctypes.c_int32(-1)
    _lib.check(lib.memt_gdn2_workspace_status(ctypes.c_void_p(ws.data_ptr()),
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                              ctypes.byref(st)), "status")
    assert st.value == 0


# ---------------------------------------------------------------------------
# reads
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("lengths", [[1, 1, 1], [3, 16, 2], [70, 1, 130], [600]])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_read_bf16(cuda, lengths, D):
    rng = np.random.default_rng(D + len(lengths))
    L, N, H = sum(lengths), len(lengths), 2
    q = O.bf16(rng.standard_normal((L, H, D)) / np.sqrt(D)).astype(np.float32)
    S = (0.05 * rng.standard_normal((N, H, D, D))).astype(np.float32)
    out = M.snapshot_read(_t(q, cuda, torch.bfloat16)[None], _t(S, cuda), lengths, D ** -0.5)
    torch.cuda.synchronize()
    cu = np.concatenate([[0], np.cumsum(lengths)])
    ref = O.read(q, S, cu, D ** -0.5, mode="bf16")
    got = out[0].float().cpu().numpy()
    assert O.rel_fro(got, ref) <= TOL_BF16
    assert np.mean(got != ref.astype(np.float32)) < 0.02


@pytest.mark.parametrize("lengths", [[16384] * 4, [16384, 1000, 7000, 3]])
def test_read_d256_long_blocks_over_one_wave(cuda, lengths):
    """A d = 256 read on its own spreads each block's runs of 1024 tokens over one resident wave
    of CTAs (64 blocks here: two CTAs a block, eight runs each, one snapshot conversion per CTA).
    Every token of every block is read, ragged and 3-token blocks included: the whole output
    against an fp32 product on the GPU, and the first and last 64 tokens of each block against
    the oracle's emulation of the reference's rounding."""
    H, D = 16, 256
    gen = torch.Generator(device=cuda).manual_seed(21)
    L, N = sum(lengths), len(lengths)
    q = (torch.randn(L, H, D, device=cuda, generator=gen) / D ** 0.5).to(torch.bfloat16)
    S = 0.05 * torch.randn(N, H, D, D, device=cuda, generator=gen)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    scale = D ** -0.5
    out = ops._read(q, S, torch.from_numpy(cu).to(cuda), N, max(lengths), scale, torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    Sb = S.to(torch.bfloat16).float()
    for n in range(N):
        a, b = int(cu[n]), int(cu[n + 1])
        # fp32 product, rounded to the output's bf16 as the kernel rounds it
        ref = (torch.einsum("thk,hkv->thv", q[a:b].float(), Sb[n]) * scale).to(torch.bfloat16).float()
        assert O.rel_fro(out[a:b].float().cpu().numpy(), ref.cpu().numpy()) <= TOL_BF16
        for lo, hi in ((a, min(a + 64, b)), (max(b - 64, a), b)):
            qs = q[lo:hi].float().cpu().numpy()
            ref_o = O.read(qs, S[n:n + 1].cpu().numpy(), np.array([0, hi - lo]), scale, mode="bf16")
            assert O.rel_fro(out[lo:hi].float().cpu().numpy(), ref_o) <= TOL_BF16


@pytest.mark.parametrize("D", [128, 256])
def test_read_tile_kernel_fp32_output(cuda, D):
    """bf16 queries read into an fp32 output on the tensor-core tile kernel: every row of the
    ragged blocks (a full-tile block, one ending mid-tile, a 3-token block) equals the fp32
    product q . bf16(S) times the scale (fp32 accumulation, so only summation order differs)."""
    lengths = [1024, 645, 3]
    H = 4
    gen = torch.Generator(device=cuda).manual_seed(D)
    L, N = sum(lengths), len(lengths)
    q = (torch.randn(L, H, D, device=cuda, generator=gen) / D ** 0.5).to(torch.bfloat16)
    S = 0.05 * torch.randn(N, H, D, D, device=cuda, generator=gen)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    scale = D ** -0.5
    out = ops._read(q, S, torch.from_numpy(cu).to(cuda), N, max(lengths), scale, torch.float32)
    torch.cuda.synchronize()
    Sb = S.to(torch.bfloat16).float()
    for n in range(N):
        a, b = int(cu[n]), int(cu[n + 1])
        ref = torch.einsum("thk,hkv->thv", q[a:b].float(), Sb[n]) * scale
        assert O.rel_fro(out[a:b].cpu().numpy(), ref.cpu().numpy()) <= 1e-5, n


@pytest.mark.parametrize("lengths", [[1, 2], [5, 40, 3]])
def test_read_fp32_exact(cuda, lengths):
    rng = np.random.default_rng(3)
    L, N, H, D = sum(lengths), len(lengths), 2, 128
    q = rng.standard_normal((L, H, D)).astype(np.float32)
    S = rng.standard_normal((N, H, D, D)).astype(np.float32)
    out = M.snapshot_read(_t(q, cuda)[None], _t(S, cuda), lengths, 0.1)
    torch.cuda.synchronize()
    ref = O.read(q, S, np.concatenate([[0], np.cumsum(lengths)]), 0.1)
    assert O.rel_fro(out[0].cpu().numpy(), ref) <= TOL_F32


def test_read_golden(golden, cuda):
    z = golden("read_qwen")
    plan = M.build_chunk_plan(torch.from_numpy(z["cu_seqlens"]).to(cuda), torch.from_numpy(z["cu_seqlens"]).to(cuda),
                              event_slice=torch.from_numpy(z["cu_seqlens"]).to(cuda))
    out = M.memt_gdn2_read_fwd(_t(z["q"], cuda)[None], _t(z["states"], cuda), plan, float(z["scale"]),
                               torch.float32)
    torch.cuda.synchronize()
    assert O.rel_fro(out[0].cpu().numpy(), z["read"]) <= TOL_F32


# ---------------------------------------------------------------------------
# fused readout
# ---------------------------------------------------------------------------

def test_readout_against_reference_bf16_golden(golden, cuda):
    z = golden("readout_bf16")
    lengths = [int(n) for n in z["lengths"]]
    bf = torch.bfloat16
    out = _t(z["attn"], cuda, bf).clone()
    M.memory_readout(_t(z["q_raw"], cuda, bf), _t(z["states"], cuda), lengths, float(z["scale"]),
                     _t(z["gate"], cuda, bf), _t(z["weight"], cuda, bf), eps=float(z["eps"]),
                     softcap=float(z["softcap"]), residual=out, out=out, normalize_q=True)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert O.rel_fro(got, z["residual"]) <= 4e-3  # the reference's own bf16 pipeline (bmm order differs)
    ref = O.readout_fused(z["q_raw"], z["states"], z["cu_seqlens"], float(z["scale"]), z["gate"], z["weight"],
                          float(z["eps"]), float(z["softcap"]), z["attn"], normalize_q=True, mode="bf16")
    assert O.rel_fro(got, ref) <= TOL_BF16


@pytest.mark.parametrize("lengths", [[1] * 9, [2, 1, 30], [100, 1]])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_readout_fused_parity(cuda, lengths, D):
    rng = np.random.default_rng(D * 7 + sum(lengths))
    L, N, H = sum(lengths), len(lengths), 3
    cu = np.concatenate([[0], np.cumsum(lengths)])
    q = O.bf16(rng.standard_normal((L, H, D))).astype(np.float32)
    S = (0.05 * rng.standard_normal((N, H, D, D))).astype(np.float32)
    gate = O.bf16(rng.normal(0.5, 2.0, (L, H, D))).astype(np.float32)
    w = O.bf16(rng.normal(1.0, 0.1, (D,))).astype(np.float32)
    head_offset = 1
    attn = O.bf16(rng.standard_normal((L, (H + head_offset) * D))).astype(np.float32)
    bf = torch.bfloat16
    out = _t(attn, cuda, bf)
    M.memory_readout(_t(q, cuda, bf), _t(S, cuda), lengths, D ** -0.5, _t(gate, cuda, bf), _t(w, cuda, bf),
                     eps=1e-6, softcap=10.0, residual=out, out=out, head_offset=head_offset, normalize_q=True)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    y = O.readout_fused(q, S, cu, D ** -0.5, gate, w, 1e-6, 10.0, None, normalize_q=True, mode="bf16")
    ref = attn.astype(np.float64).copy()
    ref[:, head_offset * D:] = O.bf16(ref[:, head_offset * D:] + y)
    assert np.array_equal(got[:, :head_offset * D], attn[:, :head_offset * D])  # other heads untouched
    assert O.rel_fro(got, ref) <= TOL_BF16


# ---------------------------------------------------------------------------
# full-size properties (BASELINE config 1 geometry)
# ---------------------------------------------------------------------------

def test_config1_pack_independence_and_sampled_oracle(cuda):
    """B=8 x T=8192, H=16, d=128. Each sample's result must not depend on the others
    (bitwise) and one (sample, head) slice is checked against the oracle."""
    lengths, H, D = [8192] * 8, 16, 128
    rng = np.random.default_rng(0)
    L = sum(lengths)
    gen = torch.Generator(device=cuda).manual_seed(0)
    bf = torch.bfloat16

    def nrm(x):
        return (x / torch.sqrt((x.float() ** 2).sum(-1, keepdim=True) + 1e-6)).to(bf)

    k = nrm(torch.randn(L, H, D, device=cuda, generator=gen))
    v = torch.randn(L, H, D, device=cuda, generator=gen).to(bf)
    g = torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L, H, device=cuda, generator=gen))
    beta = torch.sigmoid(torch.randn(L, H, device=cuda, generator=gen)).to(bf)
    w = torch.sigmoid(torch.randn(L, H, D, device=cuda, generator=gen)).to(bf)
    h0 = 0.02 * torch.randn(8, H, D, D, device=cuda, generator=gen)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=cuda)
    full = ops.gdn2_update(k, v, g, h0, cu, num_samples=8, total_tokens=L, beta=beta, write=w)
    n = 5
    sl = slice(n * 8192, (n + 1) * 8192)
    one = ops.gdn2_update(k[sl], v[sl], g[sl], h0[n:n + 1].contiguous(),
                          torch.tensor([0, 8192], dtype=torch.int32, device=cuda), num_samples=1,
                          total_tokens=8192, beta=beta[sl], write=w[sl])
    torch.cuda.synchronize()
    assert torch.isfinite(full).all()
    assert torch.equal(full[n], one[0])
    h = 9
    x = dict(lengths=[8192], cu=np.array([0, 8192], np.int32),
             k=k[sl, h:h + 1].float().cpu().numpy(), v=v[sl, h:h + 1].float().cpu().numpy(),
             g=g[sl, h:h + 1].cpu().numpy(), beta=beta[sl, h:h + 1].float().cpu().numpy(), erase=None,
             w=w[sl, h:h + 1].float().cpu().numpy(), h0=h0[n:n + 1, h:h + 1].cpu().numpy())
    ref = oracle_update(x, 2048, "bf16")
    assert O.rel_fro(full[n, h:h + 1].cpu().numpy()[None], ref) <= TOL_BF16


def _device_inputs(dev, lengths, H, D, seed):
    gen = torch.Generator(device=dev).manual_seed(seed)
    bf = torch.bfloat16
    L = sum(lengths)

    def nrm(t):
        return (t / torch.sqrt((t.float() ** 2).sum(-1, keepdim=True) + 1e-6)).to(bf)

    return dict(
        k=nrm(torch.randn(L, H, D, device=dev, generator=gen)),
        v=torch.randn(L, H, D, device=dev, generator=gen).to(bf),
        g=torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L, H, device=dev, generator=gen)),
        beta=torch.sigmoid(torch.randn(L, H, device=dev, generator=gen)).to(bf),
        w=torch.sigmoid(torch.randn(L, H, D, device=dev, generator=gen)).to(bf),
        h0=0.02 * torch.randn(len(lengths), H, D, D, device=dev, generator=gen),
        cu=torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev))


def _oracle_slice(x, t0, t1, n, h):
    return dict(lengths=[t1 - t0], cu=np.array([0, t1 - t0], np.int32),
                k=x["k"][t0:t1, h:h + 1].float().cpu().numpy(), v=x["v"][t0:t1, h:h + 1].float().cpu().numpy(),
                g=x["g"][t0:t1, h:h + 1].cpu().numpy(), beta=x["beta"][t0:t1, h:h + 1].float().cpu().numpy(),
                erase=None, w=x["w"][t0:t1, h:h + 1].float().cpu().numpy(),
                h0=x["h0"][n:n + 1, h:h + 1].cpu().numpy())


def test_config3_varlen_long_history(cuda):
    """32 packed sessions with lengths uniform in [1K, 32K] (about 512K
    tokens), H = 16, d = 128. Sessions of the pack are independent (bitwise, checked on a
    short, a long and the last session, each run alone) and the shortest session matches the
    oracle."""
    rng = np.random.default_rng(3)
    lengths = rng.integers(1024, 32768, 32).tolist()
    H, D = 16, 128
    x = _device_inputs(cuda, lengths, H, D, 3)
    L = sum(lengths)
    full = ops.gdn2_update(x["k"], x["v"], x["g"], x["h0"], x["cu"], num_samples=32, total_tokens=L,
                           beta=x["beta"], write=x["w"])
    cu = np.concatenate([[0], np.cumsum(lengths)])
    short = int(np.argmin(lengths))
    for n in sorted({short, int(np.argmax(lengths)), 31}):
        t0, t1 = int(cu[n]), int(cu[n + 1])
        one = ops.gdn2_update(x["k"][t0:t1], x["v"][t0:t1], x["g"][t0:t1], x["h0"][n:n + 1].contiguous(),
                              torch.tensor([0, t1 - t0], dtype=torch.int32, device=cuda), num_samples=1,
                              total_tokens=t1 - t0, beta=x["beta"][t0:t1], write=x["w"][t0:t1])
        torch.cuda.synchronize()
        assert torch.equal(full[n], one[0]), n
    assert torch.isfinite(full).all()
    h = 11
    t0, t1 = int(cu[short]), int(cu[short + 1])
    ref = oracle_update(_oracle_slice(x, t0, t1, short, h), 2048, "bf16")
    assert O.rel_fro(full[short, h:h + 1].cpu().numpy()[None], ref) <= TOL_BF16


def test_config4_flash_shaped(cuda):
    """BASELINE config 4 geometry: H = 128 memory heads, d = 256, bf16 inputs, fp32 state
    (B = 4 sessions, shortened from 16K to 2K tokens each so the oracle check stays quick).
    Head slices of a tensor-parallel rank (16 of 128 heads) reproduce the full run bitwise,
    and one head matches the oracle."""
    lengths, H, D = [2048] * 4, 128, 256
    x = _device_inputs(cuda, lengths, H, D, 4)
    L = sum(lengths)
    full = ops.gdn2_update(x["k"], x["v"], x["g"], x["h0"], x["cu"], num_samples=4, total_tokens=L,
                           beta=x["beta"], write=x["w"])
    from memt_b200 import shard
    h0, h1 = shard.head_range(3, 8, H)
    part = ops.gdn2_update(x["k"][:, h0:h1], x["v"][:, h0:h1], x["g"][:, h0:h1], x["h0"][:, h0:h1].contiguous(),
                           x["cu"], num_samples=4, total_tokens=L, beta=x["beta"][:, h0:h1], write=x["w"][:, h0:h1])
    torch.cuda.synchronize()
    assert torch.equal(full[:, h0:h1], part)
    n, h = 2, 77
    ref = oracle_update(_oracle_slice(x, 2048 * n, 2048 * (n + 1), n, h), 2048, "bf16")
    assert O.rel_fro(full[n, h:h + 1].cpu().numpy()[None], ref) <= TOL_BF16


# ---------------------------------------------------------------------------
# host-side validation (reference raises ValueError before launch)
# ---------------------------------------------------------------------------

def test_invalid_arguments_raise(cuda):
    x = to_bf16(make_inputs(5, [10, 6], 2, 64))
    bf = torch.bfloat16
    args = (_t(x["q"], cuda, bf)[None], _t(x["k"], cuda, bf)[None], _t(x["v"], cuda, bf)[None],
            _t(x["g"], cuda)[None], _t(x["w"], cuda, bf)[None], _t(x["r0"], cuda), _t(x["h0"], cuda))
    with pytest.raises(ValueError):
        M.token_memory_packed(*args, lengths=[10, 5], scale=0.1, chunk_tokens=2048)  # lengths do not cover L
    with pytest.raises(ValueError):
        M.token_memory_packed(*args, lengths=[16, 0], scale=0.1, chunk_tokens=2048)  # empty sample
    bad = list(args)
    bad[5] = bad[5].double()
    with pytest.raises(ValueError):
        M.token_memory_packed(*bad, lengths=[10, 6], scale=0.1, chunk_tokens=2048)  # fp64 states
    bad = list(args)
    bad[3] = bad[3].to(bf)
    with pytest.raises(ValueError):
        M.token_memory_packed(*bad, lengths=[10, 6], scale=0.1, chunk_tokens=2048)  # bf16 log-decay
