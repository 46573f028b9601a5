"""Pin the CPU oracle against the reference's own outputs (fixtures in tests/golden).

The fixtures were produced by tests/golden/make_golden.py, which runs the reference
plugin's operators on CPU: its Triton kernels under the Triton interpreter (fp32) and
its PyTorch readout / gated RMSNorm in bf16.
"""

import numpy as np
import pytest

from oracle import gdn2 as O

PACKED = ["cfg0_qwen", "varlen_qwen", "d128_qwen", "varlen_flash"]


def _chunked(z, mode):
    b = z["b"] if str(z["flavour"]) == "qwen" else None
    return O.chunked(z["q"], z["k"], z["v"], z["g"], z["h0"], z["r0"], z["cu_seqlens"], float(z["scale"]),
                     b=b, w=z["w"], chunk_tokens=int(z["chunk_tokens"]), mode=mode)


@pytest.mark.parametrize("name", PACKED)
def test_chunked_exact_matches_reference(golden, name):
    z = golden(name)
    o, s = _chunked(z, "exact")
    # the reference ran in fp32 on the interpreter; the oracle is float64
    assert O.rel_fro(s, z["final_state"]) < 2e-6
    if np.abs(z["read"]).sum() > 0:
        assert O.rel_fro(o, z["read"]) < 2e-6


@pytest.mark.parametrize("name", PACKED)
def test_recurrence_matches_reference(golden, name):
    z = golden(name)
    b = z["b"] if str(z["flavour"]) == "qwen" else None
    s = O.recurrence(z["k"], z["v"], z["g"], z["h0"], z["cu_seqlens"], b=b, w=z["w"])
    assert O.rel_fro(s, z["final_state"]) < 2e-6


@pytest.mark.parametrize("name", PACKED)
def test_bf16_emulation_is_close_to_exact(golden, name):
    """The reference's GPU rounding points keep it within a few 1e-3 of exact math."""
    z = golden(name)
    _, s_exact = _chunked(z, "exact")
    _, s_bf16 = _chunked(z, "bf16")
    err = O.rel_fro(s_bf16, s_exact)
    assert 1e-5 < err < 1e-2


def test_read_matches_reference(golden):
    z = golden("read_qwen")
    o = O.read(z["q"], z["states"], z["cu_seqlens"], float(z["scale"]))
    assert O.rel_fro(o, z["read"]) < 1e-6


def test_l2norm_matches_reference(golden):
    z = golden("l2norm")
    y = O.l2norm(z["x"], float(z["eps"]))
    assert O.rel_fro(y, z["y"]) < 1e-6


def test_bf16_readout_pipeline_matches_reference(golden):
    """l2norm -> bf16 snapshot read -> gated RMSNorm -> residual, all in bf16 on the reference."""
    z = golden("readout_bf16")
    qh = O.l2norm(z["q_raw"], mode="bf16")
    assert np.array_equal(qh.astype(np.float32), z["q_hat"])
    o = O.read(z["q_hat"], z["states"], z["cu_seqlens"], float(z["scale"]), mode="bf16")
    # reference bf16 bmm vs oracle: identical rounding points, accumulation order differs
    assert O.rel_fro(o, z["read"]) < 4e-3
    D = z["read"].shape[-1]
    y = O.gated_rms_norm(z["read"].reshape(-1, D), z["gate"].reshape(-1, D), z["weight"], float(z["eps"]),
                         float(z["softcap"]), mode="bf16")
    assert O.rel_fro(y, z["y_qwen"]) < 4e-3
    assert O.rel_fro(y, z["y_deepseek"]) < 4e-3
    mism = np.mean(y.astype(np.float32) != z["y_qwen"].reshape(y.shape))
    assert mism < 0.02  # nearly bit-identical bf16 outputs
    full = O.readout_fused(z["q_raw"], z["states"], z["cu_seqlens"], float(z["scale"]), z["gate"], z["weight"],
                           float(z["eps"]), float(z["softcap"]), z["attn"], normalize_q=True, mode="bf16")
    assert O.rel_fro(full, z["residual"]) < 4e-3


@pytest.mark.parametrize("lengths,ct", [([1], 2048), ([63, 64, 65], 2048), ([300], 128), ([130, 7], 100),
                                        ([5000], 2048), ([1, 1, 1], 64)])
def test_plan_chunks(lengths, ct):
    cu = np.concatenate([[0], np.cumsum(lengths)])
    chunks = O.plan_chunks(cu, ct)
    # every token is covered exactly once, in order, by chunks of <= 64 tokens
    covered = []
    for n, t0, ln in chunks:
        assert 1 <= ln <= 64
        assert cu[n] <= t0 and t0 + ln <= cu[n + 1]
        covered.extend(range(t0, t0 + ln))
    assert covered == list(range(int(cu[-1])))
    # chunks never straddle a write event
    for n, t0, ln in chunks:
        assert (t0 - cu[n]) // ct == (t0 + ln - 1 - cu[n]) // ct


def test_rounding_helpers():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 1e-30, 65504.0], np.float64)
    b = O.bf16(x)
    # bf16 keeps 8 significant bits
    for v, r in zip(x, b):
        assert abs(v - r) <= abs(v) * 2 ** -8 + 1e-45
    assert O.bf16(np.array([1.00390625]))[0] == 1.0  # tie to even
    t = O.tf32(np.array([1.0 + 2 ** -11]))[0]
    assert t == 1.0 + 2 ** -10  # tie away from zero


def _bf16_ulps(a, b):
    """Per-element distance in bf16 units of the last place (both already bf16 values)."""
    ia = np.asarray(a, np.float32).view(np.int32) >> 16
    ib = np.asarray(b, np.float32).view(np.int32) >> 16
    return np.abs(ia.astype(np.int64) - ib.astype(np.int64))


def test_qwen_gates_match_reference(golden):
    """The reference's _write_gates / _log_decay (eager bf16 on CPU) against the oracle's
    float32 restatement: bf16 outputs within one unit of the last place (the libm exp and log1p
    of numpy and torch may differ by an ulp), log-decay within fp32 rounding."""
    z = golden("qwen_prologue")
    es, w, g = O.qwen_gates(z["erase_gate"], z["write_gate"], z["decay_latent"], z["decay_bias"],
                            z["decay_scale_log"], mode="bf16")
    for got, ref in ((es, z["erase_sqrt"]), (w, z["write"])):
        d = _bf16_ulps(got, ref)
        assert d.max() <= 1 and np.mean(d > 0) < 0.01
    assert O.rel_fro(g, z["log_decay"]) < 1e-6
    es_x, w_x, g_x = O.qwen_gates(z["erase_gate"], z["write_gate"], z["decay_latent"], z["decay_bias"],
                                  z["decay_scale_log"], mode="exact")
    assert O.rel_fro(g_x, z["log_decay"]) < 1e-6 and O.rel_fro(es_x, z["erase_sqrt"]) < 1e-2


def test_qwen_symmetric_inputs_match_reference(golden):
    """_symmetric_inputs (FLA l2norm of q and k, the erase factor folded into the key) run by the
    reference in fp32: the oracle's l2norm and product in float64."""
    z = golden("qwen_prologue")
    eps = float(z["eps"])
    assert O.rel_fro(O.l2norm(z["q"], eps), z["q_hat"]) < 1e-6
    assert O.rel_fro(z["erase_sqrt"] * O.l2norm(z["k"], eps), z["k_scaled"]) < 1e-6


@pytest.mark.parametrize("gate", ["head", "channel"])
def test_torch_cpu_restatement_matches_recurrence(gate):
    """The fp32 PyTorch chunked restatement (the timed CPU baseline) against the float64 token
    recurrence and the reference's own fp32 outputs."""
    import torch

    from oracle import gdn2_torch as OT

    rng = np.random.default_rng(17)
    lengths, H, D = [300, 64, 129, 1], 3, 64
    L = sum(lengths)
    cu = np.concatenate([[0], np.cumsum(lengths)])
    k = rng.standard_normal((L, H, D))
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((L, H, D))
    gshape = (L, H, D) if gate == "channel" else (L, H)
    g = -np.logaddexp(0, -rng.normal(2, .5, gshape))
    w = 1 / (1 + np.exp(-rng.standard_normal((L, H, D))))
    h0 = 0.02 * rng.standard_normal((4, H, D, D))
    g3 = g if g.ndim == 3 else np.broadcast_to(g[:, :, None], (L, H, D))
    ref = O.recurrence(k, v, g3, h0, cu, w=w)

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).float()

    got = OT.chunked_update(t(k), t(v), t(g), t(h0), cu, w=t(w), chunk_tokens=128).numpy()
    assert O.rel_fro(got, ref) < 1e-5


def test_torch_cpu_restatement_matches_reference_golden(golden):
    import torch

    from oracle import gdn2_torch as OT

    z = golden("d128_qwen")
    k = z["k"]

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).float()

    # d128_qwen has no channel-wise erase (b = 1), so the key is already the update's key
    assert np.allclose(z["b"], 1.0)
    s = OT.chunked_update(t(k), t(z["v"]), t(z["g"]), t(z["h0"]), list(z["cu_seqlens"]), w=t(z["w"]),
                          chunk_tokens=int(z["chunk_tokens"])).numpy()
    assert O.rel_fro(s, z["final_state"]) < 1e-5
    o = OT.read(t(z["q"]), t(z["r0"]), list(z["cu_seqlens"]), float(z["scale"])).numpy()
    assert O.rel_fro(o, z["read"]) < 1e-5


def test_flash_projections_match_reference(golden):
    """The DeepSeek block's projections run by the reference (eager, bf16 on CPU) against the
    oracle: the grouped latent norms and up-projections, the gates, the rsqrt l2norm of q and k
    with the erase fold. bf16 results: relative Frobenius within bf16 rounding (the reference
    accumulates its bf16 matmuls in its own order)."""
    z = golden("flash_projections")
    G = int(z["groups"])
    eps = float(z["eps"])
    q, k, v = O.expand_grouped_qkv(z["q_lat"], z["k_lat"], z["v_lat"], z["q_norm"], z["q_up"], eps, z["k_up"],
                                   z["v_up"], z["k_norm"], z["v_norm"], [eps] * G, [eps] * G)
    for got, ref in ((q, z["q"]), (k, z["k"]), (v, z["v"])):
        assert O.rel_fro(got, ref) < 5e-3
    es, w, g = O.qwen_gates(z["erase_gate"].reshape(z["erase"].shape), z["write_gate"].reshape(z["write"].shape),
                            z["decay_latent"].reshape(z["log_decay"].shape), z["decay_bias"], z["decay_scale_log"],
                            mode="bf16")
    assert O.rel_fro(es, z["erase"]) < 4e-3 and O.rel_fro(w, z["write"]) < 4e-3
    assert O.rel_fro(g, z["log_decay"]) < 1e-6
    H, D = int(z["heads"]), int(z["head_dim"])
    qh = O.l2norm(z["q"].reshape(-1, H, D), 1e-6)
    kh = O.bf16(O.l2norm(z["k"].reshape(-1, H, D), 1e-6)) * z["erase"]
    assert O.rel_fro(qh, z["query"]) < 4e-3 and O.rel_fro(kh, z["key"]) < 4e-3


def test_memory_inject_is_a_grouped_product():
    rng = np.random.default_rng(3)
    T, G, d, r = 5, 2, 8, 3
    m, w, res = rng.standard_normal((T, G * d)), rng.standard_normal((G * r, d)), rng.standard_normal((T, G * r))
    out = O.memory_inject(m, w, G, res)
    for g in range(G):
        assert np.allclose(out[:, g * r:(g + 1) * r], res[:, g * r:(g + 1) * r] + m[:, g * d:(g + 1) * d] @ w[g * r:(g + 1) * r].T)
