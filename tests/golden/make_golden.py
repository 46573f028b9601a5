"""Generate golden vectors for the GDN-2 memory hot path from the reference itself.

This script is test infrastructure. It imports the MemT-1.0 reference package
(``memt_sglang``) from a local checkout, runs its own operators on CPU and stores
seeded inputs together with the reference outputs as ``.npz`` fixtures next to
this file. The fixtures are what the CPU and GPU tests compare against; the
reference checkout itself is never needed at test time.

How the reference runs on CPU:
  * Triton kernels run under ``TRITON_INTERPRET=1`` (numpy semantics, fp32 only;
    bf16 under the interpreter is not usable, so Triton cases are fp32).
  * Autotuned kernels keep only their first config (the interpreter cannot
    benchmark); ``MEMT_NO_AUTOTUNE=1`` selects the reference's own fixed config.
  * Pure-PyTorch reference operators (``snapshot_read``, ``MemTRMSNormGated``,
    DeepSeek ``_gated_rms_norm``, DeepSeek ``l2norm``) run in bf16 on CPU, which
    gives real bf16 goldens for the readout and its epilogue.

Usage:  python tests/golden/make_golden.py --reference <path to MemT-1.0 checkout>
"""

import argparse
import os
import sys
import time
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("MEMT_NO_AUTOTUNE", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def _patch_autotuner():
    from triton.runtime import autotuner

    original = autotuner.Autotuner.run

    def run(self, *args, **kwargs):
        if len(self.configs) > 1:
            self.configs = self.configs[:1]
        return original(self, *args, **kwargs)

    autotuner.Autotuner.run = run


def _lengths_to_cu(lengths):
    return np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)


def _inputs(seed, lengths, H, D, *, channel_gates, with_erase, nonzero_state, dtype=np.float32):
    """Seeded inputs with the distributions of the BASELINE configs.

    q, k ~ N(0,1) then L2-normalised per head row; v ~ N(0,1);
    log-decay = logsigmoid(N(2, 0.5)) (per head-token broadcast over K, or per channel);
    beta = sigmoid(N(0,1)) folded as sqrt(beta) into the key (stable GDN-2);
    write gate = sigmoid(N(0,1)) per (token, head, V channel);
    erase b (FLA's channel-wise erase factor) = ones or sigmoid(N(0,1)) per channel.
    """
    rng = np.random.default_rng(seed)
    L = int(sum(lengths))
    N = len(lengths)
    q = rng.standard_normal((L, H, D)).astype(np.float32)
    k = rng.standard_normal((L, H, D)).astype(np.float32)
    v = rng.standard_normal((L, H, D)).astype(np.float32)
    q /= np.sqrt((q.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6).astype(np.float32)
    k /= np.sqrt((k.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6).astype(np.float32)
    if channel_gates:
        z = rng.normal(2.0, 0.5, (L, H, D))
    else:
        z = np.broadcast_to(rng.normal(2.0, 0.5, (L, H, 1)), (L, H, D))
    g = (-np.logaddexp(0.0, -z)).astype(np.float32)  # logsigmoid
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((L, H, 1))))).astype(np.float32)
    k = (np.sqrt(beta) * k).astype(np.float32)
    w = (1.0 / (1.0 + np.exp(-rng.standard_normal((L, H, D))))).astype(np.float32)
    if with_erase:
        b = (1.0 / (1.0 + np.exp(-rng.standard_normal((L, H, D))))).astype(np.float32)
    else:
        b = np.ones((L, H, D), np.float32)
    if nonzero_state:
        h0 = (0.02 * rng.standard_normal((N, H, D, D))).astype(np.float32)
        r0 = (0.02 * rng.standard_normal((N, H, D, D))).astype(np.float32)
    else:
        h0 = np.zeros((N, H, D, D), np.float32)
        r0 = h0.copy()
    return dict(q=q, k=k, v=v, g=g, w=w, b=b, h0=h0, r0=r0,
                lengths=np.asarray(lengths, np.int32), cu_seqlens=_lengths_to_cu(lengths))


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x))


def qwen_packed_case(name, seed, lengths, H, D, *, channel_gates, with_erase, nonzero_state, chunk_tokens):
    from memt_sglang.models.qwen.ops.packed import token_memory_packed

    x = _inputs(seed, lengths, H, D, channel_gates=channel_gates, with_erase=with_erase,
                nonzero_state=nonzero_state)
    scale = D ** -0.5
    t0 = time.time()
    read, final = token_memory_packed(
        _t(x["q"])[None], _t(x["k"])[None], _t(x["v"])[None], _t(x["g"])[None],
        _t(x["w"])[None], _t(x["r0"]), _t(x["h0"]),
        erase=_t(x["b"])[None], lengths=[int(n) for n in lengths], scale=scale,
        chunk_tokens=chunk_tokens,
    )
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)
    np.savez_compressed(
        HERE / f"{name}.npz", **x, scale=np.float32(scale), chunk_tokens=np.int32(chunk_tokens),
        read=read[0].numpy(), final_state=final.numpy(), flavour=np.str_("qwen"),
    )


def flash_packed_case(name, seed, lengths, H, D, *, channel_gates, nonzero_state, chunk_tokens):
    from memt_sglang.models.deepseek.ops.packed import token_memory_packed

    x = _inputs(seed, lengths, H, D, channel_gates=channel_gates, with_erase=False,
                nonzero_state=nonzero_state)
    scale = D ** -0.5
    t0 = time.time()
    read, final = token_memory_packed(
        _t(x["q"])[None], _t(x["k"])[None], _t(x["v"])[None], _t(x["g"])[None],
        _t(x["w"])[None], _t(x["r0"]), _t(x["h0"]),
        lengths=[int(n) for n in lengths], scale=scale, chunk_tokens=chunk_tokens,
    )
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)
    np.savez_compressed(
        HERE / f"{name}.npz", **x, scale=np.float32(scale), chunk_tokens=np.int32(chunk_tokens),
        read=read[0].numpy(), final_state=final.numpy(), flavour=np.str_("flash"),
    )


def qwen_read_case(name, seed, lengths, H, D):
    """Query path of QwenMemoryBlock.packed: plan over samples, then the tiled read."""
    from memt_sglang.models.common.constants import WY_TILE_TOKENS
    from memt_sglang.models.common.packed import boundaries
    from memt_sglang.models.qwen.ops.layout import build_chunk_plan
    from memt_sglang.models.qwen.ops.read import memt_gdn2_read_fwd

    rng = np.random.default_rng(seed)
    L, N = int(sum(lengths)), len(lengths)
    q = rng.standard_normal((L, H, D)).astype(np.float32)
    q /= np.sqrt((q.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6).astype(np.float32)
    states = rng.standard_normal((N, H, D, D)).astype(np.float32)
    samples = boundaries(lengths, "cpu")
    plan = build_chunk_plan(samples, samples, WY_TILE_TOKENS, event_slice=samples,
                            commit_mask=torch.zeros(N, dtype=torch.bool))
    out = memt_gdn2_read_fwd(_t(q)[None], _t(states), plan, D ** -0.5, out_dtype=torch.float32)
    np.savez_compressed(HERE / f"{name}.npz", q=q, states=states, lengths=np.asarray(lengths, np.int32),
                        cu_seqlens=_lengths_to_cu(lengths), scale=np.float32(D ** -0.5), read=out[0].numpy())
    print(f"{name}: done", flush=True)


def bf16_readout_case(name, seed, lengths, H, D, softcap):
    """DeepSeek snapshot_read (bf16 bmm) followed by MemTRMSNormGated, both in bf16 on CPU,
    plus the Qwen/DeepSeek q preparation (l2norm) and the residual add into an attention row."""
    from memt_sglang.models.deepseek.ops.compiled_tensor_ops import _gated_rms_norm
    from memt_sglang.models.deepseek.ops.normalization import l2norm as ds_l2norm
    from memt_sglang.models.deepseek.ops.read import snapshot_read
    from memt_sglang.models.qwen.layer import MemTRMSNormGated

    rng = np.random.default_rng(seed)
    L, N = int(sum(lengths)), len(lengths)
    q_raw = torch.from_numpy(rng.standard_normal((L, H, D)).astype(np.float32)).to(torch.bfloat16)
    states = torch.from_numpy((0.05 * rng.standard_normal((N, H, D, D))).astype(np.float32))
    gate = torch.from_numpy(rng.normal(0.5, 2.0, (L, H, D)).astype(np.float32)).to(torch.bfloat16)
    weight = torch.from_numpy(rng.normal(1.0, 0.1, (D,)).astype(np.float32)).to(torch.bfloat16)
    attn = torch.from_numpy(rng.standard_normal((L, H * D)).astype(np.float32)).to(torch.bfloat16)
    q_hat = ds_l2norm(q_raw.float()).to(torch.bfloat16)
    read = snapshot_read(q_hat[None], states, [int(n) for n in lengths], D ** -0.5,
                         bf16_accumulator_output=True)[0]
    norm = MemTRMSNormGated(D, eps=1e-6, output_gate_softcap_limit=softcap)
    with torch.no_grad():
        norm.weight.copy_(weight.float())
        norm = norm.to(torch.bfloat16)
        y_qwen = norm(read.reshape(-1, D), gate.reshape(-1, D))
        y_ds = _gated_rms_norm(read.reshape(-1, D), gate.reshape(-1, D), weight, 1e-6,
                               "silu", True, softcap)
    residual = attn + y_qwen.view(L, H * D)

    def f32(t):
        return t.float().numpy()

    np.savez_compressed(
        HERE / f"{name}.npz", q_raw=f32(q_raw), q_hat=f32(q_hat), states=states.numpy(),
        gate=f32(gate), weight=f32(weight), attn=f32(attn), lengths=np.asarray(lengths, np.int32),
        cu_seqlens=_lengths_to_cu(lengths), scale=np.float32(D ** -0.5), softcap=np.float32(softcap),
        eps=np.float32(1e-6), read=f32(read), y_qwen=f32(y_qwen), y_deepseek=f32(y_ds),
        residual=f32(residual),
    )
    print(f"{name}: done", flush=True)


def l2norm_case(name, seed, rows, D):
    from memt_sglang._vendor.fla.modules.l2norm import l2norm_fwd

    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, D)).astype(np.float32)
    y, _ = l2norm_fwd(_t(x))
    np.savez_compressed(HERE / f"{name}.npz", x=x, y=y.numpy(), eps=np.float32(1e-6))
    print(f"{name}: done", flush=True)


def qwen_prologue_case(name, seed, L, H, D):
    """The Qwen memory block's own gate and input preparation on CPU: ``_write_gates`` (which
    calls ``_log_decay``) in bf16 on a block built from a small config, and
    ``_symmetric_inputs`` (the FLA l2norm, under the interpreter, so in fp32) on fp32 q, k and
    the block's erase factor."""
    from types import SimpleNamespace

    from memt_sglang.models.qwen.layer import QwenMemoryBlock

    rng = np.random.default_rng(seed)
    cfg = SimpleNamespace(hidden_size=64, num_heads=H, head_dim=D, chunk_tokens=2048, rms_norm_eps=1e-6,
                          output_gate_softcap=10.0)
    block = QwenMemoryBlock(cfg, device="cpu")
    bf = torch.bfloat16
    with torch.no_grad():
        block.f_down.weight.copy_(torch.from_numpy(0.3 * rng.standard_normal((H * D, D))).to(bf))
        block.decay_bias.copy_(torch.from_numpy(rng.normal(-1.0, 1.0, H * D)).to(bf))
        block.decay_scale_log.copy_(torch.from_numpy(rng.normal(0.0, 0.5, H)).to(bf))
    gates = torch.from_numpy(rng.normal(0.0, 2.0, (1, L, 2 * H * D + D)).astype(np.float32)).to(bf)
    *write_gates, decay_in = torch.split(gates, block.write_gate_rows, dim=-1)
    with torch.no_grad():
        decay_latent = block.f_down(decay_in)
        erase, write, log_decay = block._write_gates(gates, 1, L)
    q = rng.standard_normal((1, L, H, D)).astype(np.float32)
    k = rng.standard_normal((1, L, H, D)).astype(np.float32)
    q_hat, k_scaled, _ = QwenMemoryBlock._symmetric_inputs(_t(q), _t(k), erase.float())

    def f32(t):
        return t.detach().float().numpy()

    np.savez_compressed(
        HERE / f"{name}.npz", erase_gate=f32(write_gates[0]).reshape(L, H, D),
        write_gate=f32(write_gates[1]).reshape(L, H, D), decay_latent=f32(decay_latent).reshape(L, H, D),
        decay_bias=f32(block.decay_bias), decay_scale_log=f32(block.decay_scale_log),
        erase_sqrt=f32(erase)[0], write=f32(write)[0], log_decay=f32(log_decay)[0], q=q[0], k=k[0],
        q_hat=f32(q_hat)[0], k_scaled=f32(k_scaled)[0], eps=np.float32(1e-6))
    print(f"{name}: done", flush=True)


def flash_projection_case(name, seed, T, groups, rank, width, q_rank, H, D):
    """The DeepSeek memory block's projections, eager on CPU in bf16: expand_grouped_qkv
    (latent norms + grouped up-projections), expand_write_gates's gate math on given b_up /
    w_up / f_down outputs (the three linears replaced by identity weights) and
    prepare_stable_qk (DeepSeek rsqrt l2norm, erase fold)."""
    from memt_sglang.models.deepseek.ops.compiled_tensor_ops import (expand_grouped_qkv, expand_write_gates,
                                                                   prepare_stable_qk)

    rng = np.random.default_rng(seed)
    bf = torch.bfloat16

    def t(*shape, scale=1.0, mean=0.0):
        return torch.from_numpy((mean + scale * rng.standard_normal(shape)).astype(np.float32)).to(bf)

    q_lat, k_lat, v_lat = t(T, q_rank), t(T, groups * rank), t(T, groups * rank)
    q_norm, k_norm, v_norm = t(q_rank, scale=0.1, mean=1.0), t(groups, rank, scale=0.1, mean=1.0), \
        t(groups, rank, scale=0.1, mean=1.0)
    q_up = t(H * D, q_rank, scale=q_rank ** -0.5)
    k_up, v_up = t(groups, width, rank, scale=rank ** -0.5), t(groups, width, rank, scale=rank ** -0.5)
    eps = 1e-6
    with torch.no_grad():
        q, k, v = expand_grouped_qkv(q_lat, k_lat, v_lat, q_norm, q_up, eps, k_up, v_up, k_norm, v_norm,
                                     (eps,) * groups, (eps,) * groups)
        e_lat, w_lat, d_lat = t(1, T, H * D), t(1, T, H * D), t(1, T, H * D, mean=-2.0, scale=0.5)
        eye = torch.eye(H * D, dtype=bf)
        bias, scale_log = t(H * D, scale=0.3), t(H, scale=0.3)
        erase, write, log_decay = expand_write_gates(e_lat, w_lat, d_lat, eye, eye, eye, bias, scale_log, H, D)
        query, key = prepare_stable_qk(q.view(1, T, H, D), k.view(1, T, H, D), erase)

    def f32(x):
        return x.detach().float().numpy()

    np.savez_compressed(
        HERE / f"{name}.npz", q_lat=f32(q_lat), k_lat=f32(k_lat), v_lat=f32(v_lat), q_norm=f32(q_norm),
        k_norm=f32(k_norm), v_norm=f32(v_norm), q_up=f32(q_up), k_up=f32(k_up), v_up=f32(v_up), eps=np.float32(eps),
        q=f32(q), k=f32(k), v=f32(v), erase_gate=f32(e_lat)[0], write_gate=f32(w_lat)[0], decay_latent=f32(d_lat)[0],
        decay_bias=f32(bias), decay_scale_log=f32(scale_log), erase=f32(erase)[0], write=f32(write)[0],
        log_decay=f32(log_decay)[0], query=f32(query)[0], key=f32(key)[0], groups=np.int32(groups),
        heads=np.int32(H), head_dim=np.int32(D))
    print(f"{name}: done", flush=True)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path to the MemT-1.0 checkout")
    parser.add_argument("--only", default=None)
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "inference"))
    _patch_autotuner()
    torch.manual_seed(0)

    cases = {
        # B=1, H=4, T=512, d=64, fp32, per head-token gates, zero state.
        "cfg0_qwen": lambda: qwen_packed_case("cfg0_qwen", 0, [512], 4, 64, channel_gates=False,
                                              with_erase=False, nonzero_state=False, chunk_tokens=2048),
        # varlen, channel-wise gates, channel-wise erase b, nonzero states, several write events.
        "varlen_qwen": lambda: qwen_packed_case("varlen_qwen", 1, [100, 37, 64, 1, 65, 130], 2, 64,
                                                channel_gates=True, with_erase=True, nonzero_state=True,
                                                chunk_tokens=128),
        # d=128 (Nano geometry) on a short varlen pack.
        "d128_qwen": lambda: qwen_packed_case("d128_qwen", 2, [150, 63], 2, 128, channel_gates=True,
                                              with_erase=False, nonzero_state=True, chunk_tokens=2048),
        # DeepSeek/Flash writer (unit erase) with the bmm snapshot read.
        "varlen_flash": lambda: flash_packed_case("varlen_flash", 3, [100, 37, 64, 1, 65], 2, 64,
                                                  channel_gates=True, nonzero_state=True,
                                                  chunk_tokens=128),
        "read_qwen": lambda: qwen_read_case("read_qwen", 4, [1, 1, 3, 70, 64], 2, 64),
        "readout_bf16": lambda: bf16_readout_case("readout_bf16", 5, [1, 1, 1, 5, 1, 2], 2, 128, 10.0),
        "l2norm": lambda: l2norm_case("l2norm", 6, 300, 128),
        # the Qwen memory block's gates, decay and symmetric q/k inputs (layer.py:71-97)
        "qwen_prologue": lambda: qwen_prologue_case("qwen_prologue", 7, 37, 2, 64),
        # the DeepSeek block's grouped low-rank q/k/v expansion, gates and q/k preparation
        "flash_projections": lambda: flash_projection_case("flash_projections", 8, 33, 2, 64, 128, 96, 4, 64),
    }
    for name, fn in cases.items():
        if args.only and name not in args.only.split(","):
            continue
        fn()


if __name__ == "__main__":
    main()
