"""The DeepSeek (Flash) memory block's projections around the GDN-2 path.

Paths are relative to the reference package ``inference/memt_sglang``:

* ``expand_grouped_qkv``  models/deepseek/ops/compiled_tensor_ops.py:23-41: the low-rank q latent
                          RMS-normalised and up-projected; the k and v latents normalised per
                          group (each group its own epsilon) and expanded by a grouped
                          up-projection. The norms run in one kernel (memt_latent_rms_norm); the
                          projections are plain GEMMs (cuBLAS, grouped as one batched GEMM).
* ``head_inputs``         expand_write_gates + prepare_stable_qk (compiled_tensor_ops.py:54-78,
                          102-107) after the b_up / w_up / f_down GEMMs: l2norm of q and k
                          (rsqrt form), the sqrt-erase factor folded into k, the write sigmoid and
                          the softplus log-decay, in the prologue kernel (memt_qwen_prologue).
* ``memory_inject``       the wo_a injection of the memory output into the wo_b input
                          (models/deepseek/integration.py:56-61,66-72): per group, the memory's
                          heads times that group's wo_a rows, added to the residual in one batched
                          GEMM whose epilogue does the add (beta = 1).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import _stream, qwen_prologue

__all__ = ["latent_rms_norm", "expand_grouped_qkv", "head_inputs", "memory_inject"]


def latent_rms_norm(x, weight, eps):
    """bf16 [..., G * R] (token rows, any row stride) -> bf16 [T, G, R]:
    bf16((x * rsqrt(mean(x^2) + eps[g])) * weight[g]) per (token, group) row, fp32 math.
    weight: bf16 [G, R] (or [R] for one group); eps: a float, or one per group."""
    if weight.dim() == 1:
        weight = weight.view(1, -1)
    G, R = weight.shape
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.shape[-1] != G * R or x2.stride(-1) != 1 or x2.dtype != torch.bfloat16 or not x2.is_cuda:
        raise ValueError(f"latent rows must be bf16 [T, {G * R}] with contiguous rows")
    if weight.dtype != torch.bfloat16 or weight.device != x2.device:
        raise ValueError("weight must be bf16 on the latent's device")
    T = x2.shape[0]
    weight = weight.contiguous()
    out = torch.empty(T, G, R, device=x2.device, dtype=torch.bfloat16)
    eps_t = None
    if isinstance(eps, (tuple, list, torch.Tensor)):
        eps_t = torch.as_tensor(eps, dtype=torch.float32).reshape(G).to(x2.device)
    args = _lib.LatentNormArgs(groups=G, rank=R, total_tokens=T, x=x2.data_ptr(),
                               x_stride=x2.stride(0) if T > 1 else G * R, weight=weight.data_ptr(),
                               eps=eps_t.data_ptr() if eps_t is not None else None,
                               eps_scalar=float(eps) if eps_t is None else 0.0, out=out.data_ptr())
    _lib.check(_lib.load().memt_latent_rms_norm(ctypes.byref(args), _stream(x2.device)), "memt_latent_rms_norm")
    return out


def expand_grouped_qkv(q, k, v, q_norm, q_up, q_eps, k_up, v_up, k_norm, v_norm, k_eps, v_eps):
    """(q, k, v) of the DeepSeek memory block from its low-rank latents, with the reference's
    signature (compiled_tensor_ops.py:23-41). q: [..., q_rank]; k, v: [..., G * rank];
    q_up [value_dim, q_rank]; k_up, v_up [G, width, rank]; k_norm, v_norm [G, rank]."""
    lead = q.shape[:-1]
    qn = latent_rms_norm(q, q_norm, q_eps)
    q_out = torch.nn.functional.linear(qn.view(qn.shape[0], -1), q_up)

    def expand(latent, weight, gain, eps):
        groups, width, rank = weight.shape
        n = latent_rms_norm(latent, gain, eps)                       # [T, G, R]
        y = torch.bmm(n.transpose(0, 1), weight.transpose(1, 2))      # [G, T, width]
        return y.transpose(0, 1).reshape(*lead, groups * width)

    return q_out.reshape(*lead, -1), expand(k, k_up, k_norm, k_eps), expand(v, v_up, v_norm, v_eps)


def head_inputs(q, k, erase, write, decay, decay_bias, decay_scale_log, *, eps=1e-6):
    """(query, key, write, log_decay) for the update from the DeepSeek block's projections:
    l2norm(q), bf16(bf16(l2norm(k)) * bf16(exp(0.5 logsigmoid(erase)))), sigmoid(write) and
    -exp(decay_scale_log) softplus(decay + decay_bias), with the rsqrt l2norm of
    models/deepseek/ops/normalization.py:6-8. erase, write, decay: the b_up, w_up, f_down
    outputs [..., H * D]."""
    return qwen_prologue(q, k, erase, write, decay, decay_bias, decay_scale_log, eps=eps, rsqrt_norm=True)


def memory_inject(memory, wo_a_weight, groups, residual):
    """residual += einsum("tgd,grd->tgr", memory as [T, groups, d], wo_a as [groups, r, d]),
    flattened to [T, groups * r] (models/deepseek/integration.py:56-61,66-72), in place, with
    fp32 accumulation and one rounding of the sum. Returns residual."""
    T = memory.shape[0]
    m = memory.reshape(T, groups, -1)
    w = wo_a_weight.reshape(groups, -1, m.shape[-1])
    if residual.shape != (T, groups * w.shape[1]) or not residual.is_contiguous():
        raise ValueError(f"residual must be a contiguous [{T}, {groups * w.shape[1]}] tensor")
    r = residual.view(T, groups, -1).transpose(0, 1)                # [G, T, r] view of residual
    r.baddbmm_(m.transpose(0, 1), w.transpose(1, 2))                # C += A B in the GEMM epilogue
    return residual
