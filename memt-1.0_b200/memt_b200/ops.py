"""Drop-in operators for the MemT-1.0 memory hot path, backed by the sm_100a C ABI.

Signatures, argument meaning and error behaviour follow the reference plugin
(paths relative to ``inference/memt_sglang``):

* ``token_memory_packed``  models/qwen/ops/packed.py:34-81 (Qwen, with ``erase``) and
                           models/deepseek/ops/packed.py:70-108 (DeepSeek, no erase)
* ``memt_gdn2_read_fwd``   models/qwen/ops/read.py:10-39
* ``snapshot_read``        models/deepseek/ops/read.py:6-31
* ``memory_readout``       l2norm(q) -> read -> MemTRMSNormGated -> residual add
                           (models/qwen/layer.py:15-31,112-131; models/qwen/integration.py:61-64)
* ``qwen_prologue``        QwenMemoryBlock._write_gates / _log_decay / _symmetric_inputs and their
                           l2norm (models/qwen/layer.py:71-97)
* ``gdn2_chunked``         the BASELINE-style (q, k, v, g, beta, initial_state, cu_seqlens)
                           -> (o, final_state) entry over the same kernels.

Every operator runs on the current torch CUDA stream, never synchronises the host and
raises ``ValueError`` for invalid arguments before any launch (the reference checks in
models/common/packed.py:12-34 and runtime/executor.py:41-58).
"""

from __future__ import annotations

import ctypes
from collections import OrderedDict

import torch

from . import _lib
from .layout import ChunkPlan, read_segments

__all__ = [
    "token_memory_packed", "memt_gdn2_read_fwd", "snapshot_read", "memory_readout", "gdn2_chunked",
    "gdn2_update", "qwen_prologue", "Workspace",
]

_DTYPE = {torch.bfloat16: _lib.MEMT_BF16, torch.float32: _lib.MEMT_F32}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class Workspace:
    """Scratch for the update, one buffer per (device, stream), grown on demand and reused
    by later calls on the same stream (stream order keeps reuse race-free)."""

    _buffers: dict = {}

    @classmethod
    def get(cls, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.type, device.index, torch.cuda.current_stream(device).cuda_stream)
        buf = cls._buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            cls._buffers[key] = buf
        return buf


_cu_cache: OrderedDict = OrderedDict()


def _cu_seqlens(lengths, device) -> torch.Tensor:
    key = (tuple(lengths), device.type, device.index)
    hit = _cu_cache.get(key)
    if hit is not None:
        _cu_cache.move_to_end(key)
        return hit
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    t = torch.tensor(cu, dtype=torch.int32).to(device, non_blocking=True)
    _cu_cache[key] = t
    if len(_cu_cache) > 64:
        _cu_cache.popitem(last=False)
    return t


def _check_lengths(lengths, total):
    if not lengths or any(int(n) <= 0 for n in lengths) or sum(int(n) for n in lengths) != total:
        raise ValueError("Packed sample lengths must cover the token rows")


def _tokens(x, name):
    """Accept [1, L, H, D] (reference layout) or [L, H, D]; return a contiguous [L, H, D] view."""
    return _tokens_unchecked(x, name).contiguous()


def _token_rows_view(x, name):
    """[1, L, H, D] or [L, H, D] -> ([L, H, D] tensor, elements per token row) without a copy
    when the heads of a token are contiguous and the token rows start on 16-byte boundaries (a
    split view of a wider projection output, for instance); otherwise a contiguous copy."""
    x = _tokens_unchecked(x, name)
    L, H, D = x.shape
    if (x.dtype == torch.bfloat16 and x.stride(2) == 1 and x.stride(1) == D and L > 1 and x.stride(0) >= H * D
            and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0):
        return x, x.stride(0)
    x = x.contiguous()
    return x, H * D


def _tokens_unchecked(x, name):
    if x.dim() == 4:
        if x.shape[0] != 1:
            raise ValueError(f"{name}: packed inputs have batch size 1")
        x = x[0]
    if x.dim() != 3:
        raise ValueError(f"{name}: expected [1, L, H, D] or [L, H, D]")
    if not x.is_cuda:
        raise ValueError(f"{name}: expected a CUDA tensor")
    return x


def _gate(x, L, H, D, name, dtype=None):
    """Gate tensor in per-head [L,H] or per-channel [L,H,D] layout -> (tensor, layout)."""
    if x is None:
        return None, _lib.GATE_NONE
    if x.dim() == 4 and x.shape[0] == 1:
        x = x[0]
    if dtype is not None and x.dtype != dtype:
        raise ValueError(f"{name}: expected dtype {dtype}, got {x.dtype}")
    if not x.is_cuda:
        raise ValueError(f"{name}: expected a CUDA tensor")
    if x.dim() == 2 and tuple(x.shape) == (L, H):
        return x.contiguous(), _lib.GATE_PER_HEAD
    if x.dim() == 3 and tuple(x.shape) == (L, H, 1):
        return x.reshape(L, H).contiguous(), _lib.GATE_PER_HEAD
    if x.dim() == 3 and tuple(x.shape) == (L, H, D):
        return x.contiguous(), _lib.GATE_PER_CHANNEL
    raise ValueError(f"{name}: expected [L, H] or [L, H, {D}], got {tuple(x.shape)}")


def _states(x, N, H, K, V, device, name):
    if tuple(x.shape) != (N, H, K, V) or x.dtype != torch.float32 or x.device != device:
        raise ValueError(f"{name}: expected FP32 states {(N, H, K, V)} on {device}")
    return x.contiguous()


def _pool(states, slots, N, H, K, V, device, name):
    """states and slot arguments for the C ABI: with ``slots`` (int32 [N] on the device), states
    is a pool [S, H, K, V] and sample n uses states[slots[n]]; without, states is [N, H, K, V]."""
    if slots is None:
        return _states(states, N, H, K, V, device, name), None, 0
    if (states.dim() != 4 or tuple(states.shape[1:]) != (H, K, V) or states.dtype != torch.float32
            or states.device != device or not states.is_contiguous()):
        raise ValueError(f"{name}: expected a contiguous FP32 state pool [S, {H}, {K}, {V}] on {device}")
    if slots.dtype != torch.int32 or slots.device != device or tuple(slots.shape) != (N,):
        raise ValueError(f"{name}: slot indices must be int32 [{N}] on {device}")
    return states, slots.contiguous(), states.shape[0]


def gdn2_update(k, v, g, initial_state, cu_seqlens, *, num_samples, total_tokens, beta=None, erase=None,
                write=None, chunk_tokens=2048, final_state=None, initial_slots=None, final_slots=None):
    """GDN-2 write path over packed samples. Returns the final state [N, H, K, V] fp32.

    k, v: [L, H, D] bf16 (tensor-core path, reference GPU rounding) or fp32 (exact fp32
    recurrence). g: fp32 natural-log decay [L, H] or [L, H, K]. beta: sqrt(beta) is folded
    into k ([L, H] or [L, H, K]). erase: FLA channel-wise erase factor [L, H, K]. write:
    write gate [L, H, V]. cu_seqlens: int32 device [N+1]. final_state may alias
    initial_state (in-place update). initial_slots / final_slots (int32 [N] on the device):
    initial_state / final_state are then state pools and sample n starts from
    initial_state[initial_slots[n]] / ends in final_state[final_slots[n]] (returned: the pool).
    """
    lib, args, ws, out, _keep = _update_args(k, v, g, initial_state, cu_seqlens, num_samples, total_tokens, beta,
                                             erase, write, chunk_tokens, final_state, initial_slots, final_slots)
    _lib.check(lib.memt_gdn2_update(ctypes.byref(args), _ptr(ws), ws.numel(), _stream(out.device)), "memt_gdn2_update")
    return out


def _update_args(k, v, g, initial_state, cu_seqlens, num_samples, total_tokens, beta, erase, write, chunk_tokens,
                 final_state, initial_slots=None, final_slots=None):
    """Checked C arguments of an update (plus the tensors they point into)."""
    if _tokens_unchecked(k, "k").dtype == torch.bfloat16:  # bf16 rows are read in place
        k, k_stride = _token_rows_view(k, "k")
        v, v_stride = _token_rows_view(v, "v")
    else:
        k, v = _tokens(k, "k"), _tokens(v, "v")
        k_stride = v_stride = 0
    L, H, K = k.shape
    V = v.shape[-1]
    if v.shape[:2] != (L, H) or v.dtype != k.dtype:
        raise ValueError("k and v must share [L, H] and dtype")
    if k.dtype not in _DTYPE:
        raise ValueError(f"unsupported dtype {k.dtype}")
    if L != total_tokens:
        raise ValueError("total_tokens must equal the packed token count")
    dev = k.device
    if g.dtype != torch.float32:
        raise ValueError("log-decay must be float32")
    g, g_layout = _gate(g, L, H, K, "g")
    beta, beta_layout = _gate(beta, L, H, K, "beta", k.dtype)
    erase, erase_layout = _gate(erase, L, H, K, "erase", k.dtype)
    if erase_layout == _lib.GATE_PER_HEAD:
        raise ValueError("erase must be per channel [L, H, K]")
    w_stride = 0
    if write is not None:
        if k.dtype == torch.bfloat16:
            write, w_stride = _token_rows_view(write, "write")
        else:
            write = _tokens(write, "write")
        if tuple(write.shape) != (L, H, V) or write.dtype != k.dtype:
            raise ValueError("write gate must be [L, H, V] in the value dtype")
    N = int(num_samples)
    h0, in_slots, n_in = _pool(initial_state, initial_slots, N, H, K, V, dev, "initial_state")
    if final_state is None:
        if final_slots is not None:
            raise ValueError("final_slots index into final_state, which must then be given")
        out = torch.empty(N, H, K, V, device=dev, dtype=torch.float32)
    else:
        out = final_state
    if final_slots is None:
        _states(out, N, H, K, V, dev, "final_state")
    else:
        _pool(out, final_slots, N, H, K, V, dev, "final_state")
    if not out.is_contiguous():
        raise ValueError("final_state must be contiguous")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.device != dev or cu_seqlens.numel() != N + 1:
        raise ValueError("cu_seqlens must be int32 [N+1] on the input device")
    lib = _lib.load()
    dt = _DTYPE[k.dtype]
    need = lib.memt_gdn2_update_workspace_size(N, L, H, K, V, int(chunk_tokens), dt)
    if need == 0:
        raise ValueError("unsupported update sizes")
    ws = Workspace.get(dev, need)
    args = _lib.UpdateArgs(
        num_samples=N, num_heads=H, key_dim=K, value_dim=V, total_tokens=L, chunk_tokens=int(chunk_tokens),
        dtype=dt, cu_seqlens=cu_seqlens.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), g=g.data_ptr(),
        g_layout=g_layout, beta=beta.data_ptr() if beta is not None else None, beta_layout=beta_layout,
        erase=erase.data_ptr() if erase is not None else None, erase_layout=erase_layout,
        write=write.data_ptr() if write is not None else None,
        write_layout=_lib.GATE_PER_CHANNEL if write is not None else _lib.GATE_NONE,
        initial_state=h0.data_ptr(), final_state=out.data_ptr(),
        initial_slots=in_slots.data_ptr() if in_slots is not None else None, num_initial_slots=n_in,
        final_slots=final_slots.data_ptr() if final_slots is not None else None,
        num_final_slots=out.shape[0] if final_slots is not None else 0,
        k_stride=k_stride if k_stride != H * K else 0, v_stride=v_stride if v_stride != H * V else 0,
        write_stride=w_stride if w_stride != H * V else 0)
    return lib, args, ws, out, (k, v, g, beta, erase, write, h0, in_slots, final_slots)


def _read(q, states, cu, num_blocks, max_block_tokens, scale, out_dtype):
    lib, args, out, _keep = _read_args(q, states, cu, num_blocks, max_block_tokens, scale, out_dtype)
    _lib.check(lib.memt_gdn2_read(ctypes.byref(args), _stream(out.device)), "memt_gdn2_read")
    return out


def _read_args(q, states, cu, num_blocks, max_block_tokens, scale, out_dtype, slots=None):
    """Checked C arguments of a snapshot read (plus the tensors they point into)."""
    q = _tokens(q, "q")
    L, H, K = q.shape
    if q.dtype not in _DTYPE or out_dtype not in _DTYPE:
        raise ValueError("q and output must be bfloat16 or float32")
    states, slots, num_slots = _pool(states, slots, num_blocks, H, K, states.shape[-1], q.device, "states")
    V = states.shape[-1]
    out = torch.empty(L, H, V, device=q.device, dtype=out_dtype)
    lib = _lib.load()
    args = _lib.ReadArgs(
        num_blocks=num_blocks, num_heads=H, key_dim=K, value_dim=V, total_tokens=L,
        max_block_tokens=int(max_block_tokens), cu_seqlens=cu.data_ptr(), q=q.data_ptr(), q_dtype=_DTYPE[q.dtype],
        states=states.data_ptr(), scale=float(scale), out=out.data_ptr(), out_dtype=_DTYPE[out_dtype],
        state_slots=slots.data_ptr() if slots is not None else None, num_slots=num_slots)
    return lib, args, out, (q, states, slots)


def token_memory_packed(q, k, v, log_decay, write, read_states, write_states, *, erase=None, lengths, scale,
                        chunk_tokens, read_slots=None, write_slots=None, final_slots=None):
    """Write packed GDN-2 events and read each sample's fixed incoming snapshot.

    Returns (read [1, L, H, V] in v.dtype, final_state [N, H, K, V] fp32), like the
    reference. ``erase`` is the Qwen flavour's channel-wise erase factor; the DeepSeek
    flavour passes none. With ``read_slots`` (int32 [N] on the device) ``read_states`` is the
    state pool [S, H, K, V] and sample n reads read_states[read_slots[n]] in place. With
    ``write_slots`` ``write_states`` is a pool too: sample n starts from
    write_states[write_slots[n]] and its final state is written into write_states at
    ``final_slots`` (default: write_slots, an in-place update); the pool is returned as
    final_state.
    """
    L = _tokens_unchecked(q, "q").shape[0]
    _check_lengths(lengths, L)
    cu = _cu_seqlens(lengths, q.device)
    if write_slots is None and final_slots is not None:
        raise ValueError("final_slots needs write_slots (write_states is then the pool)")
    pool_out = write_states if write_slots is not None else None
    out_slots = (final_slots if final_slots is not None else write_slots) if write_slots is not None else None
    lib, uargs, ws, final, _keep_u = _update_args(k, v, log_decay, write_states, cu, len(lengths), L, None, erase,
                                                  write, chunk_tokens, pool_out, write_slots, out_slots)
    _, rargs, read, _keep_r = _read_args(q, read_states, cu, len(lengths), max(lengths), scale, v.dtype,
                                         slots=read_slots)
    # one call: the read of the incoming snapshot overlaps the update's state scan
    _lib.check(lib.memt_gdn2_update_read(ctypes.byref(uargs), _ptr(ws), ws.numel(), ctypes.byref(rargs),
                                         _stream(final.device)), "memt_gdn2_update_read")
    return read.unsqueeze(0), final


def memt_gdn2_read_fwd(q, snaps, plan: ChunkPlan, scale, out_dtype):
    """Read each token from its read-block snapshot (models/qwen/ops/read.py:10-39).

    ``plan`` is a plan of ``memt_b200.layout`` or the reference's own ``ChunkPlan``: each chunk
    reads the snapshot ``plan.chunk_block_ids`` names. A reference plan carries no read-block
    offsets, so its small chunk tables are copied to the host once per call to find them.
    """
    read_slice = getattr(plan, "read_slice", None)
    if read_slice is not None:
        out = _read(q, snaps, read_slice, plan.num_block, plan.max_block_tokens, scale, out_dtype)
        return out.unsqueeze(0)
    cu, ids, longest = read_segments(plan)
    dev = _tokens(q, "q").device
    cu_t = torch.tensor(cu, dtype=torch.int32).to(dev, non_blocking=True)
    ids_t = torch.tensor(ids, dtype=torch.int32).to(dev, non_blocking=True)
    lib, args, out, _keep = _read_args(q, snaps, cu_t, len(ids), max(longest, 1), scale, out_dtype, slots=ids_t)
    _lib.check(lib.memt_gdn2_read(ctypes.byref(args), _stream(out.device)), "memt_gdn2_read")
    return out.unsqueeze(0)


def snapshot_read(query, states, lengths, scale, *, bf16_accumulator_output=False):
    """DeepSeek snapshot read (models/deepseek/ops/read.py:6-31): output in the query dtype.

    Both accumulator modes accumulate in fp32 and round once to the query dtype; the
    reference's bf16 baddbmm path does the same up to accumulation order.
    """
    L = _tokens(query, "query").shape[0]
    _check_lengths(lengths, L)
    cu = _cu_seqlens(lengths, query.device)
    return _read(query, states, cu, len(lengths), max(lengths), scale, query.dtype).unsqueeze(0)


def memory_readout(q, states, lengths, scale, gate, norm_weight, *, eps=1e-6, softcap, residual=None,
                   out=None, head_offset=0, normalize_q=True, q_eps=1e-6, state_slots=None):
    """Fused decode/query readout over bf16 activations.

    y = MemTRMSNormGated(read(l2norm(q), states), gate) and out = residual + y, written into
    out[:, (head_offset + h) * D + v] (``residual`` may be ``out`` for an in-place add into
    the attention output). Returns out [L, row_stride]. With ``state_slots`` (int32 [N] on the
    device) ``states`` is the state pool [S, H, D, D] and sample n reads states[state_slots[n]]
    directly, without gathering the step's states into a new tensor first.
    """
    q = _tokens(q, "q")
    L, H, D = q.shape
    _check_lengths(lengths, L)
    if q.dtype != torch.bfloat16:
        raise ValueError("memory_readout expects bf16 activations")
    gate = _tokens(gate, "gate")
    if tuple(gate.shape) != (L, H, D) or gate.dtype != torch.bfloat16:
        raise ValueError("gate must be bf16 [L, H, D]")
    states, slots, num_slots = _pool(states, state_slots, len(lengths), H, D, D, q.device, "states")
    if tuple(norm_weight.shape) != (D,) or norm_weight.dtype != torch.bfloat16:
        raise ValueError("norm_weight must be bf16 [D]")
    norm_weight = norm_weight.contiguous()
    if out is None:
        out = torch.empty(L, (head_offset + H) * D, device=q.device, dtype=torch.bfloat16)
    if out.dim() != 2 or out.shape[0] != L or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 [L, row] tensor")
    if residual is not None and (residual.shape != out.shape or residual.dtype != torch.bfloat16
                                 or not residual.is_contiguous()):
        raise ValueError("residual must match out")
    cu = _cu_seqlens(lengths, q.device)
    lib = _lib.load()
    args = _lib.ReadoutArgs(
        num_blocks=len(lengths), num_heads=H, head_dim=D, total_tokens=L, max_block_tokens=max(lengths),
        cu_seqlens=cu.data_ptr(), q=q.data_ptr(), normalize_q=1 if normalize_q else 0, q_eps=float(q_eps),
        states=states.data_ptr(), scale=float(scale), gate=gate.data_ptr(), norm_weight=norm_weight.data_ptr(),
        norm_eps=float(eps), softcap=float(softcap),
        residual=residual.data_ptr() if residual is not None else None, out=out.data_ptr(),
        row_stride=out.shape[1], head_offset=int(head_offset),
        state_slots=slots.data_ptr() if slots is not None else None, num_slots=num_slots)
    _lib.check(lib.memt_memory_readout(ctypes.byref(args), _stream(q.device)), "memt_memory_readout")
    return out


def _token_rows(x, L, H, D, name):
    """A bf16 CUDA tensor of L token rows holding H heads of D contiguous values ([1, L, H, D],
    [L, H, D], [1, L, H*D] or [L, H*D], e.g. a split view of a projection output) ->
    (tensor, elements per token row)."""
    if x.dim() == 4 and x.shape[0] == 1:
        x = x[0]
    elif x.dim() == 3 and tuple(x.shape) != (L, H, D) and tuple(x.shape) == (1, L, H * D):
        x = x[0]
    if x.dim() == 3:
        if tuple(x.shape) != (L, H, D) or x.stride(2) != 1 or x.stride(1) != D:
            raise ValueError(f"{name}: expected [L, {H}, {D}] with contiguous heads")
    elif x.dim() == 2:
        if tuple(x.shape) != (L, H * D) or x.stride(1) != 1:
            raise ValueError(f"{name}: expected [L, {H * D}] rows")
    else:
        raise ValueError(f"{name}: expected token rows of {H} x {D} values")
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError(f"{name}: expected a bf16 CUDA tensor")
    return x, x.stride(0) if L > 1 else H * D


def qwen_prologue(q, k, erase_gate, write_gate, decay_latent, decay_bias, decay_scale_log, *, eps=1e-6,
                  rsqrt_norm=False):
    """The Qwen memory block's prologue in one kernel: (q_hat, k_scaled, write, log_decay).

    Replaces ``QwenMemoryBlock._write_gates`` / ``_log_decay`` / ``_symmetric_inputs``
    (models/qwen/layer.py:71-97) including their FLA Triton ``l2norm`` of q and k:
    q_hat = l2norm(q), k_scaled = bf16(sqrt(sigmoid(erase_gate)) * l2norm(k)),
    write = sigmoid(write_gate), log_decay = -exp(decay_scale_log) * softplus(decay_latent +
    decay_bias) (fp32). ``erase_gate`` and ``write_gate`` are the bf16 pre-activations the
    reference splits out of its gate projection and ``decay_latent`` is ``f_down`` of its
    decay rows; q, k and the gates may be the projections' split views. The erase factor the
    update needs afterwards is one, so call ``token_memory_packed`` with ``erase=None``.
    Outputs are [1, L, H, D] (bf16; log_decay fp32). ``rsqrt_norm`` selects the DeepSeek
    block's l2norm, x * rsqrt(sum x^2 + eps) (models/deepseek/ops/normalization.py:6-8).
    """
    q4 = q if q.dim() == 4 else q[None]
    if q4.dim() != 4:
        raise ValueError("q: expected [1, L, H, D] or [L, H, D]")
    _, L, H, D = q4.shape
    q2, sq = _token_rows(q, L, H, D, "q")
    k2, sk = _token_rows(k, L, H, D, "k")
    e2, se = _token_rows(erase_gate, L, H, D, "erase_gate")
    w2, sw = _token_rows(write_gate, L, H, D, "write_gate")
    d2, sd = _token_rows(decay_latent, L, H, D, "decay_latent")
    dev = q2.device
    if (decay_bias.numel() != H * D or decay_bias.dtype != torch.bfloat16 or decay_bias.device != dev
            or decay_scale_log.numel() != H or decay_scale_log.dtype != torch.bfloat16
            or decay_scale_log.device != dev):
        raise ValueError(f"decay_bias must be bf16 [{H * D}] and decay_scale_log bf16 [{H}] on {dev}")
    bias = decay_bias.contiguous()
    scale_log = decay_scale_log.contiguous()
    q_out = torch.empty(L, H, D, device=dev, dtype=torch.bfloat16)
    k_out = torch.empty_like(q_out)
    w_out = torch.empty_like(q_out)
    g_out = torch.empty(L, H, D, device=dev, dtype=torch.float32)
    lib = _lib.load()
    args = _lib.PrologueArgs(
        num_heads=H, head_dim=D, total_tokens=L, q=q2.data_ptr(), q_stride=sq, k=k2.data_ptr(), k_stride=sk,
        erase_latent=e2.data_ptr(), erase_stride=se, write_latent=w2.data_ptr(), write_stride=sw,
        decay_latent=d2.data_ptr(), decay_stride=sd, decay_bias=bias.data_ptr(),
        decay_scale_log=scale_log.data_ptr(), eps=float(eps), norm_kind=1 if rsqrt_norm else 0,
        q_out=q_out.data_ptr(), k_out=k_out.data_ptr(),
        write_out=w_out.data_ptr(), log_decay_out=g_out.data_ptr())
    _lib.check(lib.memt_qwen_prologue(ctypes.byref(args), _stream(dev)), "memt_qwen_prologue")
    return q_out[None], k_out[None], w_out[None], g_out[None]


def gdn2_chunked(q, k, v, g, beta, initial_state, cu_seqlens, *, w=None, scale=None, read_states=None,
                 chunk_tokens=2048, erase=None, max_seqlen=None):
    """(q, k, v, g, beta, initial_state, cu_seqlens) -> (o, final_state).

    q, k: L2-normalised [L, H, K]; beta enters as sqrt(beta) folded into k (stable GDN-2);
    w: optional write gate [L, H, V]; o reads the incoming snapshot (read_states, default
    initial_state) and is returned in v's dtype; final_state is fp32 [N, H, K, V].
    cu_seqlens may live on the host (validated there) or on the device; with device offsets
    pass ``max_seqlen`` (the longest sample) to avoid a device-to-host copy.
    """
    k3 = _tokens_unchecked(k, "k")
    L, H, K = k3.shape
    if cu_seqlens.is_cuda and max_seqlen is not None:
        N = cu_seqlens.numel() - 1
        max_len = int(max_seqlen)
        if N < 1 or max_len < 1:
            raise ValueError("cu_seqlens must hold at least two offsets and max_seqlen >= 1")
        cu = cu_seqlens if cu_seqlens.dtype == torch.int32 else cu_seqlens.to(torch.int32)
    else:
        cu_host = cu_seqlens.detach().to("cpu", torch.int64)
        N = cu_host.numel() - 1
        if N < 1 or int(cu_host[0]) != 0 or int(cu_host[-1]) != L or bool((cu_host[1:] < cu_host[:-1]).any()):
            raise ValueError("cu_seqlens must be nondecreasing offsets from 0 to L")
        max_len = int((cu_host[1:] - cu_host[:-1]).max())
        cu = cu_seqlens.to(device=k3.device, dtype=torch.int32).contiguous()
    scale = K ** -0.5 if scale is None else scale
    lib, uargs, ws, final, _keep_u = _update_args(k3, v, g, initial_state, cu, N, L, beta, erase, w, chunk_tokens,
                                                  None)
    rs = initial_state if read_states is None else read_states
    _, rargs, o, _keep_r = _read_args(q, rs, cu, N, max(max_len, 1), scale, _tokens(v, "v").dtype)
    # one call: the read overlaps the update's state scan (memt_gdn2_update_read)
    _lib.check(lib.memt_gdn2_update_read(ctypes.byref(uargs), _ptr(ws), ws.numel(), ctypes.byref(rargs),
                                         _stream(final.device)), "memt_gdn2_update_read")
    return o, final
