#!/usr/bin/env python
"""Benchmark of the B200 GDN-2 memory hot path (one JSON line on rank 0).

Headline workload ("Nano-shaped update"): per GPU, 8 sessions x 8192 tokens
packed via cu_seqlens, H=16 memory heads, d_k=d_v=128, bf16 q/k/v/beta and write gate, fp32
log-decay per head-token, fp32 state ~N(0, 0.02), chunk 64. One step = one memory layer's
commit: the chunked GDN-2 update (final state) plus the read of the incoming snapshot for
every token, through the BASELINE-style entry (q, k, v, g, beta, initial_state, cu_seqlens)
-> (o, final_state). Multi-GPU: one process per GPU, each rank owns its own 8 sessions
(sessions are independent; no collective on the data path), so per-GPU work is fixed
("weak" scaling) and value = all ranks' tokens / max-over-ranks time.

Also in the line (each object names its workload):
  config1_channel  the same commit shaped as the reference's Qwen block serves it: channel-wise
                   fp32 log-decay, the sqrt-erase factor folded into the key by the prologue
                   kernel (memt_qwen_prologue), write gate; plus the prologue itself in GB/s
  readout          BASELINE config 2 decode readout (256 sessions x 16 heads, fused
                   l2norm/read/gated RMSNorm/residual) in HBM GB/s
  gpu_bar          the reference's own Triton/PyTorch operators (installed in baseline/_ref)
                   timed on the same GPU at configs 1 and 2, with the distance of their outputs
                   from this library's
  head_sharded     BASELINE config 3 (32 varlen sessions, heads split over the ranks: fixed
                   global problem) and config 4 (16 heads of d=256 per GPU, the TP8 shard, with
                   the attention-output NCCL all-reduce timed beside it when N > 1)
  cpu_baseline     the fp32 PyTorch chunked restatement (oracle/gdn2_torch.py) of the update and
                   read on the host cores, and the reference's own PyTorch readout on CPU

--impl reference: the reference has no CPU implementation of its update; its fp32 CPU
restatement (oracle/gdn2_torch.py) runs the config-1 step on every host thread.
"""

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "memt-1.0_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)
REF_PATH = ROOT / "baseline" / "_ref"

SESSIONS, T, H, D = 8, 8192, 16, 128
CHUNK_TOKENS = 2048
METRIC = "GDN-2 update tokens/s (chunked update + snapshot read per memory layer)"
WORKLOAD = "config1: 8 sessions x 8192 tokens per GPU, H=16, d=128, bf16 inputs, fp32 state, chunk 64"
RO_SESSIONS, RO_LAYERS_RESIDENT = 256, 4  # decode readout, one layer per call


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def update_bytes_per_token_head(d, channel_gates, fused_read):
    """Algorithmic bytes of the update per token and head: k, v, write gate (bf16, 6d); g and beta
    (4 + 2 per head-token, or 4d channel-wise decay with the key already scaled); q and o of a
    fused read (4d)."""
    b = 6 * d + (4 * d if channel_gates else 4 + 2)
    return b + (4 * d if fused_read else 0)


def update_flops_per_token_head(d, c=64):
    """5 C d + 4 d^2: tril KK^T, w_wy, u, w_wy S and kg^T v_new (the O(C^2) solve excluded)."""
    return 5 * c * d + 4 * d * d


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    """SM clocks and clock-event reasons while the timed region runs: NVML read by a thread every
    2 ms (the timed region can be a few milliseconds), or nvidia-smi at 200 ms when NVML is not
    importable. Reads only; no setting of the GPU is changed."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.samples = []  # (sm MHz, max MHz, reason bits) from NVML
        self.nvml = None
        self.stop = threading.Event()
        self.thread = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(self.gpu_id)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _poll(self):
        nv = self.nvml
        while not self.stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM), self.max_mhz,
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)))
            except Exception:
                return
            time.sleep(0.002)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        if self.nvml is not None:
            for clk, top, bits in self.samples:
                sm.append(float(clk))
                mx = float(top)
                for name, attr in self.REASONS:
                    if bits & getattr(self.nvml, attr, 0):
                        reasons.add(name)
            n = len(self.samples)
        else:
            rows = [[c.strip() for c in ln.split(",")] for ln in self.lines if ln.count(",") >= 8]
            names = [r[0] for r in self.REASONS]
            for r in rows:
                try:
                    sm.append(float(r[1]))
                    mx = float(r[2])
                except ValueError:
                    continue
                for name, val in zip(names, r[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
            n = len(rows)
        loaded = [s for s in sm if mx and s > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": n, "source": "nvml" if self.nvml is not None else "nvidia-smi"}


def read_traffic(family):
    """Per-launch DRAM traffic of a kernel family from the committed ncu summaries."""
    pat = re.compile(rf"traffic_bytes_per_launch\[{family}\]\s*[:=]\s*([0-9.eE+]+)")
    for p in sorted((ROOT / "profiles").glob("*.md")):
        m = pat.search(p.read_text())
        if m:
            return float(m.group(1))
    return None


def algorithmic_bytes(family, L, Hh, N, D_):
    """Compulsory bytes of one launch of a kernel family for the headline workload (per-head
    decay and beta): what the family's inputs and outputs of the path must move, not the
    intermediates the library keeps in its workspace (those show in ``traffic``)."""
    th = L * Hh
    chunks_heads = math.ceil(T / 64) * N * Hh
    if family == "intra":  # the update's inputs: k, v, write (bf16) + g, beta per head-token
        return th * update_bytes_per_token_head(D_, False, False)
    if family == "scan":  # the states in and out
        return N * Hh * 8 * D_ * D_
    if family == "read_tile":  # q in, o out (bf16), snapshot in
        return th * 4 * D_ + N * Hh * 4 * D_ * D_
    if family == "plan":
        return (N + 1) * 4 + chunks_heads // Hh * 16
    return 0


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------

def time_steps(fn, steps, warmup, stream, flush=None):
    """Mean device milliseconds of fn() over `steps` calls, CUDA events on `stream`, L2 flushed
    before each timed call when `flush` is given."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush.zero_()
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / steps


def rel_fro(a, b):
    import torch

    a, b = a.double(), b.double()
    nb = torch.linalg.norm(b)
    return float(torch.linalg.norm(a - b) / (nb if nb > 0 else 1.0))


def config1_inputs(dev, gen, sessions, channel):
    import torch

    bf = torch.bfloat16
    L = sessions * T

    def nrm(x):
        return (x / torch.sqrt((x.float() ** 2).sum(-1, keepdim=True) + 1e-6)).to(bf)

    gshape = (L, H, D) if channel else (L, H)
    return dict(
        q=nrm(torch.randn(L, H, D, device=dev, generator=gen)),
        k=nrm(torch.randn(L, H, D, device=dev, generator=gen)),
        v=torch.randn(L, H, D, device=dev, generator=gen).to(bf),
        g=torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(*gshape, device=dev, generator=gen)),
        beta=torch.sigmoid(torch.randn(L, H, device=dev, generator=gen)).to(bf),
        w=torch.sigmoid(torch.randn(L, H, D, device=dev, generator=gen)).to(bf),
        h0=0.02 * torch.randn(sessions, H, D, D, device=dev, generator=gen),
        cu=torch.tensor([i * T for i in range(sessions + 1)], dtype=torch.int32, device=dev))


# ---------------------------------------------------------------------------
# legs
# ---------------------------------------------------------------------------

def leg_config1_channel(dev, gen, args, stream, flush, hbm):
    """The commit as the reference's Qwen block serves it: prologue (l2norm, sqrt-erase fold,
    write sigmoid, softplus decay) -> update + read with channel-wise decay and no erase."""
    import torch

    import memt_b200 as M

    bf = torch.bfloat16
    L = SESSIONS * T
    qkv = torch.randn(L, 3 * H * D, device=dev, generator=gen).to(bf)
    gates = torch.randn(L, 2 * H * D + D, device=dev, generator=gen).to(bf)
    q, k, v = (qkv[:, i * H * D:(i + 1) * H * D].view(L, H, D) for i in range(3))
    decay = (-2.0 + 0.5 * torch.randn(L, H * D, device=dev, generator=gen)).to(bf)
    bias = torch.zeros(H * D, device=dev, dtype=bf)
    scale_log = torch.zeros(H, device=dev, dtype=bf)
    h0 = 0.02 * torch.randn(SESSIONS, H, D, D, device=dev, generator=gen)
    lengths = [T] * SESSIONS

    def prologue():
        return M.qwen_prologue(q, k, gates[:, :H * D], gates[:, H * D:2 * H * D], decay, bias, scale_log)

    q_hat, k_s, w, g = prologue()

    def commit():
        return M.token_memory_packed(q_hat, k_s, v[None], g, w, h0, h0, erase=None, lengths=lengths,
                                     scale=D ** -0.5, chunk_tokens=CHUNK_TOKENS)

    ms = time_steps(commit, args.steps, args.warmup, stream, flush)
    ms_pro = time_steps(prologue, args.steps, args.warmup, stream, flush)
    b_th = update_bytes_per_token_head(D, True, True)
    step_bytes = L * H * b_th + SESSIONS * H * 12 * D * D
    pro_bytes = L * H * D * (5 * 2 + 3 * 2 + 4)  # q, k, erase, write, decay in; q, k, write, g out
    return {
        "workload": "config1 as the Qwen block commits: per-channel fp32 log-decay, sqrt-erase folded into "
                    "the key by the prologue, write gate, erase None; update + snapshot read",
        "ms_per_step": ms, "tokens_per_s": L / (ms * 1e-3),
        "step_roofline": {"bytes": step_bytes, "bytes_per_token_head": b_th, "gbs": step_bytes / (ms * 1e-3) / 1e9,
                          "frac": step_bytes / (ms * 1e-3) / 1e9 / hbm},
        "prologue": {"ms": ms_pro, "bytes": pro_bytes, "gbs": pro_bytes / (ms_pro * 1e-3) / 1e9,
                     "frac": pro_bytes / (ms_pro * 1e-3) / 1e9 / hbm},
    }


def leg_readout(dev, gen, stream, hbm):
    """Decode readout kernel throughput: the C entry point called with argument structs built
    once per resident layer, so the loop measures the device, not Python's per-call work
    (``python_api_us_per_layer`` is the same loop through memt_b200.memory_readout)."""
    import ctypes

    import torch

    import memt_b200 as M
    from memt_b200 import _lib, ops

    bf = torch.bfloat16
    states = torch.randn(RO_LAYERS_RESIDENT, RO_SESSIONS, H, D, D, device=dev, generator=gen) * 0.05
    q = torch.randn(RO_SESSIONS, H, D, device=dev, generator=gen).to(bf)
    gate = torch.randn(RO_SESSIONS, H, D, device=dev, generator=gen).to(bf)
    w = (1.0 + 0.1 * torch.randn(D, device=dev, generator=gen)).to(bf)
    attn = torch.randn(RO_SESSIONS, H * D, device=dev, generator=gen).to(bf)
    out = torch.empty_like(attn)
    lengths = [1] * RO_SESSIONS
    cu = torch.arange(RO_SESSIONS + 1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    args = [_lib.ReadoutArgs(
        num_blocks=RO_SESSIONS, num_heads=H, head_dim=D, total_tokens=RO_SESSIONS, max_block_tokens=1,
        cu_seqlens=cu.data_ptr(), q=q.data_ptr(), normalize_q=1, q_eps=1e-6, states=states[i].data_ptr(),
        scale=D ** -0.5, gate=gate.data_ptr(), norm_weight=w.data_ptr(), norm_eps=1e-6, softcap=10.0,
        residual=attn.data_ptr(), out=out.data_ptr(), row_stride=H * D, head_offset=0)
        for i in range(RO_LAYERS_RESIDENT)]
    sp = ops._stream(dev)
    it = [0]

    def step():
        st = lib.memt_memory_readout(ctypes.byref(args[it[0] % RO_LAYERS_RESIDENT]), sp)
        if st != 0:
            raise RuntimeError(f"memt_memory_readout: {st}")
        it[0] += 1

    def step_api():
        M.memory_readout(q, states[it[0] % RO_LAYERS_RESIDENT], lengths, D ** -0.5, gate, w, softcap=10.0,
                         residual=attn, out=out)
        it[0] += 1

    us = time_steps(step, 40, 8, stream) * 1e3  # the resident states cycle through 1 GB >> L2
    us_api = time_steps(step_api, 40, 8, stream) * 1e3
    nbytes = RO_SESSIONS * H * (4 * D * D + 4 * 2 * D) + 2 * D  # state + q, gate, attn in, out
    return {"workload": "config2: 256 sessions x 16 heads, fp32 128x128 state, 1 bf16 query each, fused "
                        "l2norm/read/gated RMSNorm/residual, one layer per call (4 layers' states cycled)",
            "us_per_layer": us, "gbs": nbytes / (us * 1e-6) / 1e9, "frac": nbytes / (us * 1e-6) / 1e9 / hbm,
            "bytes_per_layer": nbytes, "python_api_us_per_layer": us_api}


def leg_gpu_bar(dev, gen, args, stream, flush):
    """The reference's own operators on this GPU: Qwen token_memory_packed (Triton chunked update
    + Triton read) and DeepSeek token_memory_packed (Triton writer + bmm read) at config 1, and
    the Qwen decode readout (Triton read + MemTRMSNormGated + residual add) at config 2, next to
    this library's calls on the same inputs."""
    import torch

    import memt_b200 as M

    if not (REF_PATH / "memt_sglang").exists():
        return {"unavailable": "baseline/_ref holds no reference install"}
    if str(REF_PATH) not in sys.path:
        sys.path.append(str(REF_PATH))
    try:
        from memt_sglang.models.common.packed import boundaries
        from memt_sglang.models.deepseek.ops.packed import token_memory_packed as ds_packed
        from memt_sglang.models.qwen.layer import MemTRMSNormGated
        from memt_sglang.models.qwen.ops.layout import build_chunk_plan
        from memt_sglang.models.qwen.ops.packed import token_memory_packed as qw_packed
        from memt_sglang.models.qwen.ops.read import memt_gdn2_read_fwd
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference import failed: {type(e).__name__}: {e}"[:300]}
    bf = torch.bfloat16
    x = config1_inputs(dev, gen, SESSIONS, channel=True)
    L = SESSIONS * T
    lengths = [T] * SESSIONS
    q4, k4, v4, g4, w4 = (x[n][None] for n in ("q", "k", "v", "g", "w"))
    ones = torch.ones_like(k4)
    h0 = x["h0"]
    kw = dict(lengths=lengths, scale=D ** -0.5, chunk_tokens=CHUNK_TOKENS)
    out = {"workload": "config1 served shape (per-channel fp32 log-decay, write gate, Qwen erase = ones) and "
                       "config2 decode; reference Triton kernels autotuned, CUDA events, L2 flushed",
           "steps": args.steps}
    t0 = time.perf_counter()
    r_ref, s_ref = qw_packed(q4, k4, v4, g4, w4, h0, h0, erase=ones, **kw)  # compiles and autotunes
    r_ours, s_ours = M.token_memory_packed(q4, k4, v4, g4, w4, h0, h0, erase=ones, **kw)
    torch.cuda.synchronize()
    out["first_call_s"] = time.perf_counter() - t0
    out["qwen_commit"] = {
        "reference_ms": time_steps(lambda: qw_packed(q4, k4, v4, g4, w4, h0, h0, erase=ones, **kw), args.steps,
                                   2, stream, flush),
        "ours_ms": time_steps(lambda: M.token_memory_packed(q4, k4, v4, g4, w4, h0, h0, erase=ones, **kw),
                              args.steps, 2, stream, flush),
        "ours_erase_none_ms": time_steps(lambda: M.token_memory_packed(q4, k4, v4, g4, w4, h0, h0, erase=None, **kw),
                                         args.steps, 2, stream, flush),
        "state_rel_diff": rel_fro(s_ours, s_ref), "read_rel_diff": rel_fro(r_ours.float(), r_ref.float()),
    }
    c = out["qwen_commit"]
    c["speedup"] = c["reference_ms"] / c["ours_ms"]
    c["ref_tokens_per_s"] = L / (c["reference_ms"] * 1e-3)
    r_ref, s_ref = ds_packed(q4, k4, v4, g4, w4, h0, h0, **kw)
    r_ours, s_ours = M.token_memory_packed(q4, k4, v4, g4, w4, h0, h0, **kw)
    torch.cuda.synchronize()
    out["flash_commit"] = {
        "reference_ms": time_steps(lambda: ds_packed(q4, k4, v4, g4, w4, h0, h0, **kw), args.steps, 2, stream,
                                   flush),
        "ours_ms": time_steps(lambda: M.token_memory_packed(q4, k4, v4, g4, w4, h0, h0, **kw), args.steps, 2,
                              stream, flush),
        "state_rel_diff": rel_fro(s_ours, s_ref), "read_rel_diff": rel_fro(r_ours.float(), r_ref.float()),
    }
    c = out["flash_commit"]
    c["speedup"] = c["reference_ms"] / c["ours_ms"]
    del x, q4, k4, v4, g4, w4, ones
    # config 2 decode: the reference's query path (models/qwen/layer.py:112-131) after its l2norm
    states = torch.randn(RO_LAYERS_RESIDENT, RO_SESSIONS, H, D, D, device=dev, generator=gen) * 0.05
    qd = torch.randn(RO_SESSIONS, H, D, device=dev, generator=gen).to(bf)
    qd_hat = (qd.float() / torch.sqrt((qd.float() ** 2).sum(-1, keepdim=True) + 1e-6)).to(bf)
    gate = torch.randn(RO_SESSIONS, H, D, device=dev, generator=gen).to(bf)
    wn = (1.0 + 0.1 * torch.randn(D, device=dev, generator=gen)).to(bf)
    attn = torch.randn(RO_SESSIONS, H * D, device=dev, generator=gen).to(bf)
    norm = MemTRMSNormGated(D, eps=1e-6, output_gate_softcap_limit=10.0).to(dev)
    with torch.no_grad():
        norm.weight.copy_(wn.float())
    norm = norm.to(bf)
    samples = boundaries([1] * RO_SESSIONS, dev)
    plan = build_chunk_plan(samples, samples, 64, event_slice=samples,
                            commit_mask=torch.zeros(RO_SESSIONS, device=dev, dtype=torch.bool))
    it = [0]

    @torch.no_grad()
    def ref_decode():
        read = memt_gdn2_read_fwd(qd_hat[None], states[it[0] % RO_LAYERS_RESIDENT], plan, D ** -0.5, out_dtype=bf)
        y = norm(read.reshape(-1, D), gate.reshape(-1, D))
        it[0] += 1
        return attn + y.view(RO_SESSIONS, H * D)

    ours_out = torch.empty_like(attn)

    def our_decode():
        M.memory_readout(qd, states[it[0] % RO_LAYERS_RESIDENT], [1] * RO_SESSIONS, D ** -0.5, gate, wn,
                         softcap=10.0, residual=attn, out=ours_out)
        it[0] += 1
        return ours_out

    ref_y = ref_decode()
    it[0] = 0
    our_y = our_decode().clone()  # later calls overwrite the output buffer
    torch.cuda.synchronize()
    it[0] = 0
    out["qwen_decode_readout"] = {
        "reference_us": time_steps(ref_decode, 40, 8, stream) * 1e3,
        "ours_us": time_steps(our_decode, 40, 8, stream) * 1e3,
        "out_rel_diff": rel_fro(our_y.float(), ref_y.float()),
        "note": "reference: Triton read + eager MemTRMSNormGated + residual add on an l2-normalised query; "
                "ours: one fused kernel including the l2norm",
    }
    d = out["qwen_decode_readout"]
    d["speedup"] = d["reference_us"] / d["ours_us"]
    return out


def leg_head_sharded(dev, gen, args, stream, flush, rank, world, pg, hbm, only_config4=False):
    """Config 3 with heads split over the ranks (fixed global problem) and the per-GPU config-4
    shard (16 of 128 heads at d=256) with the attention-output all-reduce at N > 1."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import memt_b200 as M
    from memt_b200 import shard

    bf = torch.bfloat16
    res = {}
    # ---- config 3: 32 sessions, lengths U[1K, 32K] (seeded), H=16, d=128, heads split ----
    lengths = np.random.default_rng(3).integers(1024, 32768, 32).tolist()
    L = int(sum(lengths))
    h0_, h1_ = shard.head_range(rank, world, H)
    Hr = h1_ - h0_

    def nrm(t):
        return (t / torch.sqrt((t.float() ** 2).sum(-1, keepdim=True) + 1e-6)).to(bf)

    q = nrm(torch.randn(L, Hr, D, device=dev, generator=gen))
    k = nrm(torch.randn(L, Hr, D, device=dev, generator=gen))
    v = torch.randn(L, Hr, D, device=dev, generator=gen).to(bf)
    g = torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L, Hr, device=dev, generator=gen))
    beta = torch.sigmoid(torch.randn(L, Hr, device=dev, generator=gen)).to(bf)
    w = torch.sigmoid(torch.randn(L, Hr, D, device=dev, generator=gen)).to(bf)
    h0 = 0.02 * torch.randn(32, Hr, D, D, device=dev, generator=gen)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
    mx = int(max(lengths))

    def c3():
        return M.gdn2_chunked(q, k, v, g, beta, h0, cu, w=w, max_seqlen=mx, chunk_tokens=CHUNK_TOKENS)

    if pg:
        dist.barrier()
    ms3 = 0.0 if only_config4 else time_steps(c3, max(3, args.steps // 2), args.warmup, stream, flush)
    del q, k, v, g, beta, w, h0
    # ---- config 4 shard: 4 x 16384 tokens, 16 heads of d=256 (this rank's TP8 slice) ----
    D4, H4, N4, T4 = 256, 16, 4, 16384
    L4 = N4 * T4
    q = nrm(torch.randn(L4, H4, D4, device=dev, generator=gen))
    k = nrm(torch.randn(L4, H4, D4, device=dev, generator=gen))
    v = torch.randn(L4, H4, D4, device=dev, generator=gen).to(bf)
    g = torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L4, H4, D4, device=dev, generator=gen))
    w = torch.sigmoid(torch.randn(L4, H4, D4, device=dev, generator=gen)).to(bf)
    h0 = 0.02 * torch.randn(N4, H4, D4, D4, device=dev, generator=gen)

    def c4():
        return M.token_memory_packed(q[None], k[None], v[None], g[None], w[None], h0, h0, lengths=[T4] * N4,
                                     scale=D4 ** -0.5, chunk_tokens=CHUNK_TOKENS)

    ms4 = time_steps(c4, max(3, args.steps // 2), args.warmup, stream, flush)
    del q, k, v, g, w, h0
    ar_ms = None
    if pg:
        # the attention o_proj all-reduce of config 4 ([65536, 4096] bf16, 512 MiB), alone
        buf = torch.randn(65536, 4096, device=dev, generator=gen).to(bf)
        ar_ms = time_steps(lambda: dist.all_reduce(buf), 5, 3, stream)
        del buf
    vals = torch.tensor([ms3, ms4, ar_ms or 0.0], dtype=torch.float64, device=dev)
    if pg:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms3, ms4, ar_ms_max = [float(t) for t in vals.tolist()]
    if only_config4:
        ms3 = float("nan")
    b3 = L * H * update_bytes_per_token_head(D, False, True) + 32 * H * 12 * D * D
    res["config3"] = {
        "workload": f"config3: 32 sessions, lengths U[1K,32K] seed 3 ({L} tokens), H=16 split over {world} "
                    f"rank(s) ({Hr} heads each), d=128, per-head decay; update + read",
        "scaling": "strong", "ms_per_step": ms3, "tokens_per_s": L / (ms3 * 1e-3),
        "gbs_all_ranks": b3 / (ms3 * 1e-3) / 1e9, "frac_per_gpu": b3 / world / (ms3 * 1e-3) / 1e9 / hbm,
        "longest_session": mx}
    f4 = L4 * H4 * update_flops_per_token_head(D4)
    b4 = L4 * H4 * update_bytes_per_token_head(D4, True, True) + N4 * H4 * 12 * D4 * D4
    res["config4_shard"] = {
        "workload": "config4 per-GPU shard: 4 x 16384 tokens, 16 heads (TP8 slice of 128), d=256, per-channel "
                    "decay, write gate, no erase; update + read (every rank its own 16-head slice)",
        "ms_per_step": ms4, "tokens_per_s_per_gpu": L4 / (ms4 * 1e-3),
        "tflops_per_gpu": f4 / (ms4 * 1e-3) / 1e12, "gbs_per_gpu": b4 / (ms4 * 1e-3) / 1e9,
        "hbm_frac": b4 / (ms4 * 1e-3) / 1e9 / hbm}
    if pg:
        nbytes = 65536 * 4096 * 2
        res["config4_allreduce"] = {"bytes": nbytes, "ms": ar_ms_max,
                                    "bus_gbs": nbytes * 2 * (world - 1) / world / (ar_ms_max * 1e-3) / 1e9,
                                    "ranks": world, "collective": "torch.distributed.all_reduce (NCCL)"}
    return res


def leg_cpu_baseline(hbm):
    """fp32 PyTorch chunked restatement on the host cores (config-1 step) and the reference's own
    PyTorch readout on CPU (config 2, one layer)."""
    import torch

    from oracle import gdn2_torch as OT

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    x = cpu_inputs(SESSIONS)
    cu = [i * T for i in range(SESSIONS + 1)]
    cpu_step(x, cu)  # first touch of the work buffers
    t0 = time.perf_counter()
    reps = 2
    for _ in range(reps):
        cpu_step(x, cu)
    t = (time.perf_counter() - t0) / reps
    out = {"value": SESSIONS * T / t, "unit": "tokens/s", "cores": cores, "kind": "port",
           "sample": f"the full config-1 step ({SESSIONS} x {T} tokens, H={H}, d={D}): oracle/gdn2_torch.py fp32 "
                     f"chunked update + read, torch.set_num_threads({cores}); mean of {reps} steps after one warm-up",
           "ms_per_step": t * 1e3}
    del x
    # reference readout on CPU: snapshot_read + MemTRMSNormGated in fp32, config 2 (one layer)
    gen = torch.Generator().manual_seed(2)
    S = torch.randn(RO_SESSIONS, H, D, D, generator=gen) * 0.05
    q = torch.randn(1, RO_SESSIONS, H, D, generator=gen)
    q = q / torch.sqrt((q * q).sum(-1, keepdim=True) + 1e-6)
    gate = torch.randn(RO_SESSIONS * H, D, generator=gen)
    kind = "reference"
    try:
        if str(REF_PATH) not in sys.path:
            sys.path.append(str(REF_PATH))
        from memt_sglang.models.deepseek.ops.read import snapshot_read
        from memt_sglang.models.qwen.layer import MemTRMSNormGated
        norm = MemTRMSNormGated(D, eps=1e-6, output_gate_softcap_limit=10.0)

        @torch.no_grad()
        def ro():
            r = snapshot_read(q, S, [1] * RO_SESSIONS, D ** -0.5)
            return norm(r.reshape(-1, D), gate)
    except Exception:  # noqa: BLE001
        kind = "port"

        @torch.no_grad()
        def ro():
            return OT.read(q[0], S, list(range(RO_SESSIONS + 1)), D ** -0.5)
    ro()
    t0 = time.perf_counter()
    for _ in range(5):
        ro()
    t = (time.perf_counter() - t0) / 5
    nbytes = RO_SESSIONS * H * (4 * D * D + 4 * 2 * D)
    out["readout"] = {"kind": kind, "cores": cores, "us_per_layer": t * 1e6, "gbs": nbytes / t / 1e9,
                      "sample": "config 2, one layer, fp32: the reference's snapshot_read + MemTRMSNormGated"
                      if kind == "reference" else "config 2, one layer, fp32 read (oracle/gdn2_torch.py)"}
    return out


def cpu_inputs(sessions):
    import torch

    gen = torch.Generator().manual_seed(0)
    L = sessions * T
    nrm = torch.nn.functional.normalize
    k = nrm(torch.randn(L, H, D, generator=gen), dim=-1) * torch.sqrt(torch.sigmoid(torch.randn(L, H, 1, generator=gen)))
    return dict(
        q=nrm(torch.randn(L, H, D, generator=gen), dim=-1), k=k, v=torch.randn(L, H, D, generator=gen),
        g=torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L, H, generator=gen)),
        w=torch.sigmoid(torch.randn(L, H, D, generator=gen)), h0=0.02 * torch.randn(sessions, H, D, D, generator=gen))


def cpu_step(x, cu):
    from oracle import gdn2_torch as OT

    final = OT.chunked_update(x["k"], x["v"], x["g"], x["h0"], cu, w=x["w"], chunk_tokens=CHUNK_TOKENS)
    o = OT.read(x["q"], x["h0"], cu, D ** -0.5)
    return o, final


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import memt_b200 as M
    from memt_b200 import _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        pg = True

    hbm, tflops, peak_kind = peaks()
    sessions = args.sessions
    only_update = args.only == "update"
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    L = sessions * T
    x = config1_inputs(dev, gen, sessions, channel=args.gate == "channel")
    q, k, v, g, beta, w, h0, cu = (x[n] for n in ("q", "k", "v", "g", "beta", "w", "h0", "cu"))
    flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=dev)  # > 126 MB L2

    def step():
        return M.gdn2_chunked(q, k, v, g, beta, h0, cu, w=w, max_seqlen=T, chunk_tokens=CHUNK_TOKENS)

    def barrier():
        if pg:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps, L2 flushed between steps, CUDA events on the launch stream ----
    stream = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    gpu_uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(gpu_uuid) as clocks:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    # per-kernel device times from the library's event profiler, in a separate pass of the same
    # steps (its events between launches are kept out of the timed region above)
    _lib.profiler_reset()
    _lib.profiler_enable(True)
    for i in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    _lib.profiler_enable(False)
    prof = _lib.profiler_read()
    _lib.profiler_reset()
    launches = sum(n for _, n in prof.values())

    e2e_ms = float("nan")
    bytes_in = bytes_out = 0
    extra = {}
    if not only_update:
        # ---- end to end through the public API: pinned host inputs -> device -> result -> host ----
        host_in = {name: t.cpu().pin_memory() for name, t in dict(q=q, k=k, v=v, g=g, beta=beta, w=w, h0=h0).items()}
        # two device input sets and two host output sets: step i's inputs go up on the H2D
        # stream while step i - 1 computes and step i - 2's results come down on the D2H stream
        # (PCIe is full duplex), as a serving loop would run it
        dev_in = [{name: torch.empty_like(t, device=dev) for name, t in host_in.items()} for _ in range(2)]
        host_out = [(torch.empty(L, H, D, dtype=torch.bfloat16, pin_memory=True),
                     torch.empty(sessions, H, D, D, dtype=torch.float32, pin_memory=True)) for _ in range(2)]
        bytes_in = sum(t.numel() * t.element_size() for t in host_in.values())
        bytes_out = host_out[0][0].numel() * 2 + host_out[0][1].numel() * 4
        h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        inputs_ready = [torch.cuda.Event() for _ in range(2)]
        inputs_free = [torch.cuda.Event() for _ in range(2)]
        outputs_ready = [torch.cuda.Event() for _ in range(2)]
        outputs_free = [torch.cuda.Event() for _ in range(2)]
        for ev in inputs_free + outputs_free:
            ev.record(stream)

        def e2e_step(i):
            b = i % 2
            with torch.cuda.stream(h2d):
                h2d.wait_event(inputs_free[b])          # step i - 2 has consumed this input set
                for name, t in host_in.items():
                    dev_in[b][name].copy_(t, non_blocking=True)
                inputs_ready[b].record(h2d)
            stream.wait_event(inputs_ready[b])
            stream.wait_event(outputs_free[b])          # step i - 2's results have left the device
            xi = dev_in[b]
            o, s = M.gdn2_chunked(xi["q"], xi["k"], xi["v"], xi["g"], xi["beta"], xi["h0"], cu, w=xi["w"],
                                  max_seqlen=T, chunk_tokens=CHUNK_TOKENS)
            inputs_free[b].record(stream)
            outputs_ready[b].record(stream)
            with torch.cuda.stream(d2h):
                d2h.wait_event(outputs_ready[b])
                host_out[b][0].copy_(o, non_blocking=True)
                host_out[b][1].copy_(s, non_blocking=True)
                o.record_stream(d2h)
                s.record_stream(d2h)
                outputs_free[b].record(d2h)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        started = torch.cuda.Event()
        started.record(stream)
        h2d.wait_event(started)         # no copy of the timed steps starts before e0
        for i in range(args.steps):
            e2e_step(i)
        stream.wait_stream(d2h)         # the last results are on the host
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        barrier()
        del host_in, dev_in, host_out
        extra["config1_channel"] = leg_config1_channel(dev, gen, args, stream, flush, hbm)
        extra["readout"] = leg_readout(dev, gen, stream, hbm)
        if not args.skip_head_sharded:
            extra["head_sharded"] = leg_head_sharded(dev, gen, args, stream, flush, rank, world, pg, hbm)

    # ---- max over ranks ----
    ch = extra.get("config1_channel", {})
    ro = extra.get("readout", {})
    vals = torch.tensor([ms, e2e_ms, ch.get("ms_per_step", 0.0), ro.get("us_per_layer", 0.0)], dtype=torch.float64,
                        device=dev)
    if pg:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms, ch_ms, ro_us = [float(t) for t in vals.tolist()]

    if rank == 0:
        if world == 1 and not only_update and not args.skip_gpu_bar:
            try:
                extra["gpu_bar"] = leg_gpu_bar(dev, gen, args, stream, flush)
            except Exception as e:  # noqa: BLE001
                extra["gpu_bar"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
        cpu = None
        if world == 1 and not args.skip_cpu_baseline and not only_update:
            cpu = leg_cpu_baseline(hbm)
        tokens = L * world
        fam, (fam_ms, fam_n) = max(((f, v_) for f, v_ in prof.items() if v_[1] > 0), key=lambda kv: kv[1][0])
        per_launch_ms = fam_ms / fam_n
        alg = algorithmic_bytes(fam, L, H, sessions, D)
        achieved = alg / (per_launch_ms * 1e-3) / 1e9
        b_th = update_bytes_per_token_head(D, False, True)
        step_alg = L * H * b_th + sessions * H * 12 * D * D
        step_flops = L * H * (update_flops_per_token_head(D) + 2 * D * D)
        out = {
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sessions_per_gpu": sessions, "tokens_per_session": T,
                       "heads": H, "head_dim": D, "chunk_tokens": CHUNK_TOKENS,
                       "parallelism": f"dp{world} (sessions sharded, no collective)",
                       "l2": "flushed (256 MiB write) between timed steps"},
            "step_roofline": {"bytes": step_alg, "bytes_per_token_head": b_th,
                              "gbs": step_alg / (ms * 1e-3) / 1e9, "frac": step_alg / (ms * 1e-3) / 1e9 / hbm,
                              "flops": step_flops, "tflops": step_flops / (ms * 1e-3) / 1e12,
                              "tensor_frac": step_flops / (ms * 1e-3) / 1e12 / tflops, "peak_kind": peak_kind},
            "roofline": {"bound": "hbm", "kernel": fam, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": read_traffic(fam), "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": alg, "launch_ms": per_launch_ms},
            "kernels": {f: {"ms_per_step": v_[0] / args.steps, "launches": v_[1]} for f, v_ in prof.items() if v_[1]},
            "e2e": None if only_update else {
                "value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": bytes_in,
                "d2h_bytes_per_step": bytes_out, "ms_per_step": e2e_ms,
                "h2d_gbs": bytes_in / (e2e_ms * 1e-3) / 1e9, "d2h_gbs": bytes_out / (e2e_ms * 1e-3) / 1e9,
                "note": "bound by PCIe: the step's inputs cross the host link every step"},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        if ch:
            ch["ms_per_step"] = ch_ms
            ch["tokens_per_s"] = tokens / (ch_ms * 1e-3)
        if ro:
            ro["us_per_layer"] = ro_us
        out.update(extra)
        print(json.dumps(out), flush=True)
    if pg:
        dist.barrier()
        dist.destroy_process_group()


def run_leg(args):
    """One leg alone on cuda:0 (profiling cases): the Qwen prologue of config 1 (--sessions sets the
    size) or the config-2 decode readout."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(1234)
    hbm, _, _ = peaks()
    stream = torch.cuda.current_stream(dev)
    if args.only == "readout":
        print(json.dumps(leg_readout(dev, gen, stream, hbm)), flush=True)
        return
    if args.only == "config4":
        flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=dev)
        res = leg_head_sharded(dev, gen, args, stream, flush, 0, 1, None, hbm, only_config4=True)
        print(json.dumps(res), flush=True)
        return
    import memt_b200 as M

    bf = torch.bfloat16
    L = args.sessions * T
    qkv = torch.randn(L, 3 * H * D, device=dev, generator=gen).to(bf)
    gates = torch.randn(L, 2 * H * D + D, device=dev, generator=gen).to(bf)
    decay = (-2.0 + 0.5 * torch.randn(L, H * D, device=dev, generator=gen)).to(bf)
    bias, scale_log = torch.zeros(H * D, device=dev, dtype=bf), torch.zeros(H, device=dev, dtype=bf)
    q, k = qkv[:, :H * D].view(L, H, D), qkv[:, H * D:2 * H * D].view(L, H, D)

    def prologue():
        return M.qwen_prologue(q, k, gates[:, :H * D], gates[:, H * D:2 * H * D], decay, bias, scale_log)

    ms = time_steps(prologue, args.steps, args.warmup, stream)
    nbytes = L * H * D * (5 * 2 + 3 * 2 + 4)
    print(json.dumps({"leg": "prologue", "tokens": L, "ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9,
                      "frac": nbytes / (ms * 1e-3) / 1e9 / hbm}), flush=True)


def run_reference(args, rank, world):
    """The reference has no CPU implementation of its update (Triton only); its fp32 CPU
    restatement in the reference kernel order runs the config-1 step on every host thread."""
    if rank != 0:
        return
    import torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    x = cpu_inputs(SESSIONS)
    cu = [i * T for i in range(SESSIONS + 1)]
    for _ in range(max(1, min(args.warmup, 2))):
        cpu_step(x, cu)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(x, cu)
    total = time.perf_counter() - t0
    value = SESSIONS * T * args.steps / total
    sample = (f"every step the full config-1 step ({SESSIONS} x {T} tokens, H={H}, d={D}): oracle/gdn2_torch.py "
              f"fp32 chunked update + snapshot read (CPU restatement of the reference algorithm), "
              f"torch.set_num_threads({cores})")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": "host cores", "same_config": True},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--skip-gpu-bar", action="store_true")
    ap.add_argument("--skip-head-sharded", action="store_true")
    ap.add_argument("--sessions", type=int, default=SESSIONS, help="sessions per GPU (profiling cases)")
    ap.add_argument("--gate", choices=["head", "channel"], default="head",
                    help="log-decay layout of the headline step (channel: profiling the per-channel path)")
    ap.add_argument("--only", choices=["all", "update", "prologue", "readout", "config4"], default="all",
                    help="update: time only the commit step (no e2e, other legs, CPU baseline); "
                         "prologue / readout / config4: only that leg (profiling cases)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.only in ("prologue", "readout", "config4"):
        run_leg(args)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
