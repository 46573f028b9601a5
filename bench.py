#!/usr/bin/env python
"""Benchmark of the B200 GDN-2 memory hot path (one JSON line on rank 0).

Workload ("Nano-shaped update"): per GPU, 8 sessions x 8192 tokens packed
via cu_seqlens, H=16 memory heads, d_k=d_v=128, bf16 q/k/v/beta and write gate, fp32
log-decay per head-token, fp32 state ~N(0, 0.02), chunk 64. One step = one memory layer's
commit: the chunked GDN-2 update (final state) plus the read of the incoming snapshot for
every token, through the BASELINE-style entry (q, k, v, g, beta, initial_state, cu_seqlens)
-> (o, final_state). Multi-GPU: one process per GPU, each rank owns its own 8 sessions
(sessions are independent; no collective on the data path), so per-GPU work is fixed
("weak" scaling) and value = all ranks' tokens / max-over-ranks time.

Also reported: the decode readout of BASELINE config 2 (256 sessions x 16 heads, fp32
128x128 state, one bf16 query each, fused l2norm/read/gated RMSNorm/residual) in HBM GB/s.

--impl reference: the CPU restatement of the reference algorithm (oracle/gdn2.py, the
reference has no CPU implementation of this path) timed on the host cores.
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

SESSIONS, T, H, D = 8, 8192, 16, 128
CHUNK_TOKENS = 2048
METRIC = "GDN-2 update tokens/s (chunked update + snapshot read per memory layer)"
WORKLOAD = "config1: 8 sessions x 8192 tokens per GPU, H=16, d=128, bf16 inputs, fp32 state, chunk 64"
# decode readout, one memory layer per call
RO_SESSIONS, RO_LAYERS_RESIDENT = 256, 4
CPU_SAMPLE_TOKENS = 4096


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# CPU baseline: the oracle, parallel over heads in a spawn pool
# ---------------------------------------------------------------------------

def _cpu_head(args):
    seed, tokens, head = args
    import numpy as np

    from oracle import gdn2 as O

    rng = np.random.default_rng(seed * 131 + head)
    q = rng.standard_normal((tokens, 1, D))
    k = rng.standard_normal((tokens, 1, D))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    beta = 1 / (1 + np.exp(-rng.standard_normal((tokens, 1, 1))))
    k = np.sqrt(beta) * k
    v = rng.standard_normal((tokens, 1, D))
    g = np.broadcast_to(-np.logaddexp(0.0, -rng.normal(2.0, 0.5, (tokens, 1, 1))), (tokens, 1, D))
    w = 1 / (1 + np.exp(-rng.standard_normal((tokens, 1, D))))
    h0 = 0.02 * rng.standard_normal((1, 1, D, D))
    O.chunked(q, k, v, g, h0, h0, [0, tokens], D ** -0.5, w=w, chunk_tokens=CHUNK_TOKENS, mode="exact")
    return head


def cpu_pool():
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    return mp.get_context("spawn").Pool(min(cores, H)), min(cores, H)


def cpu_measure(pool, tokens, seed=0):
    t0 = time.perf_counter()
    pool.map(_cpu_head, [(seed, tokens, h) for h in range(H)])
    return time.perf_counter() - t0


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples (200 ms) while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = [[c.strip() for c in ln.split(",")] for ln in self.lines if ln.count(",") >= 8]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        loaded = [s for s in sm if mx and s > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(rows)}


def read_traffic(family):
    """Per-launch DRAM traffic of a kernel family from the committed ncu summaries."""
    pat = re.compile(rf"traffic_bytes_per_launch\[{family}\]\s*[:=]\s*([0-9.eE+]+)")
    for p in sorted((ROOT / "profiles").glob("*.md")):
        m = pat.search(p.read_text())
        if m:
            return float(m.group(1))
    return None


def algorithmic_bytes(family, L, Hh, N, D_):
    """Compulsory bytes one launch of a kernel family moves for the bench workload."""
    th = L * Hh
    chunks_heads = math.ceil(T / 64) * N * Hh
    if family == "intra":  # k, v, w (bf16) + g, beta per head-token in; w, u, kg (bf16) + 2^G_last out
        return th * (3 * 2 * D_ + 4 + 2) + chunks_heads * (3 * 64 * 2 * D_ + 4 * D_)
    if family == "scan":  # w, u, kg + 2^G_last in; state in + out
        return chunks_heads * (3 * 64 * 2 * D_ + 4 * D_) + N * Hh * 8 * D_ * D_
    if family == "read_tile":  # q in, o out (bf16), snapshot in
        return th * 4 * D_ + N * Hh * 4 * D_ * D_
    if family == "plan":
        return (N + 1) * 4 + chunks_heads // Hh * 16
    return 0


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import memt_b200 as M
    from memt_b200 import _lib, ops

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
        pg = True

    # CPU-baseline pool is created before any GPU work (spawn).
    pool, cores = (None, 0)
    if rank == 0 and world == 1 and not args.skip_cpu_baseline and args.only == "all":
        pool, cores = cpu_pool()

    hbm, tflops, peak_kind = peaks()
    SESSIONS = args.sessions
    only_update = args.only == "update"
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    bf = torch.bfloat16
    L = SESSIONS * T

    def nrm(x):
        return (x / torch.sqrt((x.float() ** 2).sum(-1, keepdim=True) + 1e-6)).to(bf)

    q = nrm(torch.randn(L, H, D, device=dev, generator=gen))
    k = nrm(torch.randn(L, H, D, device=dev, generator=gen))
    v = torch.randn(L, H, D, device=dev, generator=gen).to(bf)
    g = torch.nn.functional.logsigmoid(2.0 + 0.5 * torch.randn(L, H, device=dev, generator=gen))
    beta = torch.sigmoid(torch.randn(L, H, device=dev, generator=gen)).to(bf)
    w = torch.sigmoid(torch.randn(L, H, D, device=dev, generator=gen)).to(bf)
    h0 = 0.02 * torch.randn(SESSIONS, H, D, D, device=dev, generator=gen)
    cu = torch.tensor([i * T for i in range(SESSIONS + 1)], dtype=torch.int32, device=dev)
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

    e2e_ms = ro_us = ro_gbs = float("nan")
    bytes_in = bytes_out = 0
    if not only_update:
        # ---- end to end through the public API: pinned host inputs -> device -> result -> host ----
        host_in = {name: t.cpu().pin_memory() for name, t in
                   dict(q=q, k=k, v=v, g=g, beta=beta, w=w, h0=h0).items()}
        # two device input sets and two host output sets: step i's inputs go up on the H2D
        # stream while step i - 1 computes and step i - 2's results come down on the D2H stream
        # (PCIe is full duplex), as a serving loop would run it
        dev_in = [{name: torch.empty_like(t, device=dev) for name, t in host_in.items()} for _ in range(2)]
        host_out = [(torch.empty(L, H, D, dtype=bf, pin_memory=True),
                     torch.empty(SESSIONS, H, D, D, dtype=torch.float32, pin_memory=True)) for _ in range(2)]
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
            x = dev_in[b]
            o, s = M.gdn2_chunked(x["q"], x["k"], x["v"], x["g"], x["beta"], x["h0"],
                                  cu, w=x["w"], max_seqlen=T, chunk_tokens=CHUNK_TOKENS)
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

        # ---- decode readout, one layer per call, state >> L2 ----
        ro_states = torch.randn(RO_LAYERS_RESIDENT, RO_SESSIONS, H, D, D, device=dev, generator=gen) * 0.05
        ro_q = torch.randn(RO_SESSIONS, H, D, device=dev, generator=gen).to(bf)
        ro_gate = torch.randn(RO_SESSIONS, H, D, device=dev, generator=gen).to(bf)
        ro_w = (1.0 + 0.1 * torch.randn(D, device=dev, generator=gen)).to(bf)
        ro_attn = torch.randn(RO_SESSIONS, H * D, device=dev, generator=gen).to(bf)
        ro_out = torch.empty_like(ro_attn)
        lengths = [1] * RO_SESSIONS

        def ro_step(i):
            M.memory_readout(ro_q, ro_states[i % RO_LAYERS_RESIDENT], lengths, D ** -0.5, ro_gate, ro_w,
                             softcap=10.0, residual=ro_attn, out=ro_out)

        for i in range(8):
            ro_step(i)
        torch.cuda.synchronize()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ro_iters = 40
        r0.record(stream)
        for i in range(ro_iters):
            ro_step(i)
        r1.record(stream)
        torch.cuda.synchronize()
        ro_us = r0.elapsed_time(r1) * 1e3 / ro_iters
        ro_bytes = RO_SESSIONS * H * (4 * D * D + 4 * 2 * D) + 2 * D  # state + q, gate, attn in, out
        ro_gbs = ro_bytes / (ro_us * 1e-6) / 1e9

    # ---- max over ranks ----
    vals = torch.tensor([ms, e2e_ms, ro_us], dtype=torch.float64, device=dev)
    if pg:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms, ro_us = [float(x) for x in vals.tolist()]

    if rank == 0:
        tokens = L * world
        fam, (fam_ms, fam_n) = max(((f, v) for f, v in prof.items() if v[1] > 0), key=lambda kv: kv[1][0])
        per_launch_ms = fam_ms / fam_n
        alg = algorithmic_bytes(fam, L, H, SESSIONS, D)
        achieved = alg / (per_launch_ms * 1e-3) / 1e9
        step_alg = (L * H * (3 * 2 * D + 4 + 2 + 4 * D) + SESSIONS * H * 12 * D * D)
        cpu = None
        if pool is not None:
            cpu_measure(pool, 256)  # warm the workers
            t_cpu = cpu_measure(pool, CPU_SAMPLE_TOKENS)
            pool.close()
            cpu = {"value": CPU_SAMPLE_TOKENS / t_cpu, "unit": "tokens/s", "cores": cores, "kind": "port",
                   "sample": f"1 session x {CPU_SAMPLE_TOKENS} tokens x {H} heads, d={D} (oracle/gdn2.py "
                             f"chunked float64, heads in parallel)"}
        out = {
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sessions_per_gpu": SESSIONS, "tokens_per_session": T,
                       "heads": H, "head_dim": D, "chunk_tokens": CHUNK_TOKENS,
                       "parallelism": f"dp{world} (sessions sharded, no collective)",
                       "l2": "flushed (256 MiB write) between timed steps"},
            "roofline": {"bound": "hbm", "kernel": fam, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": read_traffic(fam), "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": alg, "launch_ms": per_launch_ms},
            "step_roofline": {"bytes": step_alg, "gbs": step_alg / (ms * 1e-3) / 1e9,
                              "frac": step_alg / (ms * 1e-3) / 1e9 / hbm},
            "kernels": {f: {"ms_per_step": v[0] / args.steps, "launches": v[1]} for f, v in prof.items() if v[1]},
            "e2e": None if only_update else {
                    "value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": bytes_in,
                    "d2h_bytes_per_step": bytes_out, "ms_per_step": e2e_ms},
            "readout": None if only_update else {"workload": "config2: 256 sessions x 16 heads, fp32 128x128 state, 1 bf16 query each, "
                                    "fused l2norm/read/gated RMSNorm/residual, one layer per call",
                        "us_per_layer": ro_us, "gbs": ro_gbs * world, "frac": ro_gbs / hbm},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(out), flush=True)
    if pg:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, rank, world):
    """The reference has no CPU implementation of this path; its CPU restatement (the oracle)
    runs on the host cores with the same metric and config."""
    if rank != 0:
        return
    pool, cores = cpu_pool()
    for _ in range(max(1, min(args.warmup, 1))):
        cpu_measure(pool, 256)
    total = 0.0
    for i in range(args.steps):
        total += cpu_measure(pool, args.reference_tokens, seed=i)
    pool.close()
    value = args.reference_tokens * args.steps / total
    sample = (f"each step: 1 session x {args.reference_tokens} tokens x {H} heads, d={D}, oracle/gdn2.py "
              f"chunked float64 (CPU restatement of the reference algorithm), heads in parallel")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": "host cores"},
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
    ap.add_argument("--reference-tokens", type=int, default=1024)
    ap.add_argument("--sessions", type=int, default=SESSIONS, help="sessions per GPU (profiling cases)")
    ap.add_argument("--only", choices=["all", "update"], default="all",
                    help="update: time only the commit step (no e2e, readout, CPU baseline)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
