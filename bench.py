"""Benchmark: paged decode attention (HBM GB/s) on the Llama-3-8B decode configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the headline configuration, "C2"): Llama-3-8B heads (32 q / 8 kv, head_dim 128),
block_size 16, 32 layers with their own pools, batch 64, context lengths ~ U[512, 4096],
bf16 KV ~ N(0,1), shuffled non-contiguous block tables. One step = one decode step of the
batch: for each of the 32 layers, the write of the 64 new tokens' K/V into their slots followed by
paged decode attention of the 64 queries (attention.rs:104-109 order), both in one launch of
fa_paged_decode_append (`unfused_step_ms` times the same step as fa_reshape_and_cache +
fa_paged_decode, two launches per layer). Each layer's pool
(~0.6 GB) is larger than L2, so no L2 flush is needed between timed iterations.

Metric value: algorithmic KV bytes read per step (sum ctx x Hkv x d x 2 [K,V] x 2 B, plus the
q/out/table bytes) summed over the N GPUs x steps / max-over-ranks device time. Multi-GPU:
sequence sharding, every rank owns its own pool and batch of the same context lengths (values
seeded per rank), so the work per GPU is fixed; no collective on the data path ("weak").

Extra objects on the same JSON line: ``roofline`` (decode kernel: algorithmic bytes per launch
over its average launch duration in the timed region, which holds only those launches;
``isolated_launch_ms`` times single launches between their own events),
``cpu_baseline`` (the oracle restatement of the reference CPU path on this host's cores),
``e2e`` (host buffers in/out through the C ABI, copies inside the timed region), ``clocks``
(nvidia-smi samples during the timed region), ``prefill`` (C3 varlen prefill TFLOP/s).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged decode attn HBM GB/s (% of peak) & prefill TFLOP/s at 1/2/4/8 B200"
WORKLOAD = "C2 Llama-3-8B decode step: B=64, Hq=32, Hkv=8, d=128, bs=16, 32 layers, ctx~U[512,4096]"
NUM_LAYERS = 32
BATCH = 64


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=1000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-longctx", action="store_true")
    ap.add_argument("--no-projections", action="store_true")
    ap.add_argument("--no-c5", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-tp", action="store_true", help="skip the head-sharded decode (N > 1)")
    ap.add_argument("--no-bundle", action="store_true", help="skip the FLKV export measurement")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def profile_traffic(name: str):
    """dram bytes per launch from the committed ncu summary (profiles/<name>.md), if any."""
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip().split()[0])
    return None


class ClockSampler:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None
        self.window = None  # (t0, t1) host wall-clock bounds of the timed region

    def mark(self, t0: float, t1: float) -> None:
        self.window = (t0, t1)

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                ts = time.mktime(time.strptime(r[0].strip().split(".")[0], "%Y/%m/%d %H:%M:%S"))
                if self.window and not (self.window[0] - 1.0 <= ts <= self.window[1] + 1.0):
                    continue
                sm.append(float(r[2]))
                smax.append(float(r[3]))
                power.append(float(r[4]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[6:10]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        load = [s for s, p in zip(sm, power) if p > 200.0] or sm
        pload = [p for p in power if p > 200.0] or power
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w": round(statistics.median(pload), 1) if pload else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# reference arm: the reference's CPU paged attention (oracle restatement), host cores only
# ---------------------------------------------------------------------------------------

def cpu_model() -> str:
    """The host CPU's model string (/proc/cpuinfo), for every CPU-baseline record."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_sample(seed: int, batch: int):
    """Host-resident C2-shaped layer: the first `batch` sequences of the C2 context draw."""
    import torch
    from flour_b200.workloads import LLAMA8B, c2_contexts, make_decode, to_numpy
    b = make_decode(LLAMA8B, c2_contexts(seed)[:batch], torch.bfloat16, "cpu", seed)
    arrays = dict(q=to_numpy(b.q), kc=to_numpy(b.k_caches[0]), vc=to_numpy(b.v_caches[0]),
                  cu=np.arange(b.num_seqs + 1, dtype=np.int32), ctx=b.ctx_host,
                  bt=to_numpy(b.block_tables))
    return arrays, b.kv_bytes_per_layer() + b.io_bytes_per_layer()


def time_oracle(arrays, threads: int, reps: int, budget_s: float):
    import oracle
    times = []
    t_start = time.perf_counter()
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.paged_attention(arrays["q"], arrays["kc"], arrays["vc"], arrays["cu"], arrays["ctx"],
                               arrays["bt"], 4, 1 / math.sqrt(128), dtype=oracle.DT_BF16,
                               threads=threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    return times


def cpu_config_baselines(seed: int, threads: int, budget_s: float = 4.0) -> dict:
    """The CPU restatement of the reference path (cpu.rs:57-112) timed on bounded samples of
    the other configurations, in each one's own unit: C1 whole (its 4 sequences, f32), C3 one
    group of 4 sequences sharing a prefix (causal suffix FLOPs), C4 one 16K-32K sequence, C5 32 of
    its decode sequences plus one of its prefills (tokens per second through its 28 layers)."""
    import torch
    import oracle
    from flour_b200.workloads import (LLAMA8B, QWEN7B, c4_contexts, c5_plan, make_c1, make_c3,
                                      make_decode, make_prefill, to_numpy)

    def run(b, cu, n_rep, d, dt):
        arr = (to_numpy(b.q), to_numpy(b.k_caches[0]), to_numpy(b.v_caches[0]), cu,
               np.asarray(to_numpy(b.context_lens) if hasattr(b, "cu_seqlens_q") else b.ctx_host,
                          np.int32), to_numpy(b.block_tables))
        times, t_start = [], time.perf_counter()
        while True:
            t0 = time.perf_counter()
            oracle.paged_attention(*arr, n_rep, 1 / math.sqrt(d), dtype=dt, threads=threads)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_start > budget_s or len(times) >= 200:
                return statistics.median(times), len(times)

    res = {}
    b = make_c1("cpu", seed=1)
    s, n = run(b, np.arange(b.num_seqs + 1, dtype=np.int32), 7, 64, oracle.DT_F32)
    res["C1"] = {"value": round((b.kv_bytes_per_layer() + b.io_bytes_per_layer()) / s / 1e9, 3),
                 "unit": "GB/s", "sample": f"C1 whole ({b.num_seqs} sequences, f32), {n} runs"}
    p = make_c3("cpu", seed=seed + 3, num_seqs=4)
    s, n = run(p, to_numpy(p.cu_seqlens_q), 4, 128, oracle.DT_BF16)
    res["C3"] = {"value": round(p.flops() / s / 1e12, 5), "unit": "TFLOP/s",
                 "sample": f"one C3 group: 4 sequences sharing a prefix, {int(p.lens.sum())} tokens, "
                           f"{int((p.lens - p.prefix).sum())} new, {n} runs"}
    ctx = c4_contexts(seed, 1)
    d4 = make_decode(LLAMA8B, ctx, torch.bfloat16, "cpu", seed)
    s, n = run(d4, np.arange(2, dtype=np.int32), 4, 128, oracle.DT_BF16)
    res["C4"] = {"value": round(d4.kv_bytes_per_layer() / s / 1e9, 3), "unit": "GB/s",
                 "sample": f"one C4 sequence of {int(ctx[0])} tokens, {n} runs"}
    ctx5, is_pf, pf_len, _ = c5_plan(seed)
    dec = np.nonzero(~is_pf)[0][:32]
    pf = np.nonzero(is_pf)[0][:1]
    db = make_decode(QWEN7B, ctx5[dec], torch.bfloat16, "cpu", seed)
    pb = make_prefill(QWEN7B, pf_len[pf], np.zeros(1, np.int64), torch.bfloat16, "cpu", seed + 1)
    t_dec, n1 = run(db, np.arange(len(dec) + 1, dtype=np.int32), 7, 128, oracle.DT_BF16)
    t_pf, n2 = run(pb, to_numpy(pb.cu_seqlens_q), 7, 128, oracle.DT_BF16)
    tokens = len(dec) + int(pf_len[pf].sum())
    res["C5"] = {"value": round(tokens / ((t_dec + t_pf) * 28), 1), "unit": "tokens/s",
                 "sample": f"{len(dec)} C5 decode sequences + one {int(pf_len[pf].sum())}-token "
                           f"prefill, one layer timed ({n1}/{n2} runs), x28 layers"}
    for v in res.values():
        v["cores"] = threads
        v["cpu_model"] = cpu_model()
        v["kind"] = "port"
    return res


def run_c1(torch, ops, dev, stream):
    """C1 (the reference's CPU-runnable case: Qwen2.5-0.5B heads, f32, 4 sequences): one decode
    launch, too small to load the GPU; reported for completeness (graph of 50 launches)."""
    from flour_b200.workloads import make_c1
    b = make_c1(dev, seed=1)
    ws = ops.Workspace(dev)
    out = torch.empty_like(b.q)
    scale = 1.0 / math.sqrt(b.heads.head_dim)
    call = lambda: ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables,
                                    b.context_lens, b.heads.n_rep, scale, b.max_context_len, ws,
                                    out=out)
    call()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(50):
            call()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / 50
    nbytes = b.kv_bytes_per_layer() + b.io_bytes_per_layer()
    return {"config": "C1: Qwen2.5-0.5B heads (14/2, d=64), f32, 4 sequences, ctx ~ U[33, 512]",
            "us_per_launch": round(us, 2), "gbps": round(nbytes / us / 1e3, 2), "bytes": int(nbytes)}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle
    threads = oracle.cpu_threads()
    arrays, nbytes = cpu_sample(args.seed, BATCH)
    time_oracle(arrays, threads, max(args.warmup, 0), 60.0)
    times = time_oracle(arrays, threads, args.steps, 120.0)
    steps = len(times)
    total = sum(times)
    value = nbytes * steps / total / 1e9
    sample = (f"one layer of the C2 batch (64 seqs, {nbytes / 1e6:.0f} MB of KV) per step; "
              "a full step is 32 such layers")
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 KV, C2 shapes)", "impl": "reference",
        "config": {"workload": WORKLOAD, "layers_per_step": 1, "batch": BATCH,
                   "note": "reference CPU path restated in C++ (Rust reference not buildable here)",
                   "gpus_note": "one host process on rank 0 whatever --gpus is: its value does "
                                "not scale with N, so a GPU/CPU ratio at N > 1 is not a scaling "
                                "measure"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "cpu_model": cpu_model(), "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------

def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    from flour_b200 import _lib, ops
    _lib.lib()  # loads libflour_attn.so; raises without it (no fallback path exists)
    from flour_b200.workloads import LLAMA8B, c2_contexts, make_c3, make_decode

    hbm_peak, tc_peak, tc_sustained, peak_kind = peaks()
    seed = args.seed + rank
    h = LLAMA8B
    scale = 1.0 / math.sqrt(h.head_dim)
    # Weak scaling: every rank decodes a batch with the same context lengths (the same KV bytes
    # per step), filled with its own seeded values.
    batch = make_decode(h, c2_contexts(args.seed), torch.bfloat16, dev, seed, num_layers=NUM_LAYERS)
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    B = batch.num_seqs
    qs = [torch.randn((B, h.num_heads, h.head_dim), device=dev, generator=gen).to(torch.bfloat16)
          for _ in range(NUM_LAYERS)]
    knew = [torch.randn((B, h.num_kv_heads, h.head_dim), device=dev, generator=gen).to(torch.bfloat16)
            for _ in range(NUM_LAYERS)]
    vnew = [torch.randn((B, h.num_kv_heads, h.head_dim), device=dev, generator=gen).to(torch.bfloat16)
            for _ in range(NUM_LAYERS)]
    outs = [torch.empty_like(q) for q in qs]
    ctx = batch.ctx_host
    bt_host = batch.block_tables.cpu().numpy()
    last = ctx - 1
    slots = torch.tensor(bt_host[np.arange(B), last // 16] * 16 + last % 16, dtype=torch.int32,
                         device=dev)
    ws = ops.Workspace(dev)
    ws.get(ops.workspace_size(B, h.num_heads, h.num_kv_heads, h.head_dim, batch.max_context_len, 1))
    stream = torch.cuda.current_stream()

    def layer_step(l, q, kn, vn, out):
        ops.paged_decode_append(q, batch.k_caches[l], batch.v_caches[l], kn, vn,
                                batch.block_tables, batch.context_lens, h.n_rep, scale,
                                batch.max_context_len, ws, out=out)

    def step():
        for l in range(NUM_LAYERS):
            layer_step(l, qs[l], knew[l], vnew[l], outs[l])

    def step_unfused():
        for l in range(NUM_LAYERS):
            ops.reshape_and_cache(batch.k_caches[l], batch.v_caches[l], knew[l], vnew[l], slots)
            ops.paged_decode(qs[l], batch.k_caches[l], batch.v_caches[l], batch.block_tables,
                             batch.context_lens, h.n_rep, scale, batch.max_context_len, ws,
                             out=outs[l])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert ops.device_status() == 0, "kernels reported bad device data during warm-up"

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()

    bytes_per_layer = batch.kv_bytes_per_layer() + batch.io_bytes_per_layer()
    kv_bytes_step = NUM_LAYERS * bytes_per_layer

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather(vals):
        """Every rank's list of floats, indexed by rank (the same list on every rank)."""
        if world == 1:
            return [list(vals)]
        t = torch.tensor([float(v) for v in vals], dtype=torch.float64, device=dev)
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [o.tolist() for o in out]

    # ---- timed region: K graph replays of the 32-layer decode step ----------------------
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # Pre-roll (untimed) so the sampler is up and the GPU is under load when timing starts.
        t_end = time.time() + 0.6
        while time.time() < t_end:
            graph.replay()
            torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        w0 = time.time()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        clocks.mark(w0, time.time())
        barrier()
    own_ms = e0.elapsed_time(e1)
    ms = max_over_ranks(own_ms)
    ms_per_step = ms / args.steps
    # Whole-job bytes: the sum of every rank's bytes (equal by construction) over the slowest
    # rank's time.
    job_bytes_step = sum(b for (b,) in gather([kv_bytes_step]))
    value = job_bytes_step * args.steps / (ms / 1e3) / 1e9
    assert ops.device_status() == 0
    # Per-rank step time, decode fraction of the measured peak, SM clock and power (each rank's
    # own sampler over its own GPU), so a slow GPU in a multi-GPU run is named in the record.
    clk = clocks.summary()
    own_step = own_ms / args.steps
    ranks = gather([own_step, bytes_per_layer * NUM_LAYERS / (own_step / 1e3) / 1e9 / hbm_peak,
                    clk.get("sm_mhz") or 0.0, clk.get("power_w") or 0.0])
    per_rank = [{"rank": r, "ms_per_step": round(v[0], 4), "hbm_frac": round(v[1], 4),
                 "sm_mhz": v[2], "power_w": v[3]} for r, v in enumerate(ranks)]

    # ---- per-launch duration of the decode kernel (events on the launching stream) -------
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(NUM_LAYERS)]
    dec_ms = []
    for _ in range(max(2, min(args.steps, 5))):
        for l in range(NUM_LAYERS):
            evs[l][0].record(stream)
            layer_step(l, qs[l], knew[l], vnew[l], outs[l])
            evs[l][1].record(stream)
        torch.cuda.synchronize()
        dec_ms += [a.elapsed_time(b) for a, b in evs]
    dec_avg_ms = statistics.mean(dec_ms)

    # ---- the same step as two launches per layer (reshape_and_cache, then decode) -------------
    graph_u = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_u):
        step_unfused()
    for _ in range(3):
        graph_u.replay()
    torch.cuda.synchronize()
    barrier()
    u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps_u = max(10, args.steps // 4)
    u0.record(stream)
    for _ in range(reps_u):
        graph_u.replay()
    u1.record(stream)
    torch.cuda.synchronize()
    barrier()
    unfused_ms = max_over_ranks(u0.elapsed_time(u1)) / reps_u
    del graph_u
    # The timed region holds nothing but the 32 decode launches per step (fa_paged_decode_append
    # writes the new tokens inside the same launch), so the kernel's average launch duration
    # over the timed region is the step time / 32 (inter-launch gaps included).
    launch_ms = ms_per_step / NUM_LAYERS
    achieved = bytes_per_layer / (launch_ms / 1e3) / 1e9
    traffic = profile_traffic("paged_decode_c2")

    # ---- e2e: host buffers through the C ABI, copies in the timed region -----------------
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, torch, ops, batch, h, scale, slots, ws, dev, stream, kv_bytes_step,
                      world, barrier, max_over_ranks)

    # ---- prefill (C3) ------------------------------------------------------------------------
    prefill = None
    if not args.no_prefill:
        prefill = run_prefill(args, torch, ops, make_c3, dev, stream, tc_peak, seed, max_over_ranks,
                              barrier, world)

    # ---- C5 mixed serving step, strong-scaled over the ranks ---------------------------------
    c5 = None
    if not args.no_c5:
        c5 = run_c5(args, torch, ops, dev, stream, world, rank, max_over_ranks, barrier,
                    gather)
        torch.cuda.empty_cache()  # return C5's pools before C4 sizes its pool from free memory

    # ---- long-context split-K decode (C4) ----------------------------------------------------
    longctx = None
    if not args.no_longctx:
        longctx = run_longctx(args, torch, ops, dev, stream, hbm_peak, seed, max_over_ranks,
                              barrier, world)

    # ---- head-sharded decode with the all-gather fused into the kernel (N > 1) -----------------
    tp = None
    if world > 1 and not args.no_tp:
        tp = run_tp_decode(args, torch, ops, dev, stream, world, rank, max_over_ranks, barrier)
        torch.cuda.empty_cache()

    # ---- the fused projections either side of attention ---------------------------------------
    proj = None
    if not args.no_projections:
        proj = run_projections(torch, ops, dev, stream, tc_peak, hbm_peak, seed, max_over_ranks,
                               barrier)

    bundle = run_bundle(torch, ops, batch, dev, stream, hbm_peak, seed) \
        if not args.no_bundle else None

    c1 = run_c1(torch, ops, dev, stream) if world == 1 else None

    # ---- CPU baseline (rank 0, N=1 only) -----------------------------------------------------
    cpu = None
    cpu_cfg = None
    if not args.no_cpu_baseline and world == 1 and rank == 0:
        import oracle
        threads = oracle.cpu_threads()
        arrays, nbytes = cpu_sample(args.seed, 16)
        time_oracle(arrays, threads, 1, 30.0)
        times = time_oracle(arrays, threads, 200, 10.0)
        cpu = {"value": round(nbytes * len(times) / sum(times) / 1e9, 3), "unit": "GB/s",
               "cores": threads, "cpu_model": cpu_model(), "kind": "port",
               "sample": f"{len(times)} x one C2 layer of 16 sequences ({nbytes / 1e6:.0f} MB KV), "
                         "oracle restatement of src/backend/cpu.rs:57-112"}
        cpu_cfg = cpu_config_baselines(args.seed, threads)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 KV and queries, random-init; C2 shapes)",
            "config": {"workload": WORKLOAD, "global_batch": BATCH * world, "layers": NUM_LAYERS,
                       "parallelism": f"sequence-sharded x{world} (own pool per GPU)",
                       "l2": "inputs larger than L2 (0.6 GB pool per layer), no flush",
                       "kv_gb_per_step_per_gpu": round(kv_bytes_step / 1e9, 3),
                       "hbm_frac_of_measured_peak": round(value / world / hbm_peak, 4)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                         "traffic": traffic, "kernel": "paged_decode_kernel<bf16,128,2>",
                         "launch_ms": round(launch_ms, 5),
                         "frac_uses": "launch_ms: the decode kernel's average launch duration "
                                      "inside the graph-replayed timed region (step time / 32)",
                         "isolated_launch_ms": round(dec_avg_ms, 5),
                         "isolated_frac": round(bytes_per_layer / (dec_avg_ms / 1e3) / 1e9 /
                                                hbm_peak, 4),
                         "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": bytes_per_layer},
            "per_rank": per_rank,
            "gpu_launches": NUM_LAYERS * args.steps,
            "unfused_step_ms": round(unfused_ms, 4),
            "clocks": clk,
        }
        if e2e:
            line["e2e"] = e2e
        if cpu:
            line["cpu_baseline"] = cpu
        if prefill:
            line["prefill"] = prefill
        if longctx:
            line["longctx"] = longctx
        if proj:
            line["projections"] = proj
        if c5:
            line["c5"] = c5
        if c1:
            line["c1"] = c1
        if cpu_cfg:
            gpu_vals = {"C1": c1["gbps"] if c1 else None,
                        "C3": prefill["kernel_tflops"] if prefill else None,
                        "C4": longctx["gbps"] if longctx else None,
                        "C5": c5["tokens_per_s"] if c5 else None}
            for k, v in cpu_cfg.items():
                if gpu_vals.get(k):
                    v["gpu_value"] = gpu_vals[k]
                    v["gpu_over_cpu"] = round(gpu_vals[k] / v["value"], 1)
            line["cpu_baseline_configs"] = cpu_cfg
        if tp:
            line["tp_decode"] = tp
        if bundle:
            line["bundle_export"] = bundle
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def run_e2e(args, torch, ops, batch, h, scale, slots, ws, dev, stream, kv_bytes_step, world,
            barrier, max_over_ranks):
    """Per step: the host hands per-layer q and new k/v (pinned) plus the step's metadata
    (block tables, context lengths); the library writes the cache and attends (one
    fa_paged_decode_append per layer) and the host reads every layer's output back. Copies run on
    a side stream ahead of the decodes."""
    B = batch.num_seqs
    gen = torch.Generator().manual_seed(7)
    hq = [torch.randn((B, h.num_heads, h.head_dim), generator=gen).to(torch.bfloat16).pin_memory()
          for _ in range(NUM_LAYERS)]
    hk = [torch.randn((B, h.num_kv_heads, h.head_dim), generator=gen).to(torch.bfloat16).pin_memory()
          for _ in range(NUM_LAYERS)]
    hv = [torch.randn((B, h.num_kv_heads, h.head_dim), generator=gen).to(torch.bfloat16).pin_memory()
          for _ in range(NUM_LAYERS)]
    ho = [torch.empty((B, h.num_heads, h.head_dim), dtype=torch.bfloat16).pin_memory()
          for _ in range(NUM_LAYERS)]
    h_bt = batch.block_tables.cpu().pin_memory()
    h_ctx = batch.context_lens.cpu().pin_memory()
    d_bt, d_ctx = (torch.empty_like(x, device=dev) for x in (h_bt, h_ctx))
    dq = [torch.empty_like(x, device=dev) for x in hq]
    dk = [torch.empty_like(x, device=dev) for x in hk]
    dv = [torch.empty_like(x, device=dev) for x in hv]
    do = [torch.empty_like(x, device=dev) for x in ho]
    copy = torch.cuda.Stream(device=dev)
    h2d = sum(x.numel() * x.element_size() for x in (h_bt, h_ctx)) + \
        sum(x.numel() * x.element_size() for x in hq + hk + hv)
    d2h = sum(x.numel() * x.element_size() for x in ho)

    def one_step():
        ev_in = []
        with torch.cuda.stream(copy):
            copy.wait_stream(stream)
            d_bt.copy_(h_bt, non_blocking=True)
            d_ctx.copy_(h_ctx, non_blocking=True)
            for l in range(NUM_LAYERS):
                dq[l].copy_(hq[l], non_blocking=True)
                dk[l].copy_(hk[l], non_blocking=True)
                dv[l].copy_(hv[l], non_blocking=True)
                e = torch.cuda.Event()
                e.record(copy)
                ev_in.append(e)
        ev_out = []
        for l in range(NUM_LAYERS):
            # The copies run far ahead of the decodes, so the decode stream waits only at layers
            # 0, 1, 2, 4, 8 and 16, each wait covering the inputs of layers [l, 2l): fewer waits
            # between consecutive decode launches (e2e +1.2 % against a wait before every layer).
            if l == 0 or (l & (l - 1)) == 0:
                stream.wait_event(ev_in[min(2 * l, NUM_LAYERS) - 1 if l else 0])
            ops.paged_decode_append(dq[l], batch.k_caches[l], batch.v_caches[l], dk[l], dv[l],
                                    d_bt, d_ctx, h.n_rep, scale, batch.max_context_len, ws,
                                    out=do[l])
            e = torch.cuda.Event()
            e.record(stream)
            ev_out.append(e)
        with torch.cuda.stream(copy):
            for l in range(NUM_LAYERS):
                copy.wait_event(ev_out[l])
                ho[l].copy_(do[l], non_blocking=True)
        stream.wait_stream(copy)

    for _ in range(max(args.warmup, 3)):
        one_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        one_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    assert ops.device_status() == 0
    return {"value": round(kv_bytes_step * args.steps * world / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(ms / args.steps, 4)}


def run_prefill(args, torch, ops, make_c3, dev, stream, tc_peak, seed, max_over_ranks, barrier,
                world):
    """C3: 16 packed sequences, shared cached prefixes; per layer reshape_and_cache of the
    suffix K/V then causal varlen prefill over prefix+suffix. One layer's pool repeated."""
    b = make_c3(dev, seed=seed + 3)
    h = b.heads
    scale = 1.0 / math.sqrt(h.head_dim)
    ws = ops.Workspace(dev)

    def layer():
        ops.reshape_and_cache(b.k_caches[0], b.v_caches[0], b.key, b.value, b.slot_mapping)
        return ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                                 b.block_tables, h.n_rep, scale, b.max_seqlen_q, b.max_context_len,
                                 ws)

    out = layer()
    torch.cuda.synchronize()
    reps = 8
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(2):
        layer()
    torch.cuda.synchronize()
    barrier()
    e0.record(stream)
    for _ in range(reps):
        layer()
    e1.record(stream)
    torch.cuda.synchronize()
    # The prefill kernel alone: 30 launches, each between its own events on the launching
    # stream; the median is the kernel time (the suffix K/V are already in the pool).
    ops.reshape_and_cache(b.k_caches[0], b.v_caches[0], b.key, b.value, b.slot_mapping)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(30)]
    for p0, p1 in evs:
        p0.record(stream)
        ops.paged_prefill(b.q, b.k_caches[0], b.v_caches[0], b.cu_seqlens_q, b.context_lens,
                          b.block_tables, h.n_rep, scale, b.max_seqlen_q, b.max_context_len, ws,
                          out=out)
        p1.record(stream)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    ms = max_over_ranks(e0.elapsed_time(e1)) / reps
    launches = sorted(p0.elapsed_time(p1) for p0, p1 in evs)
    kernel_ms = max_over_ranks(statistics.median(launches))
    flops = b.flops()
    return {"config": "C3 varlen causal prefill, 16 seqs L~U[128,2048], groups of 4 sharing "
                      "0-50% cached prefixes, Llama-3-8B heads, bf16",
            "tflops_aggregate": round(flops * world / (ms / 1e3) / 1e12, 2),
            "tflops_aggregate_note": "reshape_and_cache + prefill per layer, one independent C3 "
                                     "batch per rank, summed over the ranks",
            "kernel_tflops": round(flops / (kernel_ms / 1e3) / 1e12, 2),
            "kernel_ms": round(kernel_ms, 5),
            "kernel_timing": "median of 30 single launches (CUDA events on the launching stream; "
                             "max over ranks)",
            "kernel_ms_min_max": [round(launches[0], 5), round(launches[-1], 5)],
            "frac_of_measured_peak": round(flops / (kernel_ms / 1e3) / 1e12 / tc_peak, 4),
            "ms_per_layer": round(ms, 4), "suffix_tokens": int(b.q.shape[0]),
            "flops_per_layer": flops}


def run_longctx(args, torch, ops, dev, stream, hbm_peak, seed, max_over_ranks, barrier, world):
    """C4: 16 sequences with ctx ~ U[16K, 32K] on one layer's pool sized toward 150 GB (capped by
    the free device memory less 8 GB), block ids drawn at random from the whole pool; split-K
    decode, one layer repeated 32 times."""
    from flour_b200.workloads import LLAMA8B, c4_contexts, make_decode
    h = LLAMA8B
    block_bytes = 2 * h.num_kv_heads * h.block_size * h.head_dim * 2  # K and V, bf16
    free, _ = torch.cuda.mem_get_info(dev)
    nb = int(min(150e9, max(free - 8e9, 4e9)) // block_bytes)
    ctx = c4_contexts(seed + 4)
    b = make_decode(h, ctx, torch.bfloat16, dev, seed + 4, pool_blocks=nb, fill=False)
    # Only the blocks the tables reference need values; fill them (about 1.6 GB).
    bt = b.block_tables.cpu().numpy()
    pages = (b.ctx_host.astype(np.int64) + 15) // 16
    used = torch.from_numpy(np.concatenate([bt[i, :n] for i, n in enumerate(pages)]).astype(np.int64))
    gen = torch.Generator(device=dev).manual_seed(seed + 5)
    for cache in (b.k_caches[0], b.v_caches[0]):
        for chunk in used.split(4096):
            idx = chunk.to(dev)
            cache[idx] = torch.randn((len(chunk),) + tuple(cache.shape[1:]), device=dev,
                                     generator=gen).to(cache.dtype)
    scale = 1.0 / math.sqrt(h.head_dim)
    ws = ops.Workspace(dev)
    out = torch.empty_like(b.q)
    reps = 32

    def launch():
        ops.paged_decode(b.q, b.k_caches[0], b.v_caches[0], b.block_tables, b.context_lens, h.n_rep,
                         scale, b.max_context_len, ws, out=out)

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    ms = max_over_ranks(e0.elapsed_time(e1)) / reps
    nbytes = b.kv_bytes_per_layer() + b.io_bytes_per_layer()
    gbps = nbytes / (ms / 1e3) / 1e9
    res = {"config": "C4 long-context split-K decode: 16 seqs, ctx ~ U[16384, 32768], Llama-3-8B "
                     "heads, bf16, block ids random over the whole pool, one layer x32",
           "gbps": round(gbps * world, 1), "frac_of_measured_peak": round(gbps / hbm_peak, 4),
           "ms_per_layer": round(ms, 4), "bytes_per_layer": nbytes,
           "pool_gb": round(nb * block_bytes / 1e9, 1), "mean_ctx": float(np.mean(ctx))}
    del b, out, ws
    torch.cuda.empty_cache()
    return res


def run_c5(args, torch, ops, dev, stream, world, rank, max_over_ranks, barrier, gather):
    """C5 mixed serving step: Qwen2-7B heads (Hq=28, Hkv=4, d=128), 28 layers, 512 sequences
    (ctx ~ LogNormal(ln 1024, 0.8) capped at 8192); about 10 % are new prompts of L ~ U[256, 2048]
    run as prefill, the rest decode one token. The sequences are partitioned over the ranks
    (prompts first by kernel work units, then decode sequences where the two-stream step time
    grows least), so the total work is fixed as N grows (strong scaling). One step = per layer:
    the decode sequences' new K/V write + decode (one fa_paged_decode_append launch) on one
    stream, the prefill sequences' reshape_and_cache and the prefill launch on a second stream
    (the two sub-batches share no data); each rank owns its own pools. Pools, queries and new
    K/V are seeded N(0,1) (only the blocks the tables reference are allocated and filled).
    Per rank, the decode stream alone and the prefill stream alone are also timed (graphs of one
    sub-batch), so the record names the limiting kernel on the slowest rank."""
    from flour_b200.workloads import QWEN7B, c5_plan, make_mixed_step, mixed_partition
    h, L = QWEN7B, 28
    ctx, is_pf, pf_len, cost = c5_plan(args.seed)
    mine = mixed_partition(cost, is_pf, world)[rank]
    # The batch builder hands the decode sequences over longest first (the order of a batch is
    # its free choice): the long sequences' splits and merges then start first instead of
    # trailing the launch (decode stream -9 % at N=1 and at the N=8 share, measured).
    dec = sorted((i for i in mine if not is_pf[i]), key=lambda i: -int(ctx[i]))
    pf = [i for i in mine if is_pf[i]]
    ms = make_mixed_step(h, ctx[dec], pf_len[pf], torch.bfloat16, dev, args.seed + rank, L)

    for _ in range(2):
        ms.run()
    torch.cuda.synchronize()
    assert ops.device_status() == 0

    def timed_graph(fn, reps):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        graph.replay()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        del graph
        return e0.elapsed_time(e1) / reps

    # The step as one CUDA graph (decode and prefill streams forked and joined inside it): the
    # host's launch cost stays out of the timing.
    own_ms = timed_graph(ms.run, 5)
    dec_ms = timed_graph(ms.run_decode, 5) if ms.dec is not None else 0.0
    pf_ms = timed_graph(ms.run_prefill, 5) if ms.pf is not None else 0.0
    assert ops.device_status() == 0
    per_rank = gather([own_ms, dec_ms / L, pf_ms / L])
    ms_max = max(r[0] for r in per_rank)
    slow = max(range(world), key=lambda r: per_rank[r][0])
    kvb = h.num_kv_heads * h.head_dim * 2 * 2
    dec_bytes = float(ctx[~is_pf].sum()) * kvb * L
    pf_flops = float((4.0 * h.num_heads * h.head_dim * pf_len[is_pf] * (pf_len[is_pf] + 1) / 2).sum()) * L
    tokens = int((~is_pf).sum() + pf_len[is_pf].sum())
    del ms
    res = {"config": "C5 mixed serving step: Qwen2-7B heads, 28 layers, 512 seqs (ctx ~ LogNormal"
                     "(ln 1024, 0.8) <= 8192), ~10 % new prefills L ~ U[256, 2048]; partitioned "
                     "over ranks, each rank's decode sequences longest first; seeded N(0,1) "
                     "pools, queries and new K/V",
           "scaling": "strong", "step_ms": round(ms_max, 4),
           "fastest_rank_step_ms": round(min(r[0] for r in per_rank), 4),
           "tokens_per_s": round(tokens / (ms_max / 1e3), 1),
           "decode_seqs": int((~is_pf).sum()), "prefill_seqs": int(is_pf.sum()),
           "prefill_tokens": int(pf_len[is_pf].sum()),
           "decode_kv_gb_per_step": round(dec_bytes / 1e9, 3),
           "prefill_tflop_per_step": round(pf_flops / 1e12, 3),
           "per_rank": [{"rank": r, "step_ms": round(v[0], 4),
                         "decode_only_ms_per_layer": round(v[1], 5),
                         "prefill_only_ms_per_layer": round(v[2], 5)}
                        for r, v in enumerate(per_rank)],
           "slowest_rank": slow,
           "slowest_rank_limit": ("prefill" if per_rank[slow][2] >= per_rank[slow][1] else "decode")}
    return res


def run_bundle(torch, ops, batch, dev, stream, hbm_peak, seed):
    """FLKV prefix export (KvCache::export_prefix_bundle, cache.rs:166-228; payload order
    bundle.rs:15-22) of a 2048-token prefix of the C2 pools: 128 blocks x 32 layers (268 MB).
    `kernel`: the one-launch gather into a device payload (bytes read + written over its time);
    `to_host`: gather + one D2H copy into pinned memory; `per_block_route`: the same bytes as
    2 x blocks x layers cudaMemcpyAsync (fa_read_block) into pinned memory."""
    nb = batch.k_caches[0].shape[0]
    ids = torch.from_numpy(np.random.default_rng(seed + 9).permutation(nb)[:128].astype(np.int32)
                           ).to(dev)
    ks, vs = batch.k_caches, batch.v_caches
    n = ops.bundle_payload_bytes(ks, vs, 128)
    payload = torch.empty(n, dtype=torch.uint8, device=dev)
    host = torch.empty(n, dtype=torch.uint8).pin_memory()
    for _ in range(3):
        ops.export_bundle_payload(ks, vs, ids, payload)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(20)]
    for a, b in evs:
        a.record(stream)
        ops.export_bundle_payload(ks, vs, ids, payload)
        b.record(stream)
    torch.cuda.synchronize()
    k_ms = statistics.median(a.elapsed_time(b) for a, b in evs)

    def to_host():
        ops.export_bundle_payload(ks, vs, ids, payload)
        host.copy_(payload, non_blocking=True)

    def per_block():
        piece = n // (128 * len(ks) * 2)
        ids_h = ids.cpu().tolist()
        o = 0
        for b in ids_h:
            for l in range(len(ks)):
                kd = host[o:o + piece]
                vd = host[o + piece:o + 2 * piece]
                ops.read_block(ks[l], vs[l], b, kd, vd)
                o += 2 * piece

    def timed(fn, reps=5):
        fn()
        torch.cuda.synchronize()
        t = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            t.append(e0.elapsed_time(e1))
        return statistics.median(t)

    host_ms = timed(to_host)
    per_ms = timed(per_block, 3)
    want = host.clone()
    ok = bool(torch.equal(payload.cpu(), want))
    assert ops.device_status() == 0
    return {"config": "FLKV export of a 2048-token prefix: 128 blocks x 32 layers, Llama-3-8B "
                      "heads, bf16", "payload_bytes": n,
            "kernel_ms": round(k_ms, 4),
            "kernel_gbps": round(2 * n / (k_ms / 1e3) / 1e9, 1),
            "kernel_frac_of_measured_hbm_peak": round(2 * n / (k_ms / 1e3) / 1e9 / hbm_peak, 4),
            "to_host_ms": round(host_ms, 3), "to_host_gbps": round(n / (host_ms / 1e3) / 1e9, 1),
            "per_block_route_ms": round(per_ms, 3), "per_block_route_copies": 2 * 128 * len(ks),
            "payloads_equal": ok}


def run_tp_decode(args, torch, ops, dev, stream, world, rank, max_over_ranks, barrier):
    """Head-sharded decode of ONE C2 batch (64 sequences, 32 layers) over all ranks: rank r holds
    KV heads [8r/N, 8(r+1)/N) of every layer's pool and the matching query heads (strong
    scaling). Fused: fa_paged_decode_tp stores each rank's head outputs into every rank's output
    buffer over NVLink, then fa_tp_sync; NCCL: fa_paged_decode into a local buffer followed by
    all_gather_into_tensor. Both steps are CUDA graphs of the 32 layers; after either one every
    rank holds the full [64, 32, 128] output of every layer. `local` (the rank's decode alone,
    no exchange) is the floor both are measured against."""
    import torch.distributed as dist
    from flour_b200.tp import HeadShardedGroup, head_shard, torch_exchange
    from flour_b200.workloads import LLAMA8B, Heads, c2_contexts, make_decode
    h = LLAMA8B
    if h.num_kv_heads % world:
        return None
    kv0, kv1, h0, h1 = head_shard(h.num_heads, h.num_kv_heads, world, rank)
    hs = Heads(h1 - h0, kv1 - kv0, h.head_dim)
    # Same sequences, contexts and block tables on every rank (same seed); this rank's heads.
    b = make_decode(hs, c2_contexts(args.seed), torch.bfloat16, dev, args.seed, num_layers=NUM_LAYERS)
    B = b.num_seqs
    scale = 1.0 / math.sqrt(h.head_dim)
    g = torch.Generator(device=dev).manual_seed(args.seed + 7 + rank)
    qs = [torch.randn((B, hs.num_heads, h.head_dim), device=dev, generator=g).to(torch.bfloat16)
          for _ in range(NUM_LAYERS)]
    ws = ops.Workspace(dev)
    ws.get(ops.workspace_size(B, hs.num_heads, hs.num_kv_heads, h.head_dim, b.max_context_len, 1))
    grp = HeadShardedGroup(world, rank, B, h.num_heads, h.head_dim, torch.bfloat16,
                           torch_exchange(), dev)
    loc = [torch.empty_like(q) for q in qs]
    gathered = [torch.empty((world,) + tuple(q.shape), dtype=q.dtype, device=dev) for q in qs]

    def step_fused():
        for l in range(NUM_LAYERS):
            grp.decode(qs[l], b.k_caches[l], b.v_caches[l], b.block_tables, b.context_lens,
                       hs.n_rep, scale, b.max_context_len, ws)

    def step_local():
        for l in range(NUM_LAYERS):
            ops.paged_decode(qs[l], b.k_caches[l], b.v_caches[l], b.block_tables, b.context_lens,
                             hs.n_rep, scale, b.max_context_len, ws, out=loc[l])

    def step_nccl():
        for l in range(NUM_LAYERS):
            ops.paged_decode(qs[l], b.k_caches[l], b.v_caches[l], b.block_tables, b.context_lens,
                             hs.n_rep, scale, b.max_context_len, ws, out=loc[l])
            dist.all_gather_into_tensor(gathered[l], loc[l])

    res = {"config": "C2 batch (64 seqs, 32 layers, Llama-3-8B heads) head-sharded over the ranks",
           "scaling": "strong", "tp": world,
           "kv_gb_per_step": round(float(b.ctx_host.sum()) * h.num_kv_heads * h.head_dim * 4
                                   * NUM_LAYERS / 1e9, 3)}
    graphs = {}
    try:
        for name, fn in (("local", step_local), ("fused", step_fused), ("nccl", step_nccl)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            barrier()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            graphs[name] = graph
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            barrier()
            reps = max(20, args.steps // 4)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            barrier()
            ms = max_over_ranks(e0.elapsed_time(e1)) / reps
            res[f"{name}_ms_per_step"] = round(ms, 4)
            res[f"{name}_gbps"] = round(res["kv_gb_per_step"] / (ms / 1e3), 1)
        status = ops.device_status()
        assert status == 0, f"head-sharded decode reported device status 0x{status:x}"
        # The fused output of the last layer equals the NCCL-gathered one (same kernel per head).
        full = grp.output(grp.epoch, B)
        ref = gathered[-1].permute(1, 0, 2, 3).reshape(B, h.num_heads, h.head_dim)
        res["fused_equals_nccl"] = bool(torch.equal(full, ref))
        res["speedup_vs_nccl"] = round(res["nccl_ms_per_step"] / res["fused_ms_per_step"], 3)
    finally:
        graphs.clear()  # graphs holding NCCL calls go before the process group
        torch.cuda.synchronize()
        barrier()
        grp.close()
    return res


def run_projections(torch, ops, dev, stream, tc_peak, hbm_peak, seed, max_over_ranks, barrier):
    """Llama-3-8B layer projections through the fused kernels: QKV + RoPE + reshape_and_cache
    (hidden 4096 -> 48 heads x 128) and o_proj + residual (4096 -> 4096), at the C3 prefill
    token count and at the C2 decode batch (64 tokens), plus the engine's logits readback at
    the C2 batch: final RMSNorm + lm_head (128256 x 4096) on each sequence's last token, f32.
    Each measurement replays a CUDA graph of `reps` calls that cycle through three copies of
    the weights (more than L2 together), so weights stream from HBM and no host launch
    overhead is timed. The GEMMs use programmatic dependent launch, so in such a sequence each
    call's prologue and first weight loads overlap the previous call's tail, as they overlap the
    preceding kernel of a layer."""
    from flour_b200.paged import rope_tables
    hidden, Hq, Hkv, d, vocab = 4096, 32, 8, 128, 128256
    N = (Hq + 2 * Hkv) * d
    g = torch.Generator(device=dev).manual_seed(seed + 7)
    copies = 3
    ws = [(torch.randn(N, hidden, device=dev, generator=g) / 64).to(torch.bfloat16)
          for _ in range(copies)]
    wos = [(torch.randn(hidden, Hq * d, device=dev, generator=g) / 64).to(torch.bfloat16)
           for _ in range(copies)]
    cos, sin = rope_tables(d, 8192, 500000.0, torch.bfloat16, dev)

    def timed(fns, reps):
        for f in fns:
            f()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for r in range(reps):
                fns[r % len(fns)]()
        graph.replay()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return max_over_ranks(e0.elapsed_time(e1)) / reps

    from flour_b200._lib import lib as _flib_p
    _lib_tile = _flib_p().fa_gemm_tile_width
    res = {}
    for name, T in (("prefill_c3_tokens", 15401), ("decode_c2_batch", 64)):
        x = torch.randn(T, hidden, device=dev, generator=g).to(torch.bfloat16)
        a = torch.randn(T, Hq * d, device=dev, generator=g).to(torch.bfloat16)
        nb = T // 16 + 8
        kc = torch.zeros(nb, Hkv, 16, d, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        pos = torch.arange(T, dtype=torch.int32, device=dev) % 8192
        slots = torch.arange(T, dtype=torch.int32, device=dev)
        q = torch.empty(T, Hq, d, device=dev, dtype=torch.bfloat16)
        out = torch.empty(T, hidden, device=dev, dtype=torch.bfloat16)
        fns = {"qkv_rope_cache": [lambda w=w: ops.qkv_rope_cache(x, w, kc, vc, pos, slots, Hq, cos,
                                                                 sin, q_out=q) for w in ws],
               "o_proj_residual": [lambda wo=wo: ops.o_proj_residual(a, wo, x, out=out)
                                   for wo in wos]}
        flops = {"qkv_rope_cache": 2 * T * hidden * N, "o_proj_residual": 2 * T * Hq * d * hidden}
        wbytes = {"qkv_rope_cache": N * hidden * 2, "o_proj_residual": hidden * Hq * d * 2}
        entry = {"tokens": T,
                 "tile_cols": {"qkv_rope_cache": int(_lib_tile(T, N, hidden)),
                               "o_proj_residual": int(_lib_tile(T, hidden, Hq * d))}}
        for k, fl in fns.items():
            ms = timed(fl, 12 if T > 1024 else 60)
            entry[k] = {"ms": round(ms, 4), "tflops": round(flops[k] / ms / 1e9, 1),
                        "frac_of_measured_tensor_peak": round(flops[k] / ms / 1e9 / tc_peak, 4),
                        "weight_gbps": round(wbytes[k] / ms / 1e6, 1),
                        "weight_frac_of_measured_hbm_peak": round(wbytes[k] / ms / 1e6 / hbm_peak, 4)}
        res[name] = entry
    del ws, wos
    # Logits readback at the C2 batch: 64 sequences' last tokens through norm + lm_head.
    B = 64
    lm = (torch.randn(vocab, hidden, device=dev, generator=g) / 64).to(torch.bfloat16)
    hid = torch.randn(B, hidden, device=dev, generator=g).to(torch.bfloat16)
    nw = torch.ones(hidden, device=dev, dtype=torch.bfloat16)
    cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
    normed = torch.empty(B, hidden, device=dev, dtype=torch.bfloat16)
    logits = torch.empty(B, vocab, device=dev, dtype=torch.float32)
    # Five replays of a 20-call graph: the median is reported, with the spread.
    lt = sorted(timed([lambda: ops.last_token_logits(hid, cu, lm, nw, 1e-5, normed_out=normed,
                                                     logits_out=logits)], 20) for _ in range(5))
    ms = lt[2]
    host = torch.empty(B, vocab, dtype=torch.float32, pin_memory=True)
    host.copy_(logits, non_blocking=True)  # first touch of the pinned pages, untimed
    torch.cuda.synchronize()
    copies = []
    for _ in range(7):
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record(stream)
        host.copy_(logits, non_blocking=True)
        r1.record(stream)
        torch.cuda.synchronize()
        copies.append(r0.elapsed_time(r1))
    lbytes = vocab * hidden * 2
    from flour_b200._lib import lib as _flib
    res["logits_c2_batch"] = {"sequences": B, "vocab": vocab, "ms": round(ms, 4),
                              "ms_min_max_of_5": [round(lt[0], 4), round(lt[-1], 4)],
                              "tile_cols": int(_flib().fa_gemm_tile_width(B, vocab, hidden)),
                              "weight_gbps": round(lbytes / ms / 1e6, 1),
                              "weight_frac_of_measured_hbm_peak": round(lbytes / ms / 1e6 / hbm_peak, 4),
                              "readback_ms": round(sorted(copies)[3], 4),
                              "readback_bytes": B * vocab * 4}
    assert ops.device_status() == 0
    return res


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
