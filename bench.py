"""Benchmark of the paged INT8 decode-attention hot path (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config cfg1]

A step is one decode-attention call over the configuration's whole batch.  The
default workload is BASELINE configs[1] (cfg1): paged INT8 KV, B16, 32 Q/KV heads,
D128, seq 4096, page 16, pool = 4096 pages + 10% slack, shuffled block_table.
Inputs are larger than L2 (539 MB of KV), so no flush is needed between steps.

ours (default): KV pool, q and the table are resident in HBM; K timed steps of
``paged_quant_attention_cuda`` between CUDA events (barrier + synchronize on both
sides; N>1 = independent per-rank shards, max time over ranks).  ``value`` is the
aggregate algorithmic bandwidth (bytes every rank's calls must move / time).
``e2e`` times the same public call with the per-step inputs (q, block_table,
lengths) copied from pinned host memory and the output copied back, every step
(copies double-buffered on side streams and steps replayed from a CUDA graph, so
the copies overlap neighbouring steps' decode).  ``roofline`` divides the kernel's
achieved bytes/s (per-launch CUDA events, in a second pass outside the timed loop)
by the measured HBM copy peak.  ``cpu_baseline`` times the CPU oracle (a numpy port of
the reference's ``paged_quant_attention``) on a bounded sample of the same data.

reference: times that CPU port on the box's host cores over a bounded sample per
step (rank 0 only under torchrun) and reports the same metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn µs/call & achieved HBM TB/s (frac of B200 peak), paged INT8 KV"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["cfg1", "cfg2", "cfg3", "cfg4"], default="cfg1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-soak", action="store_true", help="skip the 1.5 s clock soak (for profiler launch lists)")
    return ap.parse_args()


# ------------------------------------------------------------------------------------
# helpers
# ------------------------------------------------------------------------------------


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def traffic_per_launch(config: str):
    """Per-launch DRAM bytes (read + write) of the decode kernel from the committed ncu
    summary, or None."""
    p = ROOT / "profiles" / "traffic_per_launch.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == config:
            return int(float(parts[1]))
    return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU is busy."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0: float, t1: float, gpu_index=None):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        window = [l for (t, l) in self.lines if t0 <= t <= t1] or [l for (_, l) in self.lines]
        for line in window:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            if gpu_index is not None and f[0] != str(gpu_index):
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def build_workload(config: str, rank: int, world: int = 1):
    from flashspec_b200 import configs

    seed = 1000 * rank
    if config == "cfg1":
        return configs.cfg1(seed=seed)
    if config == "cfg2":
        return configs.cfg2(seed=seed)
    return configs.cfg3_shard(rank, world)


# ------------------------------------------------------------------------------------
# CPU baseline: numpy port of the reference paged path on a bounded sample
# ------------------------------------------------------------------------------------


def cpu_sample(wl, n_req: int):
    """Host copy of the first n_req requests of the workload: their pages only, as an
    oracle cache (the reference dequantizes the whole pool it is given)."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import flashspec_oracle as O

    table = wl.cache.block_table[:n_req].cpu().numpy()
    used = np.unique(table[table >= 0])
    remap = np.full(int(used.max()) + 1, -1, np.int64)
    remap[used] = np.arange(used.size)
    import torch

    idx = torch.from_numpy(used).to(wl.cache.k_quant.values.device)

    def sub(qt):
        return O.OQuant(qt.values[idx].cpu().numpy(), qt.scale[idx].cpu().numpy(), qt.zero_point[idx].cpu().numpy(),
                        16, (used.size,) + tuple(qt.original_shape[1:]))

    t = np.where(table >= 0, remap[np.maximum(table, 0)], -1)
    lengths = np.array(wl.lengths[:n_req], np.int64)
    cache = O.OPagedCache(sub(wl.cache.k_quant), sub(wl.cache.v_quant), t, lengths, 16, int(lengths.max()))
    q = wl.q[:n_req].cpu().numpy()
    return O, q, cache


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return 1


def time_cpu_baseline(wl, n_req: int, reps: int):
    O, q, cache = cpu_sample(wl, n_req)
    O.paged_quant_attention(q, cache)  # warm-up
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        O.paged_quant_attention(q, cache)
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    frac = sum((n + 15) // 16 for n in wl.lengths[:n_req]) / sum((n + 15) // 16 for n in wl.lengths)
    full_s = t / frac  # the sample's share of the call's pages
    return full_s, ts


# ------------------------------------------------------------------------------------
# arms
# ------------------------------------------------------------------------------------


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    import torch  # noqa: F401  (device-free)

    os.environ.setdefault("CUDA_VISIBLE_DEVICES", os.environ.get("CUDA_VISIBLE_DEVICES", ""))
    wl = build_workload(args.config, 0)
    n_req = 2 if args.config != "cfg3" else 1
    steps = max(1, min(args.steps, 5))
    warm = max(0, min(args.warmup, 1))
    O, q, cache = cpu_sample(wl, n_req)
    for _ in range(warm):
        O.paged_quant_attention(q, cache)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        O.paged_quant_attention(q, cache)
        ts.append(time.perf_counter() - t0)
    frac = sum((n + 15) // 16 for n in wl.lengths[:n_req]) / sum((n + 15) // 16 for n in wl.lengths)
    per_call = statistics.median(ts) / frac
    value = wl.bytes_per_call / per_call / 1e12
    sample = (f"first {n_req} of {len(wl.lengths)} requests of {wl.name} (their pages only), median of {steps} "
              f"calls, scaled by page share {frac:.4f}")
    cores = cpu_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus, "steps": steps,
        "warmup": warm, "ms_per_step": per_call * 1e3, "us_per_call": per_call * 1e6, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 KV / fp32 accumulate", "data": "synthetic",
        "config": {"workload": wl.name, "global_batch": len(wl.lengths), "seq_len": max(wl.lengths),
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    import flashspec_b200 as fs

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    wl = build_workload(args.config, rank, world)
    q, cache = wl.q, wl.cache
    splits = wl.num_splits
    seqshard = args.config == "cfg3"
    if seqshard:
        from flashspec_b200.dist import SequenceShardedDecoder

        decoder = SequenceShardedDecoder()
        n_pages = cache.block_table.shape[1]
        # one CUDA graph per step, unless the step holds an NCCL collective
        graphable = world == 1 or decoder.transport == "p2p"
        if graphable:
            replay, _ = decoder.capture(q, cache, n_pages)

            def call():
                replay()
        else:
            def call():
                return decoder(q, cache, n_pages)
    else:
        def call():
            return fs.paged_quant_attention_cuda(q, cache, num_splits=splits)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # warm-up (W steps) and a clock soak of ~1.5 s so nvidia-smi sees the load
    sampler = ClockSampler() if rank == 0 else None
    for _ in range(max(3, args.warmup)):
        call()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.start()
    t_soak = time.time()
    while not args.no_soak and time.time() - t_soak < 1.5:
        for _ in range(200):
            call()
        torch.cuda.synchronize()

    # ---- device-resident timed region ------------------------------------------------
    stream = torch.cuda.current_stream(dev)
    barrier()
    t_wall0 = time.time()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.steps):
        call()
    end.record(stream)
    barrier()
    t_wall1 = time.time()
    elapsed_ms = start.elapsed_time(end)
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())

    # per-launch durations for the roofline: the same steps again, each bracketed by
    # events (kept out of the timed loop above, whose launches they would space apart)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        evs[i][0].record(stream)
        call()
        evs[i][1].record(stream)
    barrier()
    launch_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)

    # ---- end-to-end through the public API with host buffers ----------------------------
    # Every step copies its inputs (q, block table, lengths) from pinned host memory and
    # reads its output back.  Sequence-sharded runs do it serially on the compute stream.
    # Otherwise the step's inputs travel as one packed H2D copy on a side stream into one
    # of two device buffers, and the output comes back on a second side stream, so the
    # copies of neighbouring steps overlap the decode of this one, as a serving loop
    # arranges it; the steps are replayed from a CUDA graph of kGraphSteps pipelined steps
    # so the host's per-step launch work does not pace the GPU.
    e2e_steps = max(1, min(args.steps, 500))
    qb = q.numel() * q.element_size()
    tb = cache.block_table.numel() * 8
    lb = cache.lengths.numel() * 8
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if seqshard and not graphable:
        q_host = q.cpu().pin_memory()
        table_host = cache.block_table.cpu().pin_memory()
        lengths_host = cache.lengths.cpu().pin_memory()
        out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
        q_dev, table_dev, lengths_dev = torch.empty_like(q), torch.empty_like(cache.block_table), torch.empty_like(cache.lengths)
        cache_e2e = fs.PagedKVCache(cache.k_quant, cache.v_quant, table_dev, lengths_dev, cache.block_size,
                                    cache.max_seq_len)

        def e2e_step(i):
            q_dev.copy_(q_host, non_blocking=True)
            table_dev.copy_(table_host, non_blocking=True)
            lengths_dev.copy_(lengths_host, non_blocking=True)
            out = decoder(q_dev, cache_e2e, n_pages)
            out_host.copy_(out, non_blocking=True)
    else:
        n_in = qb + tb + lb
        host_in, dev_in, q_in, caches, outs_host = [], [], [], [], []
        for b in range(2):
            h = torch.empty(n_in, dtype=torch.uint8).pin_memory()
            h[:qb].copy_(q.cpu().contiguous().view(-1).view(torch.uint8))
            h[qb:qb + tb].copy_(cache.block_table.cpu().contiguous().view(-1).view(torch.uint8))
            h[qb + tb:].copy_(cache.lengths.cpu().contiguous().view(-1).view(torch.uint8))
            d = torch.empty(n_in, dtype=torch.uint8, device=dev)
            host_in.append(h)
            dev_in.append(d)
            q_in.append(d[:qb].view(q.dtype).view(q.shape))
            caches.append(fs.PagedKVCache(cache.k_quant, cache.v_quant,
                                          d[qb:qb + tb].view(torch.int64).view(cache.block_table.shape),
                                          d[qb + tb:].view(torch.int64).view(cache.lengths.shape),
                                          cache.block_size, cache.max_seq_len))
            outs_host.append(torch.empty(q.shape, dtype=q.dtype).pin_memory())
        h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        h2d_done = [torch.cuda.Event() for _ in range(2)]
        kern_done = [torch.cuda.Event() for _ in range(2)]
        if seqshard:  # one captured decoder step (decode + exchange) per input buffer
            graphs = []
            for b in range(2):
                dev_in[b].copy_(host_in[b])
                graphs.append(decoder.capture(q_in[b], caches[b], n_pages))

        def run(b):
            if seqshard:
                graphs[b][0]()
                return graphs[b][1]
            return fs.paged_quant_attention_cuda(q_in[b], caches[b], num_splits=splits)

        def pipelined_step(i, cur):
            b = i % 2
            if i < 2:  # the first step of each buffer forks from the compute stream
                h2d_stream.wait_stream(cur)
            else:
                h2d_stream.wait_event(kern_done[b])
            with torch.cuda.stream(h2d_stream):
                dev_in[b].copy_(host_in[b], non_blocking=True)
                h2d_done[b].record(h2d_stream)
            cur.wait_event(h2d_done[b])
            out = run(b)
            kern_done[b].record(cur)
            d2h_stream.wait_event(kern_done[b])
            with torch.cuda.stream(d2h_stream):
                outs_host[b].copy_(out, non_blocking=True)

        kGraphSteps = 10
        for i in range(4):  # eager warm-up: workspaces, tickets, kernel configuration
            pipelined_step(i, stream)
        stream.wait_stream(d2h_stream)
        torch.cuda.synchronize()
        if seqshard:  # steps are already graph replays: issued eagerly, in pipeline
            def e2e_step(i):
                pipelined_step(i + 4, stream)
                if i == e2e_steps - 1:
                    stream.wait_stream(d2h_stream)
        else:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                cap = torch.cuda.current_stream()
                for i in range(kGraphSteps):
                    pipelined_step(i, cap)
                cap.wait_stream(h2d_stream)
                cap.wait_stream(d2h_stream)
            e2e_steps = max(kGraphSteps, e2e_steps // kGraphSteps * kGraphSteps)

            def e2e_step(i):
                if i % kGraphSteps == 0:
                    graph.replay()

    for i in range(3):
        e2e_step(i if (seqshard and not graphable) else 0)
    barrier()
    e0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    te = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())
    h2d = qb + tb + lb
    d2h = qb
    if sampler is not None:
        sampler.stop()
    if rank != 0:
        return

    peak, peak_kind = measured_peaks()
    # bytes one rank's decode moves (cfg3: its own page window + q/out + table), per step
    launch_bytes = wl.bytes_per_call // world if seqshard else wl.bytes_per_call
    achieved_gbs = launch_bytes / (launch_ms * 1e-3) / 1e9
    calls_bytes = wl.bytes_per_call * (1 if seqshard else world)  # cfg3: one call spans all ranks
    total_bytes = calls_bytes * args.steps
    value = total_bytes / (elapsed_ms * 1e-3) / 1e12
    e2e_value = calls_bytes * e2e_steps / (e2e_ms * 1e-3) / 1e12
    clocks = sampler.summary(t_soak, t_wall1) if sampler is not None else {}
    line = {
        "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": elapsed_ms / args.steps,
        "us_per_call": elapsed_ms / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if seqshard else "weak",
        "vs_baseline": None, "dtype": "int8 KV, fp16 q/out, fp32 accumulate", "data": "synthetic",
        "config": {"workload": wl.name, "global_batch": len(wl.lengths) * (1 if seqshard else world),
                   "seq_len": max(wl.lengths), "q_heads": wl.q_heads, "kv_heads": wl.kv_heads, "page": 16,
                   "parallelism": (f"sequence-shard x{world} ({'peer-memory exchange' if decoder.transport == 'p2p' else 'NCCL all-gather'} of O/LSE + merge)" if seqshard
                                   else f"request-shard x{world}" if world > 1 else "single"),
                   "l2": "inputs larger than L2 (no flush)", "bytes_per_call_per_gpu": wl.bytes_per_call},
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                     "frac": achieved_gbs / peak, "traffic": traffic_per_launch(args.config),
                     "peak_kind": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                     "kernel_us": launch_ms * 1e3},
        "e2e": {"value": e2e_value, "unit": "TB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "us_per_call": e2e_ms / e2e_steps * 1e3,
                "api": ("flashspec_b200 sequence-sharded decoder, q/table/lengths copied from pinned host and "
                        "the output read back serially every step" if (seqshard and not graphable) else
                        "flashspec_b200 sequence-sharded decoder, each step a CUDA-graph replay of decode + exchange; "
                        "every step one packed H2D of q/table/lengths from pinned host (side stream, double-buffered) "
                        "and its output read back (second side stream), overlapping the neighbouring steps" if seqshard else
                        "flashspec_b200.paged_quant_attention_cuda replayed from a CUDA graph of 10 steps; every "
                        "step one packed H2D of q/table/lengths from pinned host (side stream, double-buffered) "
                        "and its output read back (second side stream), overlapping the neighbouring steps' decode")},
        "gpu_launches": args.steps * (2 if seqshard else 1),
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline and not seqshard:
        n_req = 2 if args.config != "cfg3" else 1
        full_s, ts = time_cpu_baseline(wl, n_req, reps=3)
        line["cpu_baseline"] = {
            "value": wl.bytes_per_call / full_s / 1e12, "unit": "TB/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"first {n_req} requests of {wl.name} (their pages), median of 3 calls, scaled by page share",
            "us_per_call": full_s * 1e6,
        }
    print(json.dumps(line), flush=True)


def run_serving(args, rank: int, world: int, local_rank: int):
    """cfg4: the allocator-driven serving loop; a step is one decode step of the loop
    (admission/prefill, append of one token per live request, attention, release)."""
    import torch

    from flashspec_b200.serving import ServingConfig, run

    torch.cuda.set_device(local_rank)
    cfg = ServingConfig(steps=args.steps, seed=1000 * rank)
    res = run(cfg, device=f"cuda:{local_rank}")
    if rank != 0:
        return
    step_s = res["step_ms_mean"] * 1e-3
    moved = res["attention_bytes"] + res["append_bytes"]
    peak, peak_kind = measured_peaks()
    att_gbs = res["attention_bytes"] / (res["attention_ms_total"] * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": moved / (sum([res["step_ms_mean"]] * args.steps) * 1e-3) / 1e12 * world,
        "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": 0, "ms_per_step": res["step_ms_mean"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 KV, fp16 q/out/tokens, fp32 accumulate", "data": "synthetic",
        "config": {"workload": "cfg4_serving_loop", "parallelism": f"request-shard x{world}" if world > 1 else "single",
                   **{k: v for k, v in cfg.__dict__.items()}},
        "roofline": {"bound": "hbm", "achieved": att_gbs, "peak": peak, "unit": "GB/s", "frac": att_gbs / peak,
                     "traffic": None, "peak_kind": f"{peak_kind} copy bandwidth", "kernel": "attention launches"},
        "serving": res,
        "gpu_launches": None,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.config == "cfg4":
            print(json.dumps({"impl": "reference", "unavailable": "cfg4 reference arm not implemented"}))
            return
        run_reference(args, rank, world)
        return
    if args.config == "cfg4":
        run_serving(args, rank, world, local_rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        import datetime

        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
