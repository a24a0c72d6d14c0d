"""Benchmark of the INT8 decode-attention hot path (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg0|cfg1|cfg2|cfg3|cfg4]

A step is one decode-attention call over the configuration's whole batch.  The
default workload is BASELINE configs[1] (cfg1): paged INT8 KV, B16, 32 Q/KV heads,
D128, seq 4096, page 16, pool = 4096 pages + 10% slack, shuffled block_table.  Its
539 MB of KV is larger than L2 (126 MB), so no flush is needed between steps; cfg0
(135 MB) rotates over four copies of its inputs instead.

ours (default): inputs resident in HBM; K timed steps between CUDA events on the
launching stream (barrier + synchronize on both sides; N>1 = independent per-rank
request shards of the same configuration, max time over ranks).  ``value`` is the
aggregate algorithmic bandwidth (bytes every rank's calls must move / time).
``roofline`` divides the decode kernel's algorithmic bytes per launch by its mean
launch time over that timed region and compares with the measured copy peak, the
read-only stream peak measured in the same run, and 8 TB/s nominal.  ``e2e`` times the
public call with the per-step inputs (q, block_table, lengths) copied from pinned host
memory and the output copied back every step.  Two sub-objects accompany cfg1:
``paged_vs_contiguous`` (the same KV laid out contiguously, through the fused entry
point, timed in the same run) and ``seqshard`` (cfg3, the 131072-token requests split
by page windows across the N ranks with the peer-memory exchange, plus an in-run check
of rank 0's merged output against a single-GPU decode of the whole sequence).
``cpu_baseline`` times the CPU reference arm on the box's host cores.

reference: ``oracle/torch_reference.py`` -- the reference's CPU ``fused``/``paged``
backends restated op for op in torch -- on host-built inputs of the same configuration
(never the CUDA library), whole calls, all host cores, rank 0 only under torchrun.
"""

from __future__ import annotations

import argparse
import json
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
NOMINAL_HBM_GBS = 8000.0
REFERENCE_BUDGET_S = 60.0  # timed CPU work of the reference arm, at most (3 calls minimum)


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["cfg0", "cfg1", "cfg2", "cfg3", "cfg4"], default="cfg1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-soak", action="store_true", help="skip the 1.5 s clock soak (for profiler launch lists)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the paged_vs_contiguous / seqshard sub-objects and the read probe")
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
    """(DRAM bytes read + written per launch, source) of the decode kernel for this
    configuration from the committed ncu summary, or (None, None)."""
    p = ROOT / "profiles" / "traffic_per_launch.txt"
    if not p.exists():
        return None, None
    source = None
    for line in p.read_text().splitlines():
        if line.startswith("# source:"):
            source = line[len("# source:"):].strip()
        parts = line.split()
        if len(parts) >= 2 and parts[0] == config:
            return int(float(parts[1])), source or "profiles/traffic_per_launch.txt"
    return None, None


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


def torch_reference():
    """The CPU reference arm module (measurement infrastructure under oracle/)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import torch_reference as T

    return T


def use_all_host_cores() -> int:
    """torchrun sets OMP_NUM_THREADS=1; the CPU arms use every host core explicitly."""
    import torch

    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def time_cpu_calls(call, warmup: int, steps_requested: int, budget_s: float = REFERENCE_BUDGET_S):
    """Untimed warm-up calls, then whole timed calls until ``steps_requested`` are done or
    the budget is spent (at least 3).  Returns (seconds per call list)."""
    for _ in range(warmup):
        call()
    ts, spent = [], 0.0
    while len(ts) < max(1, steps_requested) and (len(ts) < 3 or spent < budget_s):
        t0 = time.perf_counter()
        call()
        ts.append(time.perf_counter() - t0)
        spent += ts[-1]
    return ts


def cpu_reference_line(config: str, warmup: int, steps: int, budget_s: float = REFERENCE_BUDGET_S):
    """Time the torch-CPU reference path on host-built inputs of ``config``."""
    T = torch_reference()
    cores = use_all_host_cores()
    t_build = time.perf_counter()
    wl = T.host_workload(config)
    t_build = time.perf_counter() - t_build
    ts = time_cpu_calls(wl.call, warmup, steps, budget_s)
    per_call = sum(ts) / len(ts)
    return wl, ts, per_call, cores, t_build


# ------------------------------------------------------------------------------------
# reference arm
# ------------------------------------------------------------------------------------


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    if args.config == "cfg4":
        run_serving_reference(args)
        return
    warm = min(args.warmup, 1)
    wl, ts, per_call, cores, t_build = cpu_reference_line(args.config, warm, args.steps)
    value = wl.bytes_per_call / per_call / 1e12
    sample = (f"whole calls of {wl.name} (all {len(wl.lengths)} requests, inputs built on the host in "
              f"{t_build:.1f} s, not timed): {len(ts)} timed calls after {warm} warm-up; at most "
              f"{REFERENCE_BUDGET_S:.0f} s of timed calls (minimum 3), so steps may be fewer than requested")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": len(ts), "steps_requested": args.steps, "warmup": warm, "warmup_requested": args.warmup,
        "ms_per_step": per_call * 1e3, "us_per_call": per_call * 1e6,
        "tokens_per_s": len(wl.lengths) / per_call, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 KV, fp16 q/out, fp32 accumulate", "data": "synthetic",
        "config": {"workload": wl.name, "global_batch": len(wl.lengths), "seq_len": max(wl.lengths),
                   "parallelism": "cpu (rank 0 only)", "bytes_per_call": wl.bytes_per_call},
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": cores, "kind": "port", "sample": sample,
                         "os_cpu_count": os.cpu_count(), "torch_threads": cores,
                         "impl": "oracle/torch_reference.py: reference fused/paged CPU backends restated in torch"},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "call_s": ts,
    }
    print(json.dumps(line), flush=True)


def run_serving_reference(args):
    """cfg4 at reduced scale on the CPU reference allocator (oracle/torch_reference.py)."""
    T = torch_reference()
    cores = use_all_host_cores()
    res = T.serving_loop(T.ServingParams())
    value = res["bytes_moved"] / res["loop_s"] / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": res["steps"], "steps_requested": args.steps, "warmup": 0, "ms_per_step": res["loop_s"] / res["steps"] * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 KV, fp16 q/out/tokens, fp32 accumulate", "data": "synthetic",
        "config": {"workload": "cfg4_serving_loop (reduced scale)", "parallelism": "cpu (rank 0 only)",
                   **res["params"]},
        "serving": res,
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": cores, "kind": "port",
                         "sample": "reduced-scale serving loop (see config): the full-scale allocator needs more "
                                   "than 60 GB of host memory and hours of CPU time",
                         "os_cpu_count": os.cpu_count(), "torch_threads": cores},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------


class Timer:
    """Device time of ``steps`` calls on one stream (barrier + synchronize on both
    sides, max over ranks)."""

    def __init__(self, dev, world):
        import torch

        self.dev, self.world = dev, world
        self.stream = torch.cuda.current_stream(dev)

    def barrier(self):
        import torch
        import torch.distributed as dist

        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, ms: float) -> float:
        import torch
        import torch.distributed as dist

        t = torch.tensor([ms], dtype=torch.float64, device=self.dev)
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def run(self, step, steps: int) -> float:
        import torch

        self.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        for i in range(steps):
            step(i)
        b.record(self.stream)
        self.barrier()
        return self.max_over_ranks(a.elapsed_time(b))


def host_us_per_call(call, n: int = 50) -> float:
    """Host-side cost of issuing one call (validation, plan, tensor maps, launch): the
    wall time of issuing n calls right after a synchronize, before the queue fills."""
    import torch

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n):
        call()
    t1 = time.perf_counter()
    torch.cuda.synchronize()
    return (t1 - t0) / n * 1e6


class E2EPipeline:
    """Per-step host<->device traffic through the public API: every step copies its
    inputs (packed into one pinned host buffer) to one of two device buffers on a side
    stream and reads its output back on a second side stream, so neighbouring steps'
    copies overlap this step's decode, as a serving loop arranges it.  ``make_run(b,
    views)`` returns the call that consumes device buffer b's views and returns its
    output tensor."""

    def __init__(self, dev, host_tensors, make_run, out_like):
        import torch

        self.dev = dev
        sizes = [t.numel() * t.element_size() for t in host_tensors]
        self.h2d_bytes = sum(sizes)
        self.d2h_bytes = out_like.numel() * out_like.element_size()
        self.host_in, self.dev_in, self.runs, self.outs_host = [], [], [], []
        for b in range(2):
            h = torch.empty(self.h2d_bytes, dtype=torch.uint8).pin_memory()
            views, off = [], 0
            d = torch.empty(self.h2d_bytes, dtype=torch.uint8, device=dev)
            for t, n in zip(host_tensors, sizes):
                h[off:off + n].copy_(t.cpu().contiguous().view(-1).view(torch.uint8))
                views.append(d[off:off + n].view(t.dtype).view(t.shape))
                off += n
            self.host_in.append(h)
            self.dev_in.append(d)
            d.copy_(h)
            self.runs.append(make_run(b, views))
            self.outs_host.append(torch.empty(out_like.shape, dtype=out_like.dtype).pin_memory())
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.h2d_done = [torch.cuda.Event() for _ in range(2)]
        self.kern_done = [torch.cuda.Event() for _ in range(2)]

    def step(self, i, cur):
        import torch

        b = i % 2
        if i < 2:  # the first step of each buffer forks from the compute stream
            self.h2d.wait_stream(cur)
        else:
            self.h2d.wait_event(self.kern_done[b])
        with torch.cuda.stream(self.h2d):
            self.dev_in[b].copy_(self.host_in[b], non_blocking=True)
            self.h2d_done[b].record(self.h2d)
        cur.wait_event(self.h2d_done[b])
        out = self.runs[b]()
        self.kern_done[b].record(cur)
        self.d2h.wait_event(self.kern_done[b])
        with torch.cuda.stream(self.d2h):
            self.outs_host[b].copy_(out, non_blocking=True)

    def graph(self, steps: int):
        """Capture ``steps`` pipelined steps as one CUDA graph (so the host's per-step
        stream/event/copy calls do not pace the GPU); returns its replay."""
        import torch

        stream = torch.cuda.current_stream(self.dev)
        for i in range(4):  # eager warm-up: workspaces, tickets, kernel configuration
            self.step(i, stream)
        stream.wait_stream(self.d2h)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            cap = torch.cuda.current_stream()
            for i in range(steps):
                self.step(i, cap)
            cap.wait_stream(self.h2d)
            cap.wait_stream(self.d2h)
        return g.replay


def read_probe_gbs(dev, gib: float = 4.0, reps: int = 5) -> float:
    """Best-of-reps read-only HBM bandwidth (fs_read_bandwidth_probe over a buffer far
    larger than L2)."""
    import ctypes as C

    import torch

    from flashspec_b200 import _lib
    from flashspec_b200.quant import stream_of

    lib = _lib.load()
    nbytes = int(gib * (1 << 30))
    buf = torch.ones(nbytes // 4, dtype=torch.int32, device=dev)
    sink = torch.zeros(1 << 16, dtype=torch.int32, device=dev)
    used = C.c_int32(0)
    stream = stream_of(dev)

    def call():
        _lib.check(lib.fs_read_bandwidth_probe(buf.data_ptr(), nbytes, sink.data_ptr(), sink.numel(), C.byref(used),
                                               stream), "fs_read_bandwidth_probe")

    call()
    best = 0.0
    s = torch.cuda.current_stream(dev)
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        call()
        b.record(s)
        b.synchronize()
        best = max(best, nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
    del buf
    torch.cuda.empty_cache()
    return best


def build_workload(config: str, rank: int, world: int):
    from flashspec_b200 import configs

    seed = 1000 * rank
    if config == "cfg0":
        return configs.cfg0(seed=seed)
    if config == "cfg1":
        return configs.cfg1(seed=seed)
    if config == "cfg2":
        return configs.cfg2(seed=seed)
    return configs.cfg3_shard(rank, world)


def contiguous_copy(wl):
    """The paged workload's KV gathered into the contiguous (fused) layout: values
    [B, H, nblk, 16, D] in logical page order, qparams [B, H, nblk] (all requests full)."""
    import flashspec_b200 as fs

    t = wl.cache.block_table

    def gather(qt):
        v = qt.values[t].squeeze(3).permute(0, 2, 1, 3, 4).contiguous()  # [B, H, nblk, 16, D]
        s = qt.scale[t].squeeze(-1).squeeze(-1).squeeze(-1).permute(0, 2, 1).contiguous()
        z = qt.zero_point[t].squeeze(-1).squeeze(-1).squeeze(-1).permute(0, 2, 1).contiguous()
        b, h, n = s.shape
        return fs.QuantizedTensor(v, s.view(b, h, n, 1, 1), z.view(b, h, n, 1, 1), 16, (b, h, n * 16, 128))

    return gather(wl.cache.k_quant), gather(wl.cache.v_quant)


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch

    import flashspec_b200 as fs

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    timer = Timer(dev, world)
    stream = timer.stream
    cfg = args.config
    fused = cfg == "cfg0"
    seqshard = cfg == "cfg3"
    wl = build_workload(cfg, rank, world)
    decoder = None

    # ---- the call of one step ----------------------------------------------------------
    if fused:
        # cfg0 is 135 MB (about L2 size): rotate over four copies so every call reads HBM
        copies = [(wl.q, wl.k_quant, wl.v_quant)]
        for _ in range(3):
            copies.append((wl.q.clone(), fs.QuantizedTensor(wl.k_quant.values.clone(), wl.k_quant.scale.clone(),
                                                              wl.k_quant.zero_point.clone(), 16,
                                                              wl.k_quant.original_shape),
                           fs.QuantizedTensor(wl.v_quant.values.clone(), wl.v_quant.scale.clone(),
                                              wl.v_quant.zero_point.clone(), 16, wl.v_quant.original_shape)))

        def step(i):
            q, kq, vq = copies[i % 4]
            return fs.fused_dequant_attention_cuda(q, kq, vq)
    elif seqshard:
        from flashspec_b200.dist import SequenceShardedDecoder

        decoder = SequenceShardedDecoder()
        n_pages = wl.cache.block_table.shape[1]
        # graphs of kSeqGraph steps (and a one-step graph for a remainder): every step is
        # one decode call, without the start of a graph launch between most of them
        replay_n, _ = decoder.capture(wl.q, wl.cache, n_pages, steps=kSeqGraph)
        replay_1, _ = decoder.capture(wl.q, wl.cache, n_pages)

        def step(i, total=None):
            total = total or args.steps
            full = total // kSeqGraph * kSeqGraph
            if i >= full:
                replay_1()
            elif i % kSeqGraph == 0:
                replay_n()
    else:
        def step(i):
            return fs.paged_quant_attention_cuda(wl.q, wl.cache, num_splits=wl.num_splits)

    # ---- warm-up and a clock soak of ~1.5 s so nvidia-smi sees the load ------------------
    sampler = ClockSampler() if rank == 0 else None
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.start()
    t_soak = time.time()
    while not args.no_soak and time.time() - t_soak < 1.5:
        for i in range(200):
            step(i)
        torch.cuda.synchronize()

    # ---- device-resident timed region ----------------------------------------------------
    elapsed_ms = timer.run(step, args.steps)
    t_wall1 = time.time()
    host_us = (host_us_per_call(replay_n) / kSeqGraph if seqshard and args.steps >= kSeqGraph
               else host_us_per_call(lambda: step(0)))

    # ---- end-to-end through the public API with host buffers -----------------------------
    q = wl.q
    if fused:
        host = [q]

        def make_run(b, views):
            kq, vq = copies[b][1], copies[b][2]
            return lambda: fs.fused_dequant_attention_cuda(views[0], kq, vq)
    else:
        cache = wl.cache
        host = [q, cache.block_table, cache.lengths]

        def make_run(b, views):
            c = fs.PagedKVCache(cache.k_quant, cache.v_quant, views[1], views[2], cache.block_size,
                                cache.max_seq_len)
            if seqshard:  # one captured decoder step per input buffer
                rep, out = decoder.capture(views[0], c, n_pages)

                def run():
                    rep()
                    return out
                return run
            return lambda: fs.paged_quant_attention_cuda(views[0], c, num_splits=wl.num_splits)
    pipe = E2EPipeline(dev, host, make_run, q)
    kGraphSteps = 10
    e2e_steps = max(kGraphSteps, min(args.steps, 500) // kGraphSteps * kGraphSteps)
    if seqshard:  # its steps are graph replays already: issue them eagerly, in pipeline
        for i in range(4):
            pipe.step(i, stream)
        stream.wait_stream(pipe.d2h)

        def e2e(i):
            pipe.step(i + 4, stream)
            if i == e2e_steps - 1:
                stream.wait_stream(pipe.d2h)
    else:
        replay_e2e = pipe.graph(kGraphSteps)

        def e2e(i):
            if i % kGraphSteps == 0:
                replay_e2e()
    for i in range(3 * kGraphSteps):
        e2e(i)
    e2e_ms = timer.run(e2e, e2e_steps)
    if sampler is not None:
        sampler.stop()
    if decoder is not None:
        decoder.close()  # raises if any exchange timed out

    # ---- sub-objects ---------------------------------------------------------------------
    extras = {}
    if not args.no_extras and cfg == "cfg1":
        extras["seqshard"] = seqshard_sub(args, rank, world, dev, timer)
        if world == 1:
            extras["paged_vs_contiguous"] = paged_vs_contiguous(args, wl, timer)
            extras["other_configs"] = other_configs(args, timer, dev)
    read_gbs = read_probe_gbs(dev) if (rank == 0 and not args.no_extras) else None
    if rank != 0:
        return

    # ---- the JSON line -------------------------------------------------------------------
    peak, peak_kind = measured_peaks()
    per_call_ms = elapsed_ms / args.steps
    # bytes one rank's decode moves per step (cfg3: its own page window + q/out + table)
    launch_bytes = wl.bytes_per_call // world if seqshard else wl.bytes_per_call
    achieved = launch_bytes / (per_call_ms * 1e-3) / 1e9
    calls_bytes = wl.bytes_per_call * (1 if seqshard else world)  # cfg3: one call spans all ranks
    value = calls_bytes * args.steps / (elapsed_ms * 1e-3) / 1e12
    e2e_value = calls_bytes * e2e_steps / (e2e_ms * 1e-3) / 1e12
    batch = int(wl.q.shape[0]) * (1 if seqshard else world)
    seq_len = int(wl.k_quant.original_shape[2]) if fused else max(wl.lengths)
    traffic, traffic_src = traffic_per_launch(cfg)
    if seqshard and world > 1:
        traffic = None  # the committed capture is of the one-rank launch
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "traffic_source": traffic_src,
                "peak_kind": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                "kernel_us": per_call_ms * 1e3,
                "kernel_us_source": "mean launch time over the timed region (CUDA events on the launching stream)"
                                    + ("; the step's kernel includes the fused exchange epilogue"
                                       if seqshard and world > 1 else ""),
                "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS}
    if read_gbs is not None:
        roofline.update({"read_peak_gbs": read_gbs, "frac_of_read_peak": achieved / read_gbs,
                         "read_peak_kind": "measured in this run: fs_read_bandwidth_probe over 4 GiB, best of 5"})
    api = ("flashspec_b200.fused_dequant_attention_cuda" if fused else
           "flashspec_b200 sequence-sharded decoder (one captured step per call)" if seqshard else
           "flashspec_b200.paged_quant_attention_cuda")
    line = {
        "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": per_call_ms, "us_per_call": per_call_ms * 1e3,
        "tokens_per_s": batch / (per_call_ms * 1e-3), "higher_is_better": True,
        "scaling": "strong" if seqshard else "weak",
        "vs_baseline": None, "dtype": "int8 KV, fp16 q/out, fp32 accumulate", "data": "synthetic",
        "config": {"workload": wl.name, "global_batch": batch, "seq_len": seq_len,
                   "q_heads": wl.q_heads if not fused else 32, "kv_heads": wl.kv_heads if not fused else 32,
                   "page": 16,
                   "parallelism": (f"sequence-shard x{world} (decode with the peer-memory exchange of O/LSE + "
                                   "merge fused into its epilogue)" if seqshard
                                   else f"request-shard x{world}" if world > 1 else "single"),
                   "l2": ("four rotated input copies (135 MB each, > L2 together)" if fused
                          else "inputs larger than L2 (no flush)"),
                   "bytes_per_call_per_gpu": launch_bytes,
                   **({"cuda_graph": f"{kSeqGraph} steps per graph replay"} if seqshard else {})},
        "roofline": roofline,
        "e2e": {"value": e2e_value, "unit": "TB/s", "h2d_bytes_per_step": pipe.h2d_bytes,
                "d2h_bytes_per_step": pipe.d2h_bytes, "us_per_call": e2e_ms / e2e_steps * 1e3,
                "api": api + ("; each step a graph replay, its inputs copied H2D from pinned host on a side stream "
                              "(double-buffered) and its output read back on a second side stream" if seqshard else
                              " replayed from a CUDA graph of 10 steps; every step one packed H2D of its inputs from "
                              "pinned host (side stream, double-buffered) and its output read back (second side "
                              "stream), overlapping the neighbouring steps' decode")},
        "host_us_per_call": host_us,
        "gpu_launches": args.steps,  # cfg3: one kernel per step (fused exchange on N > 1, plain decode on 1)
        "clocks": sampler.summary(t_soak, t_wall1) if sampler is not None else {},
    }
    line.update(extras)
    if world == 1 and not args.no_cpu_baseline and cfg in ("cfg0", "cfg1", "cfg2"):
        _, ts, per_call, cores, _ = cpu_reference_line(cfg, 1, 3, budget_s=30.0)
        line["cpu_baseline"] = {
            "value": wl.bytes_per_call / per_call / 1e12, "unit": "TB/s", "cores": cores, "kind": "port",
            "sample": f"whole calls of {wl.name} on host-built inputs: 1 warm-up + {len(ts)} timed",
            "us_per_call": per_call * 1e6, "os_cpu_count": os.cpu_count(),
            "impl": "oracle/torch_reference.py (reference CPU backends restated in torch)",
        }
    print(json.dumps(line), flush=True)


def paged_vs_contiguous(args, wl, timer):
    """The cfg1 KV in the contiguous layout through the fused entry point, same run.  The
    two are timed alternately (five rounds each, median), both with the same lengths,
    so clock drift under the power cap does not favour either."""
    import torch

    import flashspec_b200 as fs

    kq, vq = contiguous_copy(wl)
    q, lengths = wl.q, wl.cache.lengths

    def contiguous(i):
        fs.fused_dequant_attention_cuda(q, kq, vq, lengths)

    def paged(i):
        fs.paged_quant_attention_cuda(q, wl.cache)

    for i in range(max(3, args.warmup)):
        contiguous(i)
    n = max(50, min(args.steps, 500))
    tc, tp = [], []
    for _ in range(5):
        tp.append(timer.run(paged, n) / n)
        tc.append(timer.run(contiguous, n) / n)
    mp, mc = statistics.median(tp), statistics.median(tc)
    out_c = fs.fused_dequant_attention_cuda(q, kq, vq, lengths)
    out_p = fs.paged_quant_attention_cuda(q, wl.cache)
    same = bool(torch.equal(out_c, out_p))
    del kq, vq
    torch.cuda.empty_cache()
    return {"paged_us": mp * 1e3, "contiguous_us": mc * 1e3, "paged_over_contiguous": mp / mc,
            "outputs_bit_identical": same, "rounds": 5, "calls_per_round": n,
            "note": "same int8 bytes and lengths; contiguous = values [B, H, nblk, 16, D] through fs_fused_decode; "
                    "alternating rounds, medians"}


def other_configs(args, timer, dev):
    """cfg0 (contiguous, four rotated input copies), cfg2 (ragged GQA at its configured
    4 splits and on the default plan), cfg1's shape in the symmetric per-token format, and
    cfg4 (the serving loop), each on this GPU, so one default run records every
    configuration's device time."""
    import torch

    import flashspec_b200 as fs
    from flashspec_b200 import configs
    from flashspec_b200.serving import ServingConfig, run

    peak, _ = measured_peaks()
    n = max(50, min(args.steps, 500))
    res = {}

    def line(name, nbytes, ms, **kw):
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[name] = {"us_per_call": ms * 1e3, "tb_s": gbs / 1e3, "frac_of_copy_peak": gbs / peak,
                     "frac_of_nominal_8tbs": gbs / NOMINAL_HBM_GBS, "bytes_per_call": nbytes, "calls": n, **kw}

    wl0 = configs.cfg0()
    copies = [(wl0.q, wl0.k_quant, wl0.v_quant)]
    for _ in range(3):
        copies.append((wl0.q.clone(), *(fs.QuantizedTensor(t.values.clone(), t.scale.clone(), t.zero_point.clone(), 16,
                                                           t.original_shape) for t in (wl0.k_quant, wl0.v_quant))))
    step0 = lambda i: fs.fused_dequant_attention_cuda(*copies[i % 4])
    for i in range(8):
        step0(i)
    line("cfg0", wl0.bytes_per_call, timer.run(step0, n) / n, l2="four rotated input copies")
    del copies, wl0, step0
    torch.cuda.empty_cache()

    wl2 = configs.cfg2()
    for splits, tag in [(4, "cfg2_splits4"), (None, "cfg2_default_plan")]:
        step2 = lambda i: fs.paged_quant_attention_cuda(wl2.q, wl2.cache, num_splits=splits)
        for i in range(8):
            step2(i)
        line(tag, wl2.bytes_per_call, timer.run(step2, n) / n)
    del wl2
    torch.cuda.empty_cache()

    # cfg1's shape in the symmetric per-token format of the configurations' wording
    g = torch.Generator(device=dev).manual_seed(0)
    b, h, seq, d = 16, 32, 4096, 128
    k = torch.randn(b, h, seq, d, generator=g, device=dev, dtype=torch.float16)
    v = torch.randn(b, h, seq, d, generator=g, device=dev, dtype=torch.float16)
    q = torch.randn(b, h, d, generator=g, device=dev, dtype=torch.float16)
    perm = torch.randperm(b * seq // 16, generator=torch.Generator().manual_seed(1))
    sym = fs.paged_cache_symmetric(k, v, 16, perm=perm)
    del k, v
    step_s = lambda i: fs.paged_quant_attention_cuda(q, sym)
    for i in range(8):
        step_s(i)
    sym_bytes = b * (seq // 16) * h * 2 * (16 * d + 16 * 4) + 2 * b * h * d * 2 + b * (seq // 16) * 8 + b * 8
    line("cfg1_symmetric_per_token", sym_bytes, timer.run(step_s, n) / n, kernel="tuned decode kernels, per-token scales")
    del sym, q
    torch.cuda.empty_cache()

    sc = ServingConfig(steps=2000, seed=0)
    r = run(sc, device=dev)
    res["cfg4"] = {"step_ms_mean": r["step_ms_mean"], "tokens_per_s_device": r["tokens_per_s_device"],
                   "attention_tb_s": r["attention_tbps"], "append_tb_s": r["append_tbps"],
                   "attention_frac_of_copy_peak": r["attention_tbps"] * 1e3 / peak,
                   "append_ms_per_step": r["append_ms_total"] / r["steps_measured"],
                   "gpu_launches": r["gpu_launches"], "steps": sc.steps}
    torch.cuda.empty_cache()
    return res


kSeqGraph = 10  # sequence-sharded steps recorded per CUDA graph


def seqshard_sub(args, rank: int, world: int, dev, timer):
    """cfg3 (B2, 64q/8kv, 131072 tokens) split by page windows over the N ranks and merged
    through the peer-memory exchange; rank 0 checks its merged output against a
    single-GPU decode of the whole sequence rebuilt from every rank's window."""
    import torch

    import flashspec_b200 as fs
    from flashspec_b200 import configs
    from flashspec_b200.dist import SequenceShardedDecoder, page_window

    wl = configs.cfg3_shard(rank, world)
    n_pages = int(wl.cache.block_table.shape[1])
    steps = max(20, min(args.steps, 2000)) // kSeqGraph * kSeqGraph

    def timed(transport):
        dec = SequenceShardedDecoder(transport=transport)
        replay, out = dec.capture(wl.q, wl.cache, n_pages, steps=kSeqGraph)
        for _ in range(max(3, args.warmup)):
            replay()
        ms = timer.run(lambda i: replay() if i % kSeqGraph == 0 else None, steps) / steps
        torch.cuda.synchronize()
        dec.close()  # raises if an exchange timed out
        return ms, out

    ms, out = timed("p2p")
    res = {"workload": wl.name, "n_gpus": world, "us_per_call": ms * 1e3,
           "value": wl.bytes_per_call / (ms * 1e-3) / 1e12, "unit": "TB/s (whole call, all ranks)",
           "bytes_per_call": wl.bytes_per_call, "steps": steps,
           "parallelism": (f"sequence-shard x{world}: one kernel per step, decode with the exchange fused into its "
                           "epilogue (fs_paged_decode_exchange)" if world > 1
                           else "one GPU (plain decode of the whole sequence)"),
           "gpu_launches_per_step": 1}
    if world > 1:  # the same step as decode + separate exchange kernel, for comparison
        ms_k, _ = timed("p2p_kernel")
        res["two_kernel_step"] = {"us_per_call": ms_k * 1e3, "value": wl.bytes_per_call / (ms_k * 1e-3) / 1e12,
                                  "parallelism": "decode into (O, LSE), then fs_exchange_merge"}
    if rank == 0:
        # the whole sequence on this GPU: every rank's window pool, concatenated
        pools_k, pools_v, table = [], [], torch.full_like(wl.cache.block_table, -1)
        off = 0
        for r in range(world):
            w = wl if r == 0 else configs.cfg3_shard(r, world)
            lo, hi = page_window(n_pages, r, world)
            t = w.cache.block_table[:, lo:hi]
            table[:, lo:hi] = torch.where(t >= 0, t + off, t)
            pools_k.append(w.cache.k_quant)
            pools_v.append(w.cache.v_quant)
            off += int(w.cache.k_quant.values.shape[0])

        def cat(parts):
            return fs.QuantizedTensor(torch.cat([p.values for p in parts]), torch.cat([p.scale for p in parts]),
                                      torch.cat([p.zero_point for p in parts]), 16,
                                      (off,) + tuple(parts[0].original_shape[1:]))

        full = fs.PagedKVCache(cat(pools_k), cat(pools_v), table, wl.cache.lengths, 16, wl.cache.max_seq_len)
        ref = fs.paged_quant_attention_cuda(wl.q, full).float()
        err = (out.float() - ref).abs()
        ok = bool(torch.all(err <= 2e-3 + 1e-2 * ref.abs()))
        res["parity_vs_single_gpu_full_decode"] = {"max_abs_err": float(err.max()), "within_2e-3_abs_1e-2_rel": ok}
    return res


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
    moved = res["attention_bytes"] + res["append_bytes"]
    peak, peak_kind = measured_peaks()
    att_gbs = res["attention_bytes"] / (res["attention_ms_total"] * 1e-3) / 1e9
    step_total_s = res["step_ms_mean"] * res["steps_measured"] * 1e-3
    line = {
        "metric": METRIC, "value": moved / step_total_s / 1e12 * world,
        "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": 0, "ms_per_step": res["step_ms_mean"],
        "tokens_per_s": res["tokens_per_s_device"] * world,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 KV, fp16 q/out/tokens, fp32 accumulate", "data": "synthetic",
        "config": {"workload": "cfg4_serving_loop", "parallelism": f"request-shard x{world}" if world > 1 else "single",
                   **{k: v for k, v in cfg.__dict__.items()}},
        "roofline": {"bound": "hbm", "achieved": att_gbs, "peak": peak, "unit": "GB/s", "frac": att_gbs / peak,
                     "traffic": None, "peak_kind": f"{peak_kind} copy bandwidth", "kernel": "attention launches"},
        "serving": res,
        "gpu_launches": res.get("gpu_launches"),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.config == "cfg4":
        run_serving(args, rank, world, local_rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
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
