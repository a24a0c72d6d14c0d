"""Single-point decode-attention microbenchmark, retargeted to B200.

    python -m flashspec_b200.harness.microbench --backend cuda_paged --batch 16 --heads 32 \\
        --seq-len 4096 --head-dim 128 --paged-layout shuffled --json

Keeps the JSON schema of the reference microbench (benchmarks/microbench.py:542-615:
the knob, length-pattern, layout, latency and ``measured_*`` keys) and adds the
roofline fields: algorithmic bytes of the call, achieved GB/s, and the fractions of the
measured HBM copy peak and of the 8 TB/s nominal figure.  Timing follows the reference
method (microbench.py:133-179): CUDA events around ``iters`` back-to-back calls, median
of ``repeats``.  ``--profile-ncu`` re-runs this command under ncu with the counter list of
``ncu_parse.FAST_METRICS`` and back-fills ``measured_*``.

Backends: ``cuda_paged`` / ``cuda_fused`` (the library) and ``dense`` (a plain torch
fp32 attention over fp16 K/V, usable on CPU, as a reference point and for schema tests).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
from pathlib import Path
from time import perf_counter

import torch

from . import ncu_parse

NOMINAL_HBM_GBS = 8000.0
NCU_KERNEL_REGEX = {"cuda_paged": "decode_", "cuda_fused": "decode_", "dense": "."}
COUNTER_SECTIONS = ("WarpStateStats", "SchedulerStats", "MemoryWorkloadAnalysis", "SpeedOfLight", "Occupancy")


def measured_copy_peak_gbs():
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def _percentile(values, pct):
    if not values:
        return 0.0
    v = sorted(values)
    pos = (len(v) - 1) * pct / 100.0
    lo = int(pos)
    hi = min(lo + 1, len(v) - 1)
    return v[lo] * (1 - (pos - lo)) + v[hi] * (pos - lo)


def resolve_lengths(args) -> list:
    """Per-request effective lengths (the reference's --lengths / --length-pattern rules,
    microbench.py:90-130)."""
    if args.lengths:
        vals = [int(x) for x in args.lengths.split(",") if x.strip()]
        if len(vals) == 1:
            vals = vals * args.batch
        if len(vals) != args.batch:
            raise ValueError("--lengths takes 1 or batch comma-separated values")
    elif args.length_pattern == "uniform":
        vals = [args.seq_len] * args.batch
    elif args.length_pattern == "descending":
        lo = max(1, args.seq_len // 4)
        vals = [args.seq_len] if args.batch == 1 else [
            int(round(args.seq_len - (args.seq_len - lo) * i / (args.batch - 1))) for i in range(args.batch)]
    elif args.length_pattern == "bimodal":
        short = max(1, args.seq_len // 4)
        split = args.batch // 2
        vals = [args.seq_len] * split + [short] * (args.batch - split)
    elif args.length_pattern == "random":
        g = torch.Generator().manual_seed(int(args.seed))
        vals = torch.randint(max(1, args.seq_len // 4), args.seq_len + 1, (args.batch,), generator=g).tolist()
    else:
        raise ValueError("unknown --length-pattern")
    if any(v < 1 or v > args.seq_len for v in vals):
        raise ValueError("effective lengths must lie in [1, seq_len]")
    return vals


def dense_attention(q, k, v, lengths=None):
    """fp32 masked softmax attention over dense K/V (GQA by repeating KV heads)."""
    g = q.shape[1] // k.shape[1]
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("bhd,bhsd->bhs", q.float(), kf) / math.sqrt(q.shape[-1])
    if lengths is not None:
        mask = torch.arange(k.shape[2], device=k.device)[None, :] >= lengths[:, None]
        s = s.masked_fill(mask[:, None, :], torch.finfo(torch.float32).min)
    return torch.einsum("bhs,bhsd->bhd", torch.softmax(s, -1), vf).to(q.dtype)


def measure_latency_ms(run, device, warmup, repeats, iters):
    out = run()
    for _ in range(max(0, warmup)):
        out = run()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    raw = []
    for _ in range(max(1, repeats)):
        if device.type == "cuda":
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(max(1, iters)):
                out = run()
            e.record()
            e.synchronize()
            raw.append(s.elapsed_time(e) / max(1, iters))
        else:
            t0 = perf_counter()
            for _ in range(max(1, iters)):
                out = run()
            raw.append((perf_counter() - t0) * 1e3 / max(1, iters))
    return out, raw, "cuda_event" if device.type == "cuda" else "perf_counter"


def cli_args(args, include_json: bool) -> list:
    a = ["--backend", args.backend, "--batch", str(args.batch), "--heads", str(args.heads),
         "--kv-heads", str(args.kv_heads or args.heads), "--seq-len", str(args.seq_len), "--head-dim",
         str(args.head_dim), "--block-size", str(args.block_size), "--iters", str(args.iters), "--warmup",
         str(args.warmup), "--repeats", "1", "--device", "cuda", "--dtype", args.dtype, "--paged-layout",
         args.paged_layout, "--layout-seed", str(args.layout_seed), "--length-pattern", args.length_pattern,
         "--seed", str(args.seed)]
    if args.lengths:
        a += ["--lengths", args.lengths]
    if args.num_splits:
        a += ["--num-splits", str(args.num_splits)]
    if include_json:
        a.append("--json")
    return a


def ncu_commands(args) -> dict:
    bench = " ".join(["python -m flashspec_b200.harness.microbench", *cli_args(args, include_json=True)])
    regex = NCU_KERNEL_REGEX.get(args.backend, ".")
    metrics = ",".join(ncu_parse.FAST_METRICS)
    sections = " ".join(f"--section {s}" for s in COUNTER_SECTIONS)
    return {
        "metrics_csv": f"ncu --metrics {metrics} --clock-control none -k regex:{regex} -c 5 --csv {bench}",
        # counter sections only (warp state, scheduler, memory, occupancy); the source page is not used
        "source_instruction_report": f"ncu {sections} --clock-control none -k regex:{regex} -c 1 -o mb_{args.backend} "
                                     f"{bench}",
    }


def run_ncu_and_backfill(args, result: dict) -> dict:
    cmd = [args.ncu_bin, "--metrics", ",".join(ncu_parse.FAST_METRICS), "--clock-control", "none", "-k",
           f"regex:{NCU_KERNEL_REGEX.get(args.backend, '.')}", "-c", str(args.ncu_launch_count), "--csv",
           sys.executable, "-m", "flashspec_b200.harness.microbench", *cli_args(args, include_json=False)]
    try:
        proc = subprocess.run(cmd, capture_output=True, text=True, timeout=args.ncu_timeout)
    except FileNotFoundError:
        result["profiler_error"] = f"ncu not found: {args.ncu_bin}"
        return result
    except subprocess.TimeoutExpired:
        result["profiler_error"] = f"ncu timed out after {args.ncu_timeout}s"
        return result
    if proc.returncode != 0:
        result["profiler_error"] = f"ncu exit {proc.returncode}: " + "\n".join(proc.stderr.strip().splitlines()[-6:])
        return result
    try:
        ncu_parse.apply_backfill(result, ncu_parse.parse_ncu_csv(proc.stdout))
    except ValueError as exc:
        result["profiler_error"] = f"could not parse ncu CSV: {exc}"
    return result


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description="flashspec_b200 decode-attention microbenchmark")
    ap.add_argument("--backend", choices=["dense", "cuda_fused", "cuda_paged"], default="cuda_paged")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--heads", type=int, default=8, help="query heads")
    ap.add_argument("--kv-heads", type=int, default=0, help="kv heads (0 = --heads)")
    ap.add_argument("--seq-len", type=int, default=512)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--lengths", default="")
    ap.add_argument("--length-pattern", default="uniform", choices=["uniform", "descending", "bimodal", "random"])
    ap.add_argument("--paged-layout", default="contiguous", choices=["contiguous", "shuffled", "interleaved"])
    ap.add_argument("--layout-seed", type=int, default=0)
    ap.add_argument("--num-splits", type=int, default=0)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--repeats", type=int, default=10)
    ap.add_argument("--device", default="auto")
    ap.add_argument("--dtype", default="float16", choices=["float16", "float32"])
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--output", type=Path)
    ap.add_argument("--include-raw", action="store_true")
    ap.add_argument("--profile-ncu", action="store_true")
    ap.add_argument("--ncu-bin", default="ncu")
    ap.add_argument("--ncu-launch-count", type=int, default=5)
    ap.add_argument("--ncu-timeout", type=float, default=600.0)
    return ap.parse_args(argv)


def main(argv=None) -> dict:
    args = parse_args(argv)
    device = torch.device("cuda" if args.device == "auto" and torch.cuda.is_available() else
                          ("cpu" if args.device == "auto" else args.device))
    dtype = getattr(torch, args.dtype)
    hkv = args.kv_heads or args.heads
    gen = torch.Generator(device=device).manual_seed(args.seed)
    q = torch.randn((args.batch, args.heads, args.head_dim), generator=gen, device=device, dtype=dtype)
    k = torch.randn((args.batch, hkv, args.seq_len, args.head_dim), generator=gen, device=device, dtype=dtype)
    v = torch.randn((args.batch, hkv, args.seq_len, args.head_dim), generator=gen, device=device, dtype=dtype)
    lengths_list = resolve_lengths(args)
    lengths = torch.tensor(lengths_list, dtype=torch.int64, device=device)
    attn_lengths = None if args.length_pattern == "uniform" and not args.lengths else lengths
    splits = args.num_splits or None
    stats = {}
    if args.backend == "dense":
        def run():
            return dense_attention(q, k, v, attn_lengths)
        dense_b = 2 * k.numel() * k.element_size()
        stats = {"dense_kv_bytes": float(dense_b), "quant_kv_bytes": float(dense_b), "compression_ratio": 1.0,
                 "materializes_dense_kv": 0.0}
        alg = dense_b + 2 * q.numel() * q.element_size()
    else:
        import flashspec_b200 as fs
        from flashspec_b200.configs import algorithmic_bytes

        if args.backend == "cuda_fused":
            kq, vq = fs.quantize_int8_per_block(k, args.block_size), fs.quantize_int8_per_block(v, args.block_size)

            def run():
                return fs.fused_dequant_attention_cuda(q, kq, vq, attn_lengths, num_splits=splits)

            _, stats = fs.fused_dequant_attention_cuda(q, kq, vq, attn_lengths, return_stats=True, num_splits=splits)
            alg = algorithmic_bytes(args.batch, args.heads, hkv, lengths_list if attn_lengths is not None else
                                    [args.seq_len] * args.batch, with_lengths=attn_lengths is not None)
        else:
            cache = fs.PagedKVCache.from_dense(k, v, args.block_size, lengths=attn_lengths,
                                               block_table_pattern=args.paged_layout, layout_seed=args.layout_seed)

            def run():
                return fs.paged_quant_attention_cuda(q, cache, num_splits=splits)

            _, stats = fs.paged_quant_attention_cuda(q, cache, return_stats=True, num_splits=splits)
            alg = algorithmic_bytes(args.batch, args.heads, hkv, lengths_list,
                                    table_cols=int(cache.block_table.shape[1]))
    if args.backend != "dense":
        del k, v  # only the quantized copies are needed from here on
    out, raw, method = measure_latency_ms(run, device, args.warmup, args.repeats, args.iters)
    lat = statistics.median(raw)
    peak = measured_copy_peak_gbs()
    achieved = alg / (lat * 1e-3) / 1e9
    cmds = ncu_commands(args)
    result = {
        "backend": args.backend, "device": str(device),
        "device_name": torch.cuda.get_device_name(device) if device.type == "cuda" else "cpu",
        "dtype": args.dtype, "batch": args.batch, "heads": args.heads, "kv_heads": hkv, "seq_len": args.seq_len,
        "head_dim": args.head_dim, "block_size": args.block_size, "seed": args.seed,
        "length_pattern": args.length_pattern, "passes_lengths_to_attention": attn_lengths is not None,
        "effective_lengths": lengths_list, "effective_min_seq_len": min(lengths_list),
        "effective_max_seq_len": max(lengths_list), "paged_layout": args.paged_layout,
        "paged_layout_seed": args.layout_seed, "iters": args.iters, "warmup": args.warmup, "repeats": args.repeats,
        "timing_method": method, "latency_ms": lat, "latency_mean_ms": statistics.fmean(raw),
        "latency_std_ms": statistics.pstdev(raw) if len(raw) > 1 else 0.0, "latency_min_ms": min(raw),
        "latency_max_ms": max(raw), "latency_p50_ms": _percentile(raw, 50), "latency_p90_ms": _percentile(raw, 90),
        "latency_p99_ms": _percentile(raw, 99), "tokens_per_second": args.batch / max(1e-9, lat / 1e3),
        "estimated_dense_kv_bytes": stats.get("dense_kv_bytes"), "estimated_quant_kv_bytes": stats.get("quant_kv_bytes"),
        "compression_ratio": stats.get("compression_ratio"),
        "materializes_dense_kv": bool(stats.get("materializes_dense_kv", 0.0)),
        "num_splits": stats.get("num_splits"), "block_n": stats.get("block_n"), "num_warps": stats.get("num_warps"),
        "env_flashspec_num_splits": os.environ.get("FLASHSPEC_NUM_SPLITS"),
        "env_flashspec_block_n": os.environ.get("FLASHSPEC_BLOCK_N"),
        "env_flashspec_num_warps": os.environ.get("FLASHSPEC_NUM_WARPS"),
        "bandwidth_fields_are_estimates": True,
        "estimated_effective_quant_kv_bandwidth_gbps": (stats.get("quant_kv_bytes") or 0) / max(1e-9, lat / 1e3) / 1e9,
        "algorithmic_bytes": alg, "achieved_algorithmic_gbps": achieved,
        "frac_of_measured_copy_peak": achieved / peak if peak else None,
        "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS,
        "measured_kernel_latency_ms": lat if method == "cuda_event" else None,
        "measured_dram_bytes": None, "measured_achieved_bandwidth_gbps": None, "measured_occupancy_pct": None,
        "measured_sm_utilization_pct": None, "measured_dram_throughput_pct": None,
        "measured_registers_per_thread": None, "measured_theoretical_occupancy_pct": None,
        "measured_ncu_kernel_duration_ms": None, "measured_ncu_kernel_count": None,
        "measured_ncu_kernel_names": None,
        "profiler_metrics_source": "nsight_compute_required_for_dram_occupancy_sm",
        "nsight_compute_command": cmds["metrics_csv"], "nsight_compute_source_command": cmds["source_instruction_report"],
        "nsight_compute_commands": cmds, "output_checksum": float(out.float().sum().item()),
    }
    if args.include_raw:
        result["raw_latency_ms"] = raw
    if args.profile_ncu:
        if device.type != "cuda":
            result["profiler_error"] = "--profile-ncu needs a CUDA device"
        else:
            run_ncu_and_backfill(args, result)
    if args.output:
        args.output.parent.mkdir(parents=True, exist_ok=True)
        args.output.write_text(json.dumps(result, indent=2))
    if args.json:
        print(json.dumps(result))
    else:
        for key in ("backend", "latency_ms", "achieved_algorithmic_gbps", "frac_of_measured_copy_peak", "num_splits"):
            print(f"{key}: {result[key]}")
    return result


if __name__ == "__main__":
    main()
