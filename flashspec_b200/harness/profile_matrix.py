"""Cartesian sweep of microbench runs over shapes and kernel knobs -> manifest CSV.

    python -m flashspec_b200.harness.profile_matrix --backend cuda_paged --seq-lens 2048,4096 \\
        --num-splits 0,2,4,8 --num-warps 4,8 --out sweep.csv

Same role as the reference's scripts/profile_matrix.py:62-224 (subprocess per point, env
knobs, one manifest row per run); the knobs are this library's (FLASHSPEC_NUM_SPLITS,
FLASHSPEC_NUM_WARPS) and the rows carry the roofline fields.
"""

from __future__ import annotations

import argparse
import csv
import itertools
import json
import os
import subprocess
import sys
from pathlib import Path

FIELDS = ["backend", "batch", "heads", "kv_heads", "seq_len", "paged_layout", "length_pattern", "num_splits_env",
          "num_warps_env", "latency_ms", "achieved_algorithmic_gbps", "frac_of_measured_copy_peak",
          "frac_of_nominal_8tbs", "num_splits", "returncode", "error"]


def _ints(s: str):
    return [int(x) for x in s.split(",") if x.strip()]


def points(args):
    for b, h, s, layout, pattern, ns, nw in itertools.product(
            _ints(args.batches), _ints(args.heads), _ints(args.seq_lens), args.layouts.split(","),
            args.length_patterns.split(","), _ints(args.num_splits), _ints(args.num_warps)):
        yield {"batch": b, "heads": h, "seq_len": s, "paged_layout": layout, "length_pattern": pattern,
               "num_splits_env": ns, "num_warps_env": nw}


def run_point(args, pt) -> dict:
    env = dict(os.environ)
    env.pop("FLASHSPEC_NUM_SPLITS", None)
    env.pop("FLASHSPEC_NUM_WARPS", None)
    if pt["num_splits_env"]:
        env["FLASHSPEC_NUM_SPLITS"] = str(pt["num_splits_env"])
    if pt["num_warps_env"]:
        env["FLASHSPEC_NUM_WARPS"] = str(pt["num_warps_env"])
    cmd = [sys.executable, "-m", "flashspec_b200.harness.microbench", "--backend", args.backend,
           "--batch", str(pt["batch"]), "--heads", str(pt["heads"]), "--kv-heads", str(args.kv_heads or pt["heads"]),
           "--seq-len", str(pt["seq_len"]), "--paged-layout", pt["paged_layout"], "--length-pattern",
           pt["length_pattern"], "--iters", str(args.iters), "--repeats", str(args.repeats), "--device", args.device,
           "--json"]
    row = {"backend": args.backend, "kv_heads": args.kv_heads or pt["heads"], **pt}
    if args.dry_run:
        row.update(returncode=0, error="dry-run: " + " ".join(cmd))
        return row
    proc = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=args.timeout)
    row["returncode"] = proc.returncode
    if proc.returncode != 0:
        row["error"] = proc.stderr.strip().splitlines()[-1] if proc.stderr.strip() else "failed"
        return row
    data = json.loads(proc.stdout.strip().splitlines()[-1])
    for k in ("latency_ms", "achieved_algorithmic_gbps", "frac_of_measured_copy_peak", "frac_of_nominal_8tbs",
              "num_splits"):
        row[k] = data.get(k)
    return row


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--backend", default="cuda_paged", choices=["cuda_paged", "cuda_fused", "dense"])
    ap.add_argument("--batches", default="16")
    ap.add_argument("--heads", default="32")
    ap.add_argument("--kv-heads", type=int, default=0)
    ap.add_argument("--seq-lens", default="4096")
    ap.add_argument("--layouts", default="shuffled")
    ap.add_argument("--length-patterns", default="uniform")
    ap.add_argument("--num-splits", default="0")
    ap.add_argument("--num-warps", default="0")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--repeats", type=int, default=5)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--timeout", type=float, default=600)
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--out", type=Path, default=Path("profile_matrix.csv"))
    args = ap.parse_args(argv)
    rows = [run_point(args, pt) for pt in points(args)]
    args.out.parent.mkdir(parents=True, exist_ok=True)
    with args.out.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=FIELDS, extrasaction="ignore")
        w.writeheader()
        for r in rows:
            w.writerow(r)
    print(f"{len(rows)} rows -> {args.out}")
    return rows


if __name__ == "__main__":
    main()
