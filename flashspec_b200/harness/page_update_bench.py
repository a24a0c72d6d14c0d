"""Device time of the allocator's write path (``fs_page_update``): a decode append
(one new row in each of ``--requests`` pages, all heads, K and V) and a prefill of
``--prefill-pages`` fresh pages.

    python -m flashspec_b200.harness.page_update_bench --json
    python -m flashspec_b200.harness.page_update_bench --launch-only --calls 3 --prefill-pages 1024  # for ncu

The calls are the ones ``PagedKVAllocator.append_batch`` / ``add_request`` make
(src/flashspec/paged.py:108-136,226-255 of the reference), launched directly with fixed
item lists so that only the kernel is timed.  Times are per-launch device durations
from CUPTI (``torch.profiler``), median over ``--calls`` launches.  Algorithmic bytes:
an append reads the old page (bs * D codes + scale + zero point) and the new row, and
writes the page back; a prefill reads bs rows of the source and writes the page.
``FLASHSPEC_PAGE_UPDATE_SCALAR=1`` selects the shared-memory kernel with the correctly
rounded division for comparison; both give identical bytes.
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys

import numpy as np
import torch


def run(args) -> dict:
    from torch.profiler import ProfilerActivity, profile

    from flashspec_b200 import paged as P

    if not torch.cuda.is_available():
        raise SystemExit("page_update_bench needs a CUDA device")
    H, D, bs = args.heads, args.head_dim, args.block_size
    pages = max(args.pool_pages, args.requests + args.prefill_pages)
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    dk, dv = (P.empty_pool(pages, H, bs, D, "cuda") for _ in range(2))
    for t in (dk, dv):
        t.values.random_(-128, 127, generator=g)
        t.scale.uniform_(0.001, 0.05, generator=g)
        t.zero_point.random_(0, 255, generator=g)
    rng = np.random.default_rng(args.seed)
    R = args.requests
    app = np.zeros(R, P.ITEM_DTYPE)
    app["page"] = rng.permutation(pages - args.prefill_pages)[:R]
    app["src_b"] = np.arange(R)
    app["dst_row"] = bs // 3
    app["n_rows"] = 1
    kn = torch.randn(R, H, 1, D, device="cuda", dtype=torch.float16, generator=g)
    NP = args.prefill_pages
    pre = np.zeros(NP, P.ITEM_DTYPE)
    pre["page"] = np.arange(NP) + (pages - NP)
    pre["src_t"] = np.arange(NP) * bs
    pre["n_rows"] = bs
    pre["from_zero"] = 1
    pk = torch.randn(1, H, NP * bs, D, device="cuda", dtype=torch.float16, generator=g)
    for _ in range(args.warmup):
        P.page_update(app, kn, kn, dk, dv)
        P.page_update(pre, pk, pk, dk, dv)
    torch.cuda.synchronize()
    if args.launch_only:  # no CUPTI session of our own: the case to run under ncu
        for _ in range(args.calls):
            P.page_update(app, kn, kn, dk, dv)
        for _ in range(args.calls):
            P.page_update(pre, pk, pk, dk, dv)
        torch.cuda.synchronize()
        return {"launch_only": True, "append_launches": args.calls, "prefill_launches": args.calls}
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.calls):
            P.page_update(app, kn, kn, dk, dv)
        torch.cuda.synchronize()
        for _ in range(args.calls):
            P.page_update(pre, pk, pk, dk, dv)
        torch.cuda.synchronize()
    ev = [e for e in prof.events() if e.device_type.name == "CUDA" and "page_update" in e.name]
    if len(ev) != 2 * args.calls:
        raise RuntimeError(f"expected {2 * args.calls} page-update launches, saw {len(ev)}")
    t_app = statistics.median(e.device_time for e in ev[: args.calls])
    t_pre = statistics.median(e.device_time for e in ev[args.calls:])
    unit = bs * D
    app_bytes = R * H * 2 * (2 * unit + 2 * 6 + D * 2)
    pre_bytes = NP * H * 2 * (unit * 2 + unit + 6)
    return {
        "kernel": ev[0].name,
        "heads": H, "head_dim": D, "block_size": bs,
        "append": {"pages": R, "us": t_app, "algorithmic_bytes": app_bytes, "GB_per_s": app_bytes / t_app / 1e3},
        "prefill": {"pages": NP, "us": t_pre, "algorithmic_bytes": pre_bytes, "GB_per_s": pre_bytes / t_pre / 1e3},
        "calls": args.calls,
    }


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--prefill-pages", type=int, default=4096)
    ap.add_argument("--pool-pages", type=int, default=8192)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--calls", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--launch-only", action="store_true", help="launch the calls without timing them (for ncu)")
    args = ap.parse_args(argv)
    res = run(args)
    if args.json or args.launch_only:
        print(json.dumps(res))
    else:
        for k in ("append", "prefill"):
            r = res[k]
            print(f"{k:8s} {r['pages']:6d} pages  {r['us']:9.1f} us  {r['GB_per_s']:8.1f} GB/s")
    return res


if __name__ == "__main__":
    main(sys.argv[1:])
