"""Per-phase timeline of the split decode kernel on one rank's window of the long-context
configuration (B2, 64 q / 8 kv heads, 131072 tokens split into ``--ranks`` page windows,
the window of rank 0 decoded on this GPU).

    python -m flashspec_b200.harness.split_timeline --ranks 8 --json

The library's profiling switch ``FLASHSPEC_TRACE_PTR`` (the device address of a zeroed
int64 buffer) makes the split kernel stamp %globaltimer at fixed points: per CTA its
entry, the end of its page stream and the write of its partial; per (request, kv head)
pair the last CTA's merge: start, partial LSEs loaded, weights formed, each staging
round of partial rows arrived and summed, and the end.  The calls are launched back to
back (one untraced call ahead of them), so the gap from one call's last stamp to the
next call's first entry is the launch interval.  Times are microseconds from the first
CTA entry of the first traced call; per-call device time (CUDA events over 300 calls)
is reported beside them.
"""

from __future__ import annotations

import argparse
import json
import os

import numpy as np
import torch


def _phases(buf: np.ndarray, ctas: int, pairs: int, t0: int) -> dict:
    c = buf[:4 * ctas].reshape(ctas, 4)
    q = buf[4 * ctas:4 * ctas + 16 * pairs].reshape(pairs, 16)
    us = lambda x: round((int(x) - t0) / 1e3, 2)  # noqa: E731
    last = int(np.argmax(q[:, 4]))
    rel = lambda x: round((int(x) - int(q[last, 0])) / 1e3, 2) if x > 0 else None  # noqa: E731
    return {
        "cta_entry_first_last": [us(c[:, 0].min()), us(c[:, 0].max())],
        "stream_done_first_median_last": [us(c[:, 1].min()), us(np.median(c[:, 1])), us(c[:, 1].max())],
        "partials_written_last": us(c[:, 2].max()),
        "end_last": us(q[:, 4].max()),
        "last_pair_merge_from_its_start": {
            "lse_loaded": rel(q[last, 5]), "weights": rel(q[last, 6]),
            "round0_arrived": rel(q[last, 8]), "round0_summed": rel(q[last, 9]),
            "round1_arrived": rel(q[last, 10]), "round1_summed": rel(q[last, 11]),
            "rows_summed": rel(q[last, 7]), "end": rel(q[last, 4])},
    }


def run(args) -> dict:
    import flashspec_b200 as fs
    from flashspec_b200 import configs
    from flashspec_b200.dist import page_window

    dev = torch.device("cuda", 0)
    wl = configs.cfg3_shard(0, args.ranks)
    n_pages = int(wl.cache.block_table.shape[1])
    win = page_window(n_pages, 0, args.ranks)
    o = torch.empty(wl.q.shape, dtype=torch.float32, device=dev)
    lse = torch.empty(wl.q.shape[:2], dtype=torch.float32, device=dev)

    def call():
        return fs.paged_quant_attention_cuda(wl.q, wl.cache, page_range=win, partial_out=(o, lse),
                                             return_stats=True)

    splits = call()[1]["num_splits"]
    pairs = int(wl.q.shape[0]) * wl.kv_heads
    ctas = pairs * int(splits)
    for _ in range(50):
        call()
    torch.cuda.synchronize()
    times = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(300):
            fs.paged_quant_attention_cuda(wl.q, wl.cache, page_range=win, partial_out=(o, lse))
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) / 300 * 1e3)
    bufs = [torch.zeros(4 * ctas + 16 * pairs, dtype=torch.int64, device=dev) for _ in range(args.calls)]
    torch.cuda.synchronize()
    call()
    try:
        for bf in bufs:
            os.environ["FLASHSPEC_TRACE_PTR"] = str(bf.data_ptr())
            fs.paged_quant_attention_cuda(wl.q, wl.cache, page_range=win, partial_out=(o, lse))
    finally:
        os.environ.pop("FLASHSPEC_TRACE_PTR", None)
    torch.cuda.synchronize()
    host = [bf.cpu().numpy().astype(np.int64) for bf in bufs]
    t0 = int(host[0][:4 * ctas:4].min())
    return {"workload": wl.name, "window_pages": list(win), "splits": int(splits), "ctas": ctas,
            "us_per_call_sorted": sorted(round(t, 2) for t in times),
            "calls": [_phases(h, ctas, pairs, t0) for h in host]}


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ranks", type=int, default=8)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args()
    res = run(args)
    print(json.dumps(res) if args.json else json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
