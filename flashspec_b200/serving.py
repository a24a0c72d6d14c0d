"""Allocator-driven decode serving loop (benchmark configuration 4) on the GPU.

Each step (the step order of the reference simulator, src/flashspec/serving.py:126-162,
with the token append placed before attention as the configuration specifies):

  1. admit waiting requests FIFO while fewer than ``max_live`` are live and the pool
     has pages: prefill = ``PagedKVAllocator.add_request`` (pages quantized on device);
  2. append one new fp16 K/V token per live request into its tail page
     (``append_batch``: one ``fs_page_update`` launch, bit-exact requantization);
  3. paged decode attention over the live batch (``to_cache`` -> ``cuda_paged``);
  4. requests that produced their output length are released (pages back to the
     lowest-first free list, never zeroed).

Arrivals are Poisson(rate) per step, prompt lengths U[prompt_min, prompt_max], output
lengths U[out_min, out_max]; everything is seeded.  The same schedule can be replayed
on the CPU oracle allocator (``schedule`` is pure host logic).
"""

from __future__ import annotations

import argparse
import json
import time
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch


@dataclass
class ServingConfig:
    steps: int = 2000
    arrival_rate: float = 8.0
    max_live: int = 256
    prompt_min: int = 128
    prompt_max: int = 4096
    out_min: int = 64
    out_max: int = 1024
    heads: int = 32
    head_dim: int = 128
    page: int = 16
    seed: int = 0
    capacity_pages: Optional[int] = None  # default: max_live * pages of the longest request

    def capacity(self) -> int:
        if self.capacity_pages:
            return int(self.capacity_pages)
        return self.max_live * ((self.prompt_max + self.out_max + self.page - 1) // self.page)


@dataclass
class Request:
    rid: int
    prompt: int
    out_len: int
    generated: int = 0


class Schedule:
    """Seeded arrivals and admission decisions (host only)."""

    def __init__(self, cfg: ServingConfig):
        self.cfg = cfg
        self.rng = np.random.default_rng(cfg.seed)
        self.queue: List[Request] = []
        self.next_id = 0

    def arrivals(self) -> None:
        for _ in range(int(self.rng.poisson(self.cfg.arrival_rate))):
            p = int(self.rng.integers(self.cfg.prompt_min, self.cfg.prompt_max + 1))
            o = int(self.rng.integers(self.cfg.out_min, self.cfg.out_max + 1))
            self.queue.append(Request(self.next_id, p, o))
            self.next_id += 1


def _pages(n: int, page: int) -> int:
    return (n + page - 1) // page


def run(cfg: ServingConfig, device="cuda", measure: bool = True, recorder: Optional[list] = None) -> Dict[str, float]:
    """Run the loop on ``device``; returns aggregate metrics.  With ``recorder`` (a list)
    every operation and its host-copied data is appended, so a test can replay the run
    on another allocator and compare."""
    import flashspec_b200 as fs
    from flashspec_b200.configs import algorithmic_bytes

    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(cfg.seed + 1)
    alloc = fs.PagedKVAllocator(capacity_blocks=cfg.capacity(), heads=cfg.heads, head_dim=cfg.head_dim,
                                block_size=cfg.page, device=device)
    sched = Schedule(cfg)
    live: Dict[int, Request] = {}
    committed = 0  # pages the live requests will hold at their full length
    t_attn = t_append = t_prefill = 0.0
    attn_bytes = append_bytes = 0
    tokens = finished = admitted = 0
    launches = 0  # this library's kernels: one page update per prefill, per append, one decode per step
    ev = lambda: torch.cuda.Event(enable_timing=True)
    step_times = []
    marks = []
    wall0 = time.perf_counter()
    for step in range(cfg.steps):
        s0 = ev()
        s0.record()
        # 1. arrivals + FIFO admission
        sched.arrivals()
        p0 = ev()
        p0.record()
        while sched.queue and len(live) < cfg.max_live:
            r = sched.queue[0]
            need = _pages(r.prompt + r.out_len, cfg.page)
            if committed + need > alloc.capacity_blocks:
                break
            sched.queue.pop(0)
            k = torch.randn((1, cfg.heads, r.prompt, cfg.head_dim), generator=gen, device=device, dtype=torch.float16)
            v = torch.randn((1, cfg.heads, r.prompt, cfg.head_dim), generator=gen, device=device, dtype=torch.float16)
            alloc.add_request(r.rid, k, v)
            launches += 1 if r.prompt > 0 else 0
            if recorder is not None:
                recorder.append(("add", r.rid, k.cpu().numpy(), v.cpu().numpy()))
            live[r.rid] = r
            committed += need
            admitted += 1
        p1 = ev()
        p1.record()
        if not live:
            continue
        ids = list(live.keys())
        b = len(ids)
        # 2. append one token per live request
        kn = torch.randn((b, cfg.heads, 1, cfg.head_dim), generator=gen, device=device, dtype=torch.float16)
        vn = torch.randn((b, cfg.heads, 1, cfg.head_dim), generator=gen, device=device, dtype=torch.float16)
        a0 = ev()
        a0.record()
        alloc.append_batch(ids, kn, vn)
        if recorder is not None:
            recorder.append(("append", list(ids), kn.cpu().numpy(), vn.cpu().numpy()))
        a1 = ev()
        a1.record()
        append_bytes += b * cfg.heads * 2 * (2 * cfg.page * cfg.head_dim + 2 * 6) + 2 * kn.numel() * 2
        # 3. attention
        q = torch.randn((b, cfg.heads, cfg.head_dim), generator=gen, device=device, dtype=torch.float16)
        cache = alloc.to_cache(ids)
        lens = [alloc._requests[i].length for i in ids]
        t0 = ev()
        t0.record()
        out = fs.paged_quant_attention_cuda(q, cache)
        t1 = ev()
        t1.record()
        attn_bytes += algorithmic_bytes(b, cfg.heads, cfg.heads, lens, table_cols=int(cache.block_table.shape[1]))
        tokens += b
        launches += 2
        if recorder is not None:
            recorder.append(("attn", list(ids), q.cpu().numpy(), out.cpu().numpy()))
        # 4. release finished requests
        for rid in ids:
            live[rid].generated += 1
            if live[rid].generated >= live[rid].out_len:
                alloc.release_request(rid)
                if recorder is not None:
                    recorder.append(("release", rid, None, None))
                committed -= _pages(live[rid].prompt + live[rid].out_len, cfg.page)
                del live[rid]
                finished += 1
        s1 = ev()
        s1.record()
        if measure:  # read after the loop: no host synchronisation inside it
            marks.append((s0, s1, p0, p1, a0, a1, t0, t1))
    torch.cuda.synchronize(device)
    for s0, s1, p0, p1, a0, a1, t0, t1 in marks:
        t_attn += t0.elapsed_time(t1)
        t_append += a0.elapsed_time(a1)
        t_prefill += p0.elapsed_time(p1)
        step_times.append(s0.elapsed_time(s1))
    wall = time.perf_counter() - wall0
    if recorder is not None:
        recorder.append(("final", alloc, None, None))
    st = alloc.stats()
    res = {
        "steps": cfg.steps, "decode_tokens": tokens, "admitted": admitted, "finished": finished,
        "waiting_at_end": len(sched.queue), "live_at_end": len(live), "wall_s": wall,
        "tokens_per_s_wall": tokens / wall,
        "allocated_blocks": st["allocated_blocks"], "free_blocks": st["free_blocks"],
        "block_utilization": st["block_utilization"], "fragmentation": st["fragmentation"],
    }
    if measure and step_times:
        res.update({
            "step_ms_median": float(np.median(step_times)), "step_ms_mean": float(np.mean(step_times)),
            "attention_ms_total": t_attn, "append_ms_total": t_append, "prefill_ms_total": t_prefill,
            "attention_tbps": attn_bytes / (t_attn * 1e-3) / 1e12 if t_attn else None,
            "append_tbps": append_bytes / (t_append * 1e-3) / 1e12 if t_append else None,
            "attention_bytes": attn_bytes, "append_bytes": append_bytes,
            "tokens_per_s_device": tokens / (sum(step_times) * 1e-3),
            "steps_measured": len(step_times), "gpu_launches": launches,
        })
    return res


def main(argv=None):
    ap = argparse.ArgumentParser(description="cfg4 allocator-driven serving decode loop")
    for f_name, f_def in asdict(ServingConfig()).items():
        ap.add_argument("--" + f_name.replace("_", "-"), type=type(f_def) if f_def is not None else int,
                        default=f_def)
    args = ap.parse_args(argv)
    cfg = ServingConfig(**{k: getattr(args, k) for k in asdict(ServingConfig())})
    print(json.dumps({"config": asdict(cfg), **run(cfg)}))


if __name__ == "__main__":
    main()
