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
        admitted_before = admitted
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
            marks.append((s0, s1, p0, p1, a0, a1, t0, t1, admitted - admitted_before))
    torch.cuda.synchronize(device)
    ttft_sum, ttft_n = 0.0, 0
    for s0, s1, p0, p1, a0, a1, t0, t1, n_adm in marks:
        if n_adm:  # a request admitted in this step gets its first token at the step's attention
            ttft_sum += n_adm * p0.elapsed_time(t1)
            ttft_n += n_adm
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
            "ttft_ms_mean": ttft_sum / max(1, ttft_n), "tpot_ms": float(np.mean(step_times)),
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


# ------------------------------------------------------------------------------------
# The reference's serving simulation API on the GPU allocator
# ------------------------------------------------------------------------------------


@dataclass(frozen=True)
class SimulationConfig:
    """The fields and defaults of the reference's serving ``ServingConfig``
    (src/flashspec/serving.py:15-30); device is a CUDA device here."""

    requests: int = 8
    prompt_len: int = 128
    prompt_lens: Optional[tuple] = None
    prompt_length_distribution: str = "uniform"
    decode_steps: int = 16
    request_life_steps: int = 0
    heads: int = 8
    head_dim: int = 64
    block_size: int = 16
    allocator_blocks: Optional[int] = None
    seed: int = 0
    device: str = "cuda"
    dtype: str = "auto"


def _sim_dtype(name: str) -> torch.dtype:
    n = name.strip().lower()
    if n in ("auto", "float16", "fp16"):
        return torch.float16
    if n in ("bfloat16", "bf16"):
        return torch.bfloat16
    raise ValueError("dtype must be auto, float16 or bfloat16 (the CUDA decode takes fp16 / bf16 q)")


def run_decode_simulation(config: SimulationConfig) -> Dict[str, object]:
    """The reference's deterministic serving simulation (src/flashspec/serving.py:33-190)
    with the same steps, prompt-length sampling, allocator sizing and result keys, on
    this package's device allocator and CUDA decode: prefill of ``requests`` requests, the
    first decode attention (TTFT = prefill + first attention), then ``decode_steps``
    steps of attention + append of one token per request (K = out, V = tanh(out), as the
    reference derives them), with optional finish / arrival every ``request_life_steps``.
    Times are host wall clock around synchronised regions, as in the reference."""
    import flashspec_b200 as fs

    if config.requests <= 0 or config.prompt_len <= 0:
        raise ValueError("requests and prompt_len must be positive")
    if config.decode_steps < 0 or config.request_life_steps < 0:
        raise ValueError("decode_steps and request_life_steps must not be negative")
    if config.heads <= 0 or config.head_dim <= 0 or config.block_size <= 0:
        raise ValueError("heads, head_dim and block_size must be positive")
    device = torch.device(config.device)
    if device.type != "cuda":
        raise RuntimeError("the simulation runs on a CUDA device")
    dtype = _sim_dtype(config.dtype)
    gen = torch.Generator(device=device).manual_seed(config.seed)
    lens = tuple(int(x) for x in (config.prompt_lens if config.prompt_lens is not None else (config.prompt_len,)))
    if not lens or any(x <= 0 for x in lens):
        raise ValueError("prompt_lens must be positive")
    if config.allocator_blocks is not None:
        capacity = int(config.allocator_blocks)
    else:
        per_live = max(lens) + max(1, config.decode_steps)
        capacity = max(1, config.requests * ((per_live + config.block_size - 1) // config.block_size))
    alloc = fs.PagedKVAllocator(capacity_blocks=capacity, heads=config.heads, head_dim=config.head_dim,
                                block_size=config.block_size, device=device)
    mode = config.prompt_length_distribution.strip().lower()
    if mode not in ("uniform", "cycle", "random", "bimodal"):
        raise ValueError("prompt_length_distribution must be uniform, random or bimodal")

    def sample_len(i: int) -> int:
        if mode in ("uniform", "cycle"):
            return lens[i % len(lens)]
        if mode == "random":
            return lens[int(torch.randint(len(lens), (1,), generator=gen, device=device).item())]
        return lens[0] if (len(lens) == 1 or i % 2 == 0) else lens[-1]

    state = {"next": 0, "prefill_ms": 0.0, "arrival_prefill_ms": 0.0, "arrivals": 0}
    active: List[int] = []
    generated: Dict[int, int] = {}
    prompt_of: Dict[int, int] = {}

    def add(initial: bool) -> int:
        rid = state["next"]
        state["next"] += 1
        n = sample_len(rid)
        k = torch.randn((1, config.heads, n, config.head_dim), generator=gen, device=device, dtype=dtype)
        v = torch.randn((1, config.heads, n, config.head_dim), generator=gen, device=device, dtype=dtype)
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        alloc.add_request(rid, k, v)
        torch.cuda.synchronize(device)
        state["prefill_ms" if initial else "arrival_prefill_ms"] += (time.perf_counter() - t0) * 1e3
        state["arrivals"] += 1
        generated[rid] = 0
        prompt_of[rid] = n
        return rid

    for _ in range(config.requests):
        active.append(add(True))
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    q = torch.randn((len(active), config.heads, config.head_dim), generator=gen, device=device, dtype=dtype)
    fs.paged_quant_attention_cuda(q, alloc.to_cache(active))
    torch.cuda.synchronize(device)
    first_ms = (time.perf_counter() - t0) * 1e3
    decode_ms, tokens, finishes = 0.0, 0, 0
    for _ in range(config.decode_steps):
        if not active:
            break
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        q = torch.randn((len(active), config.heads, config.head_dim), generator=gen, device=device, dtype=dtype)
        out = fs.paged_quant_attention_cuda(q, alloc.to_cache(active))
        alloc.append_batch(active, out.unsqueeze(2).to(dtype), torch.tanh(out).unsqueeze(2).to(dtype))
        torch.cuda.synchronize(device)
        decode_ms += (time.perf_counter() - t0) * 1e3
        for rid in active:
            generated[rid] += 1
        tokens += len(active)
        if config.request_life_steps > 0:
            done = [rid for rid in active if generated[rid] >= config.request_life_steps]
            for rid in done:
                alloc.release_request(rid)
                active.remove(rid)
                generated.pop(rid, None)
                finishes += 1
            for _ in done:
                active.append(add(False))
    st = alloc.stats()
    return {
        "device": str(device), "device_name": torch.cuda.get_device_name(device),
        "dtype": str(dtype).replace("torch.", ""), "requests": config.requests, "prompt_len": config.prompt_len,
        "prompt_lens": list(lens), "prompt_length_distribution": config.prompt_length_distribution,
        "average_prompt_len": sum(prompt_of.values()) / max(1, len(prompt_of)),
        "decode_steps": config.decode_steps, "request_life_steps": config.request_life_steps,
        "arrivals": state["arrivals"], "finishes": finishes, "prefill_ms": state["prefill_ms"],
        "arrival_prefill_ms": state["arrival_prefill_ms"],
        "total_prefill_ms": state["prefill_ms"] + state["arrival_prefill_ms"], "first_attention_ms": first_ms,
        "decode_ms": decode_ms, "ttft_ms": state["prefill_ms"] + first_ms,
        "tpot_ms": decode_ms / max(1, config.decode_steps),
        "tokens_per_second": tokens / max(1.0e-9, decode_ms / 1000.0), "generated_tokens": tokens, **st,
    }
