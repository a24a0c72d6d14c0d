"""Seeded synthetic workloads of the benchmark configurations, built on the GPU.

The reference benchmarks on seeded ``randn`` data (benchmarks/microbench.py:450-454);
these builders draw fp16 N(0,1) Q/K/V with a seeded torch generator on the device
and quantize K/V with the bit-exact CUDA quantizer into the reference cache formats.

    cfg0  contiguous INT8 KV: B8, H32, S2048, D128
    cfg1  paged: B16, H32, S4096, page 16, pool = 4096 pages + 10% slack, shuffled table
    cfg2  ragged GQA paged: B64, Hq32/Hkv8, lengths 8192 -> 128 linear, round-robin pages,
          4 splits
    cfg3  long context: B2, Hq64/Hkv8, S131072, shuffled table, sequence-sharded
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from .paged import PagedKVCache
from .quant import QuantizedTensor, quantize_int8_per_block

PAGE = 16
HEAD_DIM = 128


def algorithmic_bytes(batch: int, q_heads: int, kv_heads: int, lengths: Sequence[int], table_cols: int = 0,
                      page: int = PAGE, head_dim: int = HEAD_DIM, with_lengths: bool = True) -> int:
    """Bytes one decode call must move: for each referenced (page, kv head) the int8
    K and V blocks plus fp32 scale and int16 zero point of each; fp16 q and out; the
    int64 block table and lengths."""
    pages = sum((int(n) + page - 1) // page for n in lengths)
    kv = pages * kv_heads * 2 * (page * head_dim + 4 + 2)
    return kv + 2 * batch * q_heads * head_dim * 2 + batch * table_cols * 8 + (batch * 8 if with_lengths else 0)


@dataclass
class PagedWorkload:
    name: str
    q: torch.Tensor
    cache: PagedKVCache
    lengths: List[int]
    q_heads: int
    kv_heads: int
    num_splits: Optional[int]
    bytes_per_call: int


@dataclass
class FusedWorkload:
    name: str
    q: torch.Tensor
    k_quant: QuantizedTensor
    v_quant: QuantizedTensor
    lengths: Optional[torch.Tensor]
    bytes_per_call: int


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _quant_pool(pages: int, heads: int, gen: torch.Generator, device, chunk: int = 2048) -> QuantizedTensor:
    """Quantized pool [pages, heads, 1, 16, 128] of N(0,1) fp16 pages, built in chunks to
    bound the fp16 staging memory."""
    values = torch.empty((pages, heads, 1, PAGE, HEAD_DIM), dtype=torch.int8, device=device)
    scale = torch.empty((pages, heads, 1, 1, 1), dtype=torch.float32, device=device)
    zp = torch.empty((pages, heads, 1, 1, 1), dtype=torch.int16, device=device)
    for s in range(0, pages, chunk):
        e = min(pages, s + chunk)
        x = torch.randn((e - s, heads, PAGE, HEAD_DIM), generator=gen, device=device, dtype=torch.float16)
        qt = quantize_int8_per_block(x, PAGE)
        values[s:e], scale[s:e], zp[s:e] = qt.values, qt.scale, qt.zero_point
    return QuantizedTensor(values, scale, zp, PAGE, (pages, heads, PAGE, HEAD_DIM))


def paged_workload(name: str, batch: int, q_heads: int, kv_heads: int, lengths: Sequence[int], *,
                   slack: float = 0.10, layout: str = "shuffled", seed: int = 0, device="cuda",
                   num_splits: Optional[int] = None) -> PagedWorkload:
    """Pool of sum(pages) * (1 + slack) pages; table by ``layout``:
    shuffled = seeded random permutation of physical pages over the request-major
    logical pages; roundrobin = physical pages handed out one at a time to the
    requests that still need pages; contiguous = request-major order."""
    device = torch.device(device)
    gen = _gen(seed, device)
    need = [(int(n) + PAGE - 1) // PAGE for n in lengths]
    total = sum(need)
    pool_pages = int(math.ceil(total * (1.0 + slack)))
    cols = max(need)
    table = torch.full((batch, cols), -1, dtype=torch.int64)
    if layout == "shuffled":
        perm = torch.randperm(pool_pages, generator=_gen(seed + 1, "cpu"))[:total]
        pos = 0
        for b, n in enumerate(need):
            table[b, :n] = perm[pos:pos + n]
            pos += n
    elif layout == "roundrobin":
        nxt, filled = 0, [0] * batch
        while nxt < total:
            for b in range(batch):
                if filled[b] < need[b]:
                    table[b, filled[b]] = nxt
                    filled[b] += 1
                    nxt += 1
    elif layout == "contiguous":
        pos = 0
        for b, n in enumerate(need):
            table[b, :n] = torch.arange(pos, pos + n)
            pos += n
    else:
        raise ValueError(f"unknown layout {layout}")
    kq = _quant_pool(pool_pages, kv_heads, gen, device)
    vq = _quant_pool(pool_pages, kv_heads, gen, device)
    q = torch.randn((batch, q_heads, HEAD_DIM), generator=gen, device=device, dtype=torch.float16)
    lens_t = torch.tensor([int(n) for n in lengths], dtype=torch.int64, device=device)
    cache = PagedKVCache(kq, vq, table.to(device), lens_t, PAGE, int(max(lengths)))
    nbytes = algorithmic_bytes(batch, q_heads, kv_heads, lengths, table_cols=cols)
    return PagedWorkload(name, q, cache, [int(n) for n in lengths], q_heads, kv_heads, num_splits, nbytes)


def cfg1(seed: int = 0, device="cuda") -> PagedWorkload:
    return paged_workload("cfg1_paged_b16_h32_s4096_shuffled", 16, 32, 32, [4096] * 16, seed=seed, device=device)


def cfg2_lengths(batch: int = 64, hi: int = 8192, lo: int = 128) -> List[int]:
    """Lengths descending linearly from hi to lo across the batch (the 'descending'
    pattern of benchmarks/microbench.py:112-115 with explicit endpoints)."""
    return [int(round(hi - (hi - lo) * i / (batch - 1))) for i in range(batch)]


def cfg2(seed: int = 0, device="cuda") -> PagedWorkload:
    return paged_workload("cfg2_ragged_gqa_b64_32q8kv", 64, 32, 8, cfg2_lengths(), layout="roundrobin",
                          seed=seed, device=device, num_splits=4)


def cfg3(seed: int = 0, device="cuda", seq: int = 131072) -> PagedWorkload:
    return paged_workload("cfg3_long_b2_64q8kv_s131072", 2, 64, 8, [seq] * 2, seed=seed, device=device)


def cfg0(seed: int = 0, device="cuda") -> FusedWorkload:
    device = torch.device(device)
    gen = _gen(seed, device)
    b, h, s = 8, 32, 2048
    k = torch.randn((b, h, s, HEAD_DIM), generator=gen, device=device, dtype=torch.float16)
    kq = quantize_int8_per_block(k, PAGE)
    del k
    v = torch.randn((b, h, s, HEAD_DIM), generator=gen, device=device, dtype=torch.float16)
    vq = quantize_int8_per_block(v, PAGE)
    del v
    q = torch.randn((b, h, HEAD_DIM), generator=gen, device=device, dtype=torch.float16)
    return FusedWorkload("cfg0_fused_b8_h32_s2048", q, kq, vq, None, algorithmic_bytes(b, h, h, [s] * b))


def cfg3_shard(rank: int, world: int, seed: int = 0, device="cuda", seq: int = 131072) -> PagedWorkload:
    """Config 3 as seen by one rank of a sequence-sharded run: only the logical pages
    ``page_window(n_pages, rank, world)`` of each of the 2 requests are resident (in a
    local pool with 10% slack, shuffled); the block_table has the full width with -1
    outside the window.  q is identical on every rank.  ``bytes_per_call`` is the
    algorithmic size of the WHOLE call (all ranks together)."""
    from .dist import page_window

    device = torch.device(device)
    b, hq, hkv = 2, 64, 8
    n_pages = (seq + PAGE - 1) // PAGE
    lo, hi = page_window(n_pages, rank, world)
    local = (hi - lo) * b
    pool_pages = max(1, int(math.ceil(local * 1.10)))
    gen = _gen(seed + 7919 * (rank + 1), device)
    kq = _quant_pool(pool_pages, hkv, gen, device)
    vq = _quant_pool(pool_pages, hkv, gen, device)
    perm = torch.randperm(pool_pages, generator=_gen(seed + 31 * (rank + 1), "cpu"))[:local]
    table = torch.full((b, n_pages), -1, dtype=torch.int64)
    table[:, lo:hi] = perm.reshape(b, hi - lo)
    q = torch.randn((b, hq, HEAD_DIM), generator=_gen(seed, device), device=device, dtype=torch.float16)
    lens = torch.full((b,), seq, dtype=torch.int64, device=device)
    cache = PagedKVCache(kq, vq, table.to(device), lens, PAGE, seq)
    nbytes = algorithmic_bytes(b, hq, hkv, [seq] * b, table_cols=n_pages)
    return PagedWorkload(f"cfg3_long_b2_64q8kv_s{seq}_seqshard{world}", q, cache, [seq] * b, hq, hkv, None, nbytes)
