"""CPU reference arm of the decode-attention path (TEST AND MEASUREMENT INFRASTRUCTURE).

A restatement, in torch on the CPU, of the reference FlashSpec CPU backends that the
CUDA library replaces -- the same torch operations in the same order, so the timed
CPU path does the work the reference's own ``fused`` / ``paged`` backends do on the
host (the reference package itself is not importable on the measurement box):

* quantize_int8_per_block      src/flashspec/quant.py:69-165
* dequantize_int8_per_block    src/flashspec/quant.py:168-204
* reference_attention          src/flashspec/attention.py:70-121
* fused_dequant_attention      src/flashspec/attention.py:124-168
* PagedKVCache.to_dense        src/flashspec/paged.py:421-461
* paged_quant_attention        src/flashspec/attention.py:171-223
  (GQA, which the reference does not have, as G calls on q[:, g::G]; each call
  materialises the dense cache again, as G calls of the reference would)

plus host-side builders of the benchmark configurations (seeded CPU generator, fp16
N(0,1) data, the restated quantizer), so that ``bench.py --impl reference`` and the
CPU baseline never touch the GPU or the CUDA library.  Only ``tests/`` and
``bench.py``'s reference / CPU-baseline legs use this module; it is pinned against the
golden vectors recorded from the reference (``tests/test_torch_reference.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

PAGE = 16
HEAD_DIM = 128


@dataclass
class TQuant:
    """Fields of the reference QuantizedTensor (quant.py:9-43)."""

    values: torch.Tensor
    scale: torch.Tensor
    zero_point: torch.Tensor
    block_size: int
    original_shape: Tuple[int, ...]


@dataclass
class TPagedCache:
    """Fields of the reference PagedKVCache (paged.py:258-300)."""

    k_quant: TQuant
    v_quant: TQuant
    block_table: torch.Tensor
    lengths: torch.Tensor
    block_size: int
    max_seq_len: int


def quantize_int8_per_block(x: torch.Tensor, block_size: int = PAGE) -> TQuant:
    """quant.py:94-165: zero-pad the sequence axis to a block multiple, then per
    [block_size, D] block scale = max((max - min) / 255, 1e-8), zp = clamp(round(-min /
    scale), 0, 255), u = clamp(round(x / scale + zp), 0, 255), stored as u - 128."""
    shape = tuple(x.shape)
    xf = x.detach().to(torch.float32)
    pad = (block_size - xf.shape[-2] % block_size) % block_size
    if pad:
        xf = torch.cat([xf, xf.new_zeros((*xf.shape[:-2], pad, xf.shape[-1]))], dim=-2)
    blocks = xf.reshape(*xf.shape[:-2], xf.shape[-2] // block_size, block_size, xf.shape[-1])
    lo = blocks.amin(dim=(-2, -1), keepdim=True)
    hi = blocks.amax(dim=(-2, -1), keepdim=True)
    scale = ((hi - lo) / 255.0).clamp_min(1.0e-8)
    zp = torch.round(-lo / scale).clamp(0, 255)
    u = torch.round(blocks / scale + zp).clamp(0, 255)
    return TQuant((u.to(torch.int16) - 128).to(torch.int8), scale, zp.to(torch.int16), block_size, shape)


def dequantize_int8_per_block(q: TQuant) -> torch.Tensor:
    """quant.py:168-204: (float(v + 128) - float(zp)) * scale, back to the original
    sequence length, fp32."""
    u = q.values.to(torch.int16) + 128
    x = (u.to(torch.float32) - q.zero_point.to(torch.float32)) * q.scale.to(torch.float32)
    lead, seq, d = q.original_shape[:-2], q.original_shape[-2], q.original_shape[-1]
    return x.reshape(*lead, -1, d)[..., :seq, :]


def reference_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """attention.py:70-121: fp32 scores q.k * 1/sqrt(D), positions >= length set to the
    fp32 minimum, softmax, fp32 probs.v, cast to q's dtype.  MHA shapes."""
    scores = torch.einsum("bhd,bhsd->bhs", q.to(torch.float32), k.to(torch.float32)) * (1.0 / math.sqrt(q.shape[-1]))
    if lengths is not None:
        mask = torch.arange(k.shape[-2]).unsqueeze(0) >= lengths.unsqueeze(1)
        scores = scores.masked_fill(mask[:, None, :], torch.finfo(scores.dtype).min)
    probs = torch.softmax(scores, dim=-1)
    return torch.einsum("bhs,bhsd->bhd", probs, v.to(torch.float32)).to(q.dtype)


def _per_group(q: torch.Tensor, kv_heads: int, call) -> torch.Tensor:
    """Run ``call(q_g)`` on q[:, g::G] for each g and interleave the results (GQA as
    G MHA calls: q head h reads kv head h // G)."""
    groups = q.shape[1] // kv_heads
    if groups == 1:
        return call(q)
    out = torch.empty_like(q)
    for g in range(groups):
        out[:, g::groups] = call(q[:, g::groups].contiguous())
    return out


def fused_dequant_attention(q: torch.Tensor, kq: TQuant, vq: TQuant,
                            lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """attention.py:124-168: dequantize K and V, then reference_attention."""

    def call(qg):
        return reference_attention(qg, dequantize_int8_per_block(kq), dequantize_int8_per_block(vq), lengths)

    return _per_group(q, int(kq.original_shape[1]), call)


def paged_to_dense(cache: TPagedCache) -> Tuple[torch.Tensor, torch.Tensor]:
    """paged.py:421-461: dequantize the whole pool, gather pages by
    table.clamp_min(0), lay out as [B, H, S, D], keep max_seq_len tokens."""
    b = cache.block_table.shape[0]
    h, d = int(cache.k_quant.original_shape[1]), int(cache.k_quant.original_shape[-1])
    table = cache.block_table.clamp_min(0)

    def dense(qt):
        g = dequantize_int8_per_block(qt)[table]  # [B, cols, H, block, D]
        return g.permute(0, 2, 1, 3, 4).contiguous().reshape(b, h, -1, d)[..., : cache.max_seq_len, :]

    return dense(cache.k_quant), dense(cache.v_quant)


def paged_quant_attention(q: torch.Tensor, cache: TPagedCache) -> torch.Tensor:
    """attention.py:171-223: to_dense, then reference_attention masked by lengths."""

    def call(qg):
        k, v = paged_to_dense(cache)
        return reference_attention(qg, k, v, cache.lengths)

    return _per_group(q, int(cache.k_quant.original_shape[1]), call)


# ------------------------------------------------------------------------------------
# host-side benchmark configurations (same shapes and distributions as the GPU builders)
# ------------------------------------------------------------------------------------


def algorithmic_bytes(batch: int, q_heads: int, kv_heads: int, lengths: Sequence[int], table_cols: int = 0,
                      with_lengths: bool = True) -> int:
    """Bytes one decode call must move: int8 K and V plus fp32 scale and int16 zero
    point per referenced (page, kv head), fp16 q and out, the int64 table and lengths."""
    pages = sum((int(n) + PAGE - 1) // PAGE for n in lengths)
    kv = pages * kv_heads * 2 * (PAGE * HEAD_DIM + 4 + 2)
    return kv + 2 * batch * q_heads * HEAD_DIM * 2 + batch * table_cols * 8 + (batch * 8 if with_lengths else 0)


@dataclass
class HostWorkload:
    name: str
    kind: str  # "paged" or "fused"
    q: torch.Tensor
    cache: Optional[TPagedCache]
    k_quant: Optional[TQuant]
    v_quant: Optional[TQuant]
    lengths: List[int]
    bytes_per_call: int

    def call(self) -> torch.Tensor:
        if self.kind == "paged":
            return paged_quant_attention(self.q, self.cache)
        return fused_dequant_attention(self.q, self.k_quant, self.v_quant)


def _quant_pool(pages: int, heads: int, gen: torch.Generator, chunk: int = 1024) -> TQuant:
    values = torch.empty((pages, heads, 1, PAGE, HEAD_DIM), dtype=torch.int8)
    scale = torch.empty((pages, heads, 1, 1, 1), dtype=torch.float32)
    zp = torch.empty((pages, heads, 1, 1, 1), dtype=torch.int16)
    for s in range(0, pages, chunk):
        e = min(pages, s + chunk)
        qt = quantize_int8_per_block(torch.randn((e - s, heads, PAGE, HEAD_DIM), generator=gen, dtype=torch.float16))
        values[s:e], scale[s:e], zp[s:e] = qt.values, qt.scale, qt.zero_point
    return TQuant(values, scale, zp, PAGE, (pages, heads, PAGE, HEAD_DIM))


def paged_host_workload(name: str, batch: int, q_heads: int, kv_heads: int, lengths: Sequence[int], *,
                        layout: str = "shuffled", slack: float = 0.10, seed: int = 0) -> HostWorkload:
    """Pool of ceil(pages * (1 + slack)) pages; table shuffled (seeded permutation of the
    pool over the request-major logical pages) or round-robin (one page at a time to
    each request that still needs pages)."""
    gen = torch.Generator().manual_seed(seed)
    need = [(int(n) + PAGE - 1) // PAGE for n in lengths]
    total = sum(need)
    pool = int(math.ceil(total * (1.0 + slack)))
    table = torch.full((batch, max(need)), -1, dtype=torch.int64)
    if layout == "shuffled":
        perm = torch.randperm(pool, generator=torch.Generator().manual_seed(seed + 1))[:total]
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
    else:
        raise ValueError(f"unknown layout {layout}")
    kq = _quant_pool(pool, kv_heads, gen)
    vq = _quant_pool(pool, kv_heads, gen)
    q = torch.randn((batch, q_heads, HEAD_DIM), generator=gen, dtype=torch.float16)
    cache = TPagedCache(kq, vq, table, torch.tensor([int(n) for n in lengths], dtype=torch.int64), PAGE,
                        int(max(lengths)))
    return HostWorkload(name, "paged", q, cache, None, None, [int(n) for n in lengths],
                        algorithmic_bytes(batch, q_heads, kv_heads, lengths, table_cols=max(need)))


def cfg2_lengths(batch: int = 64, hi: int = 8192, lo: int = 128) -> List[int]:
    return [int(round(hi - (hi - lo) * i / (batch - 1))) for i in range(batch)]


def host_workload(config: str, seed: int = 0) -> HostWorkload:
    """The named benchmark configuration, built on the host."""
    if config == "cfg0":
        gen = torch.Generator().manual_seed(seed)
        b, h, s = 8, 32, 2048
        kq = quantize_int8_per_block(torch.randn((b, h, s, HEAD_DIM), generator=gen, dtype=torch.float16))
        vq = quantize_int8_per_block(torch.randn((b, h, s, HEAD_DIM), generator=gen, dtype=torch.float16))
        q = torch.randn((b, h, HEAD_DIM), generator=gen, dtype=torch.float16)
        return HostWorkload("cfg0_fused_b8_h32_s2048", "fused", q, None, kq, vq, [s] * b,
                            algorithmic_bytes(b, h, h, [s] * b, with_lengths=False))
    if config == "cfg1":
        return paged_host_workload("cfg1_paged_b16_h32_s4096_shuffled", 16, 32, 32, [4096] * 16, seed=seed)
    if config == "cfg2":
        return paged_host_workload("cfg2_ragged_gqa_b64_32q8kv", 64, 32, 8, cfg2_lengths(), layout="roundrobin",
                                   seed=seed)
    if config == "cfg3":
        return paged_host_workload("cfg3_long_b2_64q8kv_s131072", 2, 64, 8, [131072] * 2, seed=seed)
    raise ValueError(f"no host builder for {config}")


# ------------------------------------------------------------------------------------
# allocator and serving loop (configuration 4) at reduced scale
# ------------------------------------------------------------------------------------


class TAllocator:
    """The reference PagedKVAllocator (paged.py:17-255) restated in torch on the CPU: a
    pool of quantized zero pages, an ascending free list taken from the front
    (paged.py:221-224), release = extend + sort (paged.py:146-151), prefill page by page
    from zero-padded blocks (paged.py:66-106) and appends that dequantize the touched
    page, insert the rows and requantize it (paged.py:108-136, 226-255)."""

    def __init__(self, capacity_blocks: int, heads: int, head_dim: int = HEAD_DIM, block_size: int = PAGE):
        self.capacity_blocks, self.heads, self.head_dim, self.block_size = capacity_blocks, heads, head_dim, block_size
        zeros = torch.zeros((capacity_blocks, heads, block_size, head_dim), dtype=torch.float32)
        self.k_quant = quantize_int8_per_block(zeros, block_size)
        self.v_quant = quantize_int8_per_block(zeros, block_size)
        self.free_blocks: List[int] = list(range(capacity_blocks))
        self.requests = {}  # id -> [pages, length]

    def _allocate(self) -> int:
        if not self.free_blocks:
            raise RuntimeError("out of pages")
        return self.free_blocks.pop(0)

    def _page(self, p: int):
        def one(qt):
            u = qt.values[p : p + 1].to(torch.int16) + 128
            x = (u.to(torch.float32) - qt.zero_point[p : p + 1].to(torch.float32)) * qt.scale[p : p + 1]
            return x.reshape(1, self.heads, self.block_size, self.head_dim).clone()

        return one(self.k_quant), one(self.v_quant)

    def _write(self, p: int, kb: torch.Tensor, vb: torch.Tensor) -> None:
        for qt, blk in ((self.k_quant, kb), (self.v_quant, vb)):
            nq = quantize_int8_per_block(blk, self.block_size)
            qt.values[p : p + 1] = nq.values
            qt.scale[p : p + 1] = nq.scale
            qt.zero_point[p : p + 1] = nq.zero_point

    def add_request(self, rid: int, k: torch.Tensor, v: torch.Tensor) -> None:
        n = int(k.shape[2])
        pages = []
        for lb in range((n + self.block_size - 1) // self.block_size):
            p = self._allocate()
            pages.append(p)
            s0, s1 = lb * self.block_size, min((lb + 1) * self.block_size, n)
            kb = torch.zeros((1, self.heads, self.block_size, self.head_dim))
            vb = torch.zeros_like(kb)
            kb[:, :, : s1 - s0] = k[:, :, s0:s1].to(torch.float32)
            vb[:, :, : s1 - s0] = v[:, :, s0:s1].to(torch.float32)
            self._write(p, kb, vb)
        self.requests[rid] = [pages, n]

    def append_batch(self, rids: Sequence[int], k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        for i, rid in enumerate(rids):
            pages, n = self.requests[rid]
            touched = {}
            for t in range(int(k_new.shape[2])):
                lb, off = divmod(n + t, self.block_size)
                if lb == len(pages):
                    pages.append(self._allocate())
                p = pages[lb]
                if p not in touched:
                    touched[p] = self._page(p)
                touched[p][0][:, :, off] = k_new[i : i + 1, :, t].to(torch.float32)
                touched[p][1][:, :, off] = v_new[i : i + 1, :, t].to(torch.float32)
            for p, (kb, vb) in touched.items():
                self._write(p, kb, vb)
            self.requests[rid][1] = n + int(k_new.shape[2])

    def release_request(self, rid: int) -> None:
        pages, _ = self.requests.pop(rid)
        self.free_blocks.extend(pages)
        self.free_blocks.sort()

    def to_cache(self, rids: Sequence[int]) -> TPagedCache:
        cols = max(1, max(len(self.requests[r][0]) for r in rids))
        table = torch.full((len(rids), cols), -1, dtype=torch.int64)
        lengths = torch.empty((len(rids),), dtype=torch.int64)
        for i, r in enumerate(rids):
            pages, n = self.requests[r]
            table[i, : len(pages)] = torch.tensor(pages, dtype=torch.int64)
            lengths[i] = n
        return TPagedCache(self.k_quant, self.v_quant, table, lengths, self.block_size, int(lengths.max()))


@dataclass
class ServingParams:
    """Configuration 4 scaled down for the CPU: the step logic and distributions are
    those of the GPU loop (Poisson arrivals, prompt U[128, 4096], output U[64, 1024],
    32 heads), with fewer live requests and steps, because every decode step of the
    reference dequantizes the allocator's whole pool."""

    steps: int = 30
    arrival_rate: float = 8.0
    max_live: int = 16
    prompt_min: int = 128
    prompt_max: int = 4096
    out_min: int = 64
    out_max: int = 1024
    heads: int = 32
    seed: int = 0


def serving_loop(sp: ServingParams):
    """The decode loop of configuration 4 on TAllocator: arrivals + FIFO admission
    (prefill), append one token per live request, paged attention over the live batch,
    release finished requests.  Times the whole loop (prefill included) and counts the
    same algorithmic bytes the GPU loop reports (attention + append)."""
    import time

    import numpy as np

    rng = np.random.default_rng(sp.seed)
    gen = torch.Generator().manual_seed(sp.seed + 1)
    cap = sp.max_live * ((sp.prompt_max + sp.out_max + PAGE - 1) // PAGE)
    alloc = TAllocator(cap, sp.heads)
    queue, live, nxt = [], {}, 0
    committed = attn_bytes = append_bytes = tokens = 0
    t0 = time.perf_counter()
    for _ in range(sp.steps):
        for _ in range(int(rng.poisson(sp.arrival_rate))):
            queue.append([nxt, int(rng.integers(sp.prompt_min, sp.prompt_max + 1)),
                          int(rng.integers(sp.out_min, sp.out_max + 1)), 0])
            nxt += 1
        while queue and len(live) < sp.max_live:
            rid, p, o, _ = queue[0]
            need = (p + o + PAGE - 1) // PAGE
            if committed + need > cap:
                break
            queue.pop(0)
            k = torch.randn((1, sp.heads, p, HEAD_DIM), generator=gen, dtype=torch.float16)
            v = torch.randn((1, sp.heads, p, HEAD_DIM), generator=gen, dtype=torch.float16)
            alloc.add_request(rid, k, v)
            live[rid] = [rid, p, o, 0]
            committed += need
        if not live:
            continue
        ids = list(live.keys())
        b = len(ids)
        kn = torch.randn((b, sp.heads, 1, HEAD_DIM), generator=gen, dtype=torch.float16)
        vn = torch.randn((b, sp.heads, 1, HEAD_DIM), generator=gen, dtype=torch.float16)
        alloc.append_batch(ids, kn, vn)
        append_bytes += b * sp.heads * 2 * (2 * PAGE * HEAD_DIM + 2 * 6) + 2 * kn.numel() * 2
        q = torch.randn((b, sp.heads, HEAD_DIM), generator=gen, dtype=torch.float16)
        cache = alloc.to_cache(ids)
        paged_quant_attention(q, cache)
        attn_bytes += algorithmic_bytes(b, sp.heads, sp.heads, cache.lengths.tolist(),
                                        table_cols=int(cache.block_table.shape[1]))
        tokens += b
        for rid in ids:
            live[rid][3] += 1
            if live[rid][3] >= live[rid][2]:
                alloc.release_request(rid)
                committed -= (live[rid][1] + live[rid][2] + PAGE - 1) // PAGE
                del live[rid]
    loop_s = time.perf_counter() - t0
    return {"steps": sp.steps, "loop_s": loop_s, "decode_tokens": tokens, "tokens_per_s": tokens / loop_s,
            "bytes_moved": attn_bytes + append_bytes, "attention_bytes": attn_bytes, "append_bytes": append_bytes,
            "capacity_pages": cap, "params": {k: getattr(sp, k) for k in sp.__dataclass_fields__}}
