"""CPU oracle for the INT8 decode-attention hot path (TEST INFRASTRUCTURE ONLY).

This module is a plain-numpy restatement of the reference FlashSpec algorithms
that the CUDA library replaces.  It is the checker, never the product: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it.  The shipped package (``flashspec_b200``) must never route through it.

Parity is pinned: ``tests/golden/*.npz`` were produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference package and records its
outputs), and ``tests/test_oracle_golden.py`` checks every function here against
those vectors (bit-exact for the quantizer / allocator, fp16-ulp level for
attention).

Every function cites the reference file:line (paths inside the FlashSpec
project) whose behaviour it restates.

Conventions (same as the reference):
* quantized values are int8 = uint8 - 128; scale fp32; zero_point int16 in the
  uint8 domain; one (scale, zero_point) per [block_size, head_dim] block.
* sequence is axis -2, feature (head_dim) is axis -1.
* GQA (an extension; the reference is MHA only): q head h reads kv head
  h // (Hq // Hkv), equivalent to ``repeat_interleave`` of the KV heads.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

F32 = np.float32
_SCALE_FLOOR = F32(1.0e-8)  # quant.py:146 clamp_min(1e-8) evaluated in fp32
_F32_MIN = np.finfo(np.float32).min  # attention.py:112 masked_fill value


# ---------------------------------------------------------------------------
# quantizer -- src/flashspec/quant.py
# ---------------------------------------------------------------------------


@dataclass
class OQuant:
    """Mirror of ``QuantizedTensor`` (quant.py:9-43) holding numpy arrays."""

    values: np.ndarray  # int8 [..., n_blocks, block_size, D]
    scale: np.ndarray  # fp32 [..., n_blocks, 1, 1]
    zero_point: np.ndarray  # int16 [..., n_blocks, 1, 1]
    block_size: int
    original_shape: Tuple[int, ...]


def quantize_int8_per_block(x: np.ndarray, block_size: int = 16) -> OQuant:
    """quant.py:94-165.  Zero-pad seq to a block multiple (quant.py:69-91), then per
    [block_size, D] block: min/max, scale=max((max-min)/255, 1e-8),
    zp=clamp(rint(-min/scale),0,255), q=clamp(rint(x/scale + zp),0,255) - 128.
    Every step is a separate fp32 operation with round-to-nearest-even, exactly
    as torch evaluates the reference expression."""
    if x.ndim < 2:
        raise ValueError("need sequence and feature dims")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    original_shape = tuple(x.shape)
    xf = np.asarray(x, dtype=F32)
    seq = xf.shape[-2]
    pad = (block_size - seq % block_size) % block_size
    if pad:
        xf = np.concatenate([xf, np.zeros((*xf.shape[:-2], pad, xf.shape[-1]), F32)], axis=-2)
    lead = xf.shape[:-2]
    nblk = xf.shape[-2] // block_size
    blocked = xf.reshape(*lead, nblk, block_size, xf.shape[-1])
    bmin = blocked.min(axis=(-2, -1), keepdims=True)
    bmax = blocked.max(axis=(-2, -1), keepdims=True)
    scale = np.maximum((bmax - bmin) / F32(255.0), _SCALE_FLOOR).astype(F32)
    zp = np.clip(np.rint((-bmin) / scale), F32(0), F32(255)).astype(F32)
    q = np.clip(np.rint(blocked / scale + zp), F32(0), F32(255))
    values = (q.astype(np.int16) - 128).astype(np.int8)
    return OQuant(values, scale, zp.astype(np.int16), block_size, original_shape)


def dequantize_int8_per_block(q: OQuant) -> np.ndarray:
    """quant.py:168-204: (float(v+128) - float(zp)) * scale, reshape, drop padding."""
    u = q.values.astype(np.int16) + 128
    x = (u.astype(F32) - q.zero_point.astype(F32)) * q.scale.astype(F32)
    lead = q.original_shape[:-2]
    seq, d = q.original_shape[-2], q.original_shape[-1]
    return x.reshape(*lead, -1, d)[..., :seq, :]


def estimate_quantized_bytes(q: OQuant) -> int:
    """quant.py:232-247."""
    return int(q.values.size + q.scale.size * 4 + q.zero_point.size * 2)


# ---------------------------------------------------------------------------
# attention -- src/flashspec/attention.py
# ---------------------------------------------------------------------------


def reference_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                        lengths: Optional[np.ndarray] = None, out_dtype=None) -> np.ndarray:
    """attention.py:70-121: fp32 scores * 1/sqrt(D), mask pos>=len with fp32 min,
    softmax, fp32 PV, cast to q dtype.  MHA: q [B,H,D], k/v [B,H,S,D]."""
    out_dtype = out_dtype or q.dtype
    qf = q.astype(F32)
    kf = k.astype(F32)
    vf = v.astype(F32)
    scale = F32(1.0 / math.sqrt(q.shape[-1]))
    scores = np.matmul(kf, qf[..., None])[..., 0] * scale  # [B,H,S]
    if lengths is not None:
        pos = np.arange(k.shape[-2])[None, :]
        mask = pos >= np.asarray(lengths).reshape(-1, 1)
        scores = np.where(mask[:, None, :], _F32_MIN, scores)
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - m)
    p = e / e.sum(axis=-1, keepdims=True)
    out = np.matmul(p[..., None, :], vf)[..., 0, :]
    return out.astype(out_dtype)


def _gqa_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, lengths) -> np.ndarray:
    """GQA restated as G MHA calls on q[:, g::G] (the reference has no GQA;
    attention.py:41 requires Hq == Hkv)."""
    hq, hkv = q.shape[1], k.shape[1]
    if hq % hkv:
        raise ValueError("q heads must be a multiple of kv heads")
    g_count = hq // hkv
    if g_count == 1:
        return reference_attention(q, k, v, lengths)
    out = np.empty(q.shape, dtype=q.dtype)
    for g in range(g_count):
        out[:, g::g_count] = reference_attention(q[:, g::g_count], k, v, lengths)
    return out


def fused_dequant_attention(q: np.ndarray, kq: OQuant, vq: OQuant,
                            lengths: Optional[np.ndarray] = None) -> np.ndarray:
    """attention.py:124-168 (the reference CPU ``fused`` backend): dequantize, then
    reference_attention.  GQA handled by ``_gqa_attention``."""
    k = dequantize_int8_per_block(kq)
    v = dequantize_int8_per_block(vq)
    return _gqa_attention(q, k, v, lengths)


# ---------------------------------------------------------------------------
# paged cache -- src/flashspec/paged.py
# ---------------------------------------------------------------------------


@dataclass
class OPagedCache:
    """Mirror of ``PagedKVCache`` (paged.py:258-300)."""

    k_quant: OQuant
    v_quant: OQuant
    block_table: np.ndarray  # int64 [B, cols], -1 = unallocated
    lengths: np.ndarray  # int64 [B]
    block_size: int
    max_seq_len: int

    @property
    def batch_size(self) -> int:
        return int(self.block_table.shape[0])

    @property
    def num_heads(self) -> int:
        return int(self.k_quant.original_shape[1])

    @property
    def head_dim(self) -> int:
        return int(self.k_quant.original_shape[-1])

    def estimated_bytes(self) -> int:
        """paged.py:559-577."""
        return (estimate_quantized_bytes(self.k_quant) + estimate_quantized_bytes(self.v_quant)
                + self.block_table.size * 8 + self.lengths.size * 8)


def paged_from_dense(k: np.ndarray, v: np.ndarray, block_size: int = 16, *,
                     lengths: Optional[np.ndarray] = None, pattern: str = "contiguous",
                     perm: Optional[np.ndarray] = None) -> OPagedCache:
    """paged.py:303-419.  Physical page order: contiguous = batch-major logical order
    (paged.py:374); shuffled = ``perm`` (the reference draws it with torch.randperm,
    paged.py:380-388 -- the permutation is passed in so the oracle needs no torch RNG);
    interleaved = logical-block-major (paged.py:389-398).  The table is the inverse
    permutation."""
    b, h, s, d = k.shape
    bps = (s + block_size - 1) // block_size
    total = b * bps
    pad = bps * block_size - s

    def to_phys(x):
        x = np.asarray(x, dtype=F32)
        if pad:
            x = np.concatenate([x, np.zeros((b, h, pad, d), F32)], axis=2)
        return x.reshape(b, h, bps, block_size, d).transpose(0, 2, 1, 3, 4).reshape(total, h, block_size, d)

    pk, pv = to_phys(k), to_phys(v)
    table = np.arange(total, dtype=np.int64).reshape(b, bps)
    pattern = pattern.strip().lower()
    if pattern in ("shuffled", "random"):
        if perm is None:
            raise ValueError("shuffled layout needs perm")
        perm = np.asarray(perm, dtype=np.int64)
    elif pattern == "interleaved":
        perm = np.arange(total, dtype=np.int64).reshape(b, bps).T.reshape(-1)
    elif pattern in ("contiguous", ""):
        perm = None
    else:
        raise ValueError("bad pattern")
    if perm is not None:
        pk, pv = pk[perm], pv[perm]
        inv = np.empty_like(perm)
        inv[perm] = np.arange(total, dtype=np.int64)
        table = inv.reshape(b, bps)
    lens = np.full((b,), s, np.int64) if lengths is None else np.asarray(lengths, np.int64)
    return OPagedCache(quantize_int8_per_block(pk, block_size), quantize_int8_per_block(pv, block_size),
                       table, lens, block_size, s)


def paged_to_dense(cache: OPagedCache) -> Tuple[np.ndarray, np.ndarray]:
    """paged.py:421-461: dequantize the WHOLE physical pool, gather by
    ``table.clamp_min(0)``, permute to [B,H,S,D], truncate to max_seq_len."""
    pk = dequantize_int8_per_block(cache.k_quant)
    pv = dequantize_int8_per_block(cache.v_quant)
    table = np.maximum(cache.block_table, 0)
    b, h, d = cache.batch_size, cache.num_heads, cache.head_dim

    def gather(p):
        g = p[table]  # [B, cols, H, bs, D]
        return g.transpose(0, 2, 1, 3, 4).reshape(b, h, -1, d)[..., : cache.max_seq_len, :]

    return gather(pk), gather(pv)


def paged_quant_attention(q: np.ndarray, cache: OPagedCache) -> np.ndarray:
    """attention.py:171-223 (the reference CPU ``paged`` backend): to_dense + masked
    reference attention with cache.lengths.  GQA via G MHA calls."""
    k, v = paged_to_dense(cache)
    return _gqa_attention(q, k, v, cache.lengths)


def paged_quant_attention_gathered(q: np.ndarray, cache: OPagedCache) -> np.ndarray:
    """Same math as ``paged_quant_attention`` but dequantizes only the pages the
    table references (used for large parity cases where dequantizing the slack
    of the pool would only cost time; results are identical because unreferenced
    pages never enter the gather)."""
    b, cols = cache.block_table.shape
    table = np.maximum(cache.block_table, 0)
    used = np.unique(table)
    remap = np.zeros(int(table.max()) + 1, np.int64)
    remap[used] = np.arange(used.size)
    sub = lambda qt: OQuant(qt.values[used], qt.scale[used], qt.zero_point[used], qt.block_size,
                            (used.size,) + tuple(qt.original_shape[1:]))
    small = OPagedCache(sub(cache.k_quant), sub(cache.v_quant), remap[table], cache.lengths,
                        cache.block_size, cache.max_seq_len)
    return paged_quant_attention(q, small)


def paged_cache_append(cache: OPagedCache, k_new: np.ndarray, v_new: np.ndarray) -> OPagedCache:
    """paged.py:463-557 functional append: dequantize the whole store, widen the
    table, write new tokens (allocating new pages at the END of the store in
    (batch, token) order), re-quantize the whole store."""
    bs = cache.block_size
    pk = dequantize_int8_per_block(cache.k_quant).copy()
    pv = dequantize_int8_per_block(cache.v_quant).copy()
    table = cache.block_table.copy()
    lengths = cache.lengths.copy()
    t_new = k_new.shape[2]
    req_cols = int(((lengths + t_new + bs - 1) // bs).max())
    if req_cols > table.shape[1]:
        table = np.concatenate([table, np.full((table.shape[0], req_cols - table.shape[1]), -1, np.int64)], 1)
    kn = np.asarray(k_new, F32)
    vn = np.asarray(v_new, F32)
    h, d = cache.num_heads, cache.head_dim
    for bi in range(table.shape[0]):
        start = int(lengths[bi])
        for ti in range(t_new):
            pos = start + ti
            lb, off = pos // bs, pos % bs
            pidx = int(table[bi, lb])
            if pidx < 0:
                pidx = pk.shape[0]
                pk = np.concatenate([pk, np.zeros((1, h, bs, d), F32)], 0)
                pv = np.concatenate([pv, np.zeros((1, h, bs, d), F32)], 0)
                table[bi, lb] = pidx
            pk[pidx, :, off, :] = kn[bi, :, ti, :]
            pv[pidx, :, off, :] = vn[bi, :, ti, :]
    lengths = lengths + t_new
    return OPagedCache(quantize_int8_per_block(pk, bs), quantize_int8_per_block(pv, bs), table, lengths,
                       bs, int(lengths.max()))


class OAllocator:
    """paged.py:17-255 ``PagedKVAllocator``: fixed pool of pages initialised to
    quantized zeros, ascending free list with lowest-first allocation
    (``pop(0)``, paged.py:221-224), release = extend + sort (paged.py:146-151),
    page-granular dequantize -> insert -> requantize appends (paged.py:108-136,
    226-255) that keep stale rows of reused pages."""

    def __init__(self, capacity_blocks: int, heads: int, head_dim: int, block_size: int = 16):
        self.capacity_blocks, self.heads, self.head_dim, self.block_size = capacity_blocks, heads, head_dim, block_size
        zeros = np.zeros((capacity_blocks, heads, block_size, head_dim), F32)
        self.k_quant = quantize_int8_per_block(zeros, block_size)
        self.v_quant = quantize_int8_per_block(zeros, block_size)
        self.free_blocks: List[int] = list(range(capacity_blocks))
        self.requests: Dict[int, Tuple[List[int], int]] = {}

    def _alloc(self) -> int:
        if not self.free_blocks:
            raise RuntimeError("out of pages")
        return self.free_blocks.pop(0)

    def _deq_page(self, p: int) -> Tuple[np.ndarray, np.ndarray]:
        """paged.py:226-245."""
        def one(qt):
            u = qt.values[p].astype(np.int16) + 128  # [H,1,bs,D]
            x = (u.astype(F32) - qt.zero_point[p].astype(F32)) * qt.scale[p].astype(F32)
            return x.reshape(self.heads, self.block_size, self.head_dim).copy()
        return one(self.k_quant), one(self.v_quant)

    def _write_page(self, p: int, kb: np.ndarray, vb: np.ndarray) -> None:
        """paged.py:247-255: quantize [1,H,bs,D] with block=bs and store."""
        for qt, blk in ((self.k_quant, kb), (self.v_quant, vb)):
            nq = quantize_int8_per_block(blk[None], self.block_size)
            qt.values[p] = nq.values[0]
            qt.scale[p] = nq.scale[0]
            qt.zero_point[p] = nq.zero_point[0]

    def add_request(self, rid: int, k: np.ndarray, v: np.ndarray, length: Optional[int] = None) -> None:
        """paged.py:66-106: zero-padded pages, quantized one by one."""
        if rid in self.requests:
            raise ValueError("duplicate request")
        seq = k.shape[2]
        eff = seq if length is None else int(length)
        need = (eff + self.block_size - 1) // self.block_size
        if len(self.free_blocks) < need:
            raise RuntimeError("out of pages")
        pages = []
        for lb in range(need):
            p = self._alloc()
            pages.append(p)
            s0, s1 = lb * self.block_size, min(lb * self.block_size + self.block_size, eff)
            kb = np.zeros((self.heads, self.block_size, self.head_dim), F32)
            vb = np.zeros_like(kb)
            kb[:, : s1 - s0] = np.asarray(k[0, :, s0:s1], F32)
            vb[:, : s1 - s0] = np.asarray(v[0, :, s0:s1], F32)
            self._write_page(p, kb, vb)
        self.requests[rid] = (pages, eff)

    def append_request(self, rid: int, k_new: np.ndarray, v_new: np.ndarray) -> None:
        """paged.py:108-136."""
        pages, length = self.requests[rid]
        t = k_new.shape[2]
        touched: Dict[int, Tuple[np.ndarray, np.ndarray]] = {}
        for ti in range(t):
            pos = length + ti
            lb, off = pos // self.block_size, pos % self.block_size
            if lb == len(pages):
                pages.append(self._alloc())
            p = pages[lb]
            if p not in touched:
                touched[p] = self._deq_page(p)
            touched[p][0][:, off] = np.asarray(k_new[0, :, ti], F32)
            touched[p][1][:, off] = np.asarray(v_new[0, :, ti], F32)
        for p, (kb, vb) in touched.items():
            self._write_page(p, kb, vb)
        self.requests[rid] = (pages, length + t)

    def append_batch(self, rids: Sequence[int], k_new: np.ndarray, v_new: np.ndarray) -> None:
        """paged.py:138-144."""
        for i, rid in enumerate(rids):
            self.append_request(int(rid), k_new[i : i + 1], v_new[i : i + 1])

    def release_request(self, rid: int) -> None:
        """paged.py:146-151."""
        pages, _ = self.requests.pop(int(rid))
        self.free_blocks.extend(pages)
        self.free_blocks.sort()

    def to_cache(self, rids: Optional[Sequence[int]] = None) -> OPagedCache:
        """paged.py:153-179."""
        ids = list(self.requests.keys()) if rids is None else [int(r) for r in rids]
        reqs = [self.requests[r] for r in ids]
        cols = max(1, max(len(p) for p, _ in reqs))
        table = np.full((len(reqs), cols), -1, np.int64)
        lens = np.empty((len(reqs),), np.int64)
        for i, (p, ln) in enumerate(reqs):
            table[i, : len(p)] = p
            lens[i] = ln
        return OPagedCache(self.k_quant, self.v_quant, table, lens, self.block_size, int(lens.max()))

    def stats(self) -> Dict[str, float]:
        """paged.py:181-199."""
        alloc = self.capacity_blocks - len(self.free_blocks)
        used = sum(ln for _, ln in self.requests.values())
        at = alloc * self.block_size
        cap = self.capacity_blocks * self.block_size
        waste = max(0, at - used)
        return {
            "allocated_blocks": float(alloc), "free_blocks": float(len(self.free_blocks)),
            "live_requests": float(len(self.requests)), "used_tokens": float(used),
            "capacity_tokens": float(cap), "block_utilization": used / max(1, at),
            "capacity_utilization": used / max(1, cap), "padding_waste": float(waste),
            "fragmentation": waste / max(1, at),
        }


# ---------------------------------------------------------------------------
# split-K / cross-GPU merge -- src/flashspec/triton_fused.py:446-503
# ---------------------------------------------------------------------------


def partial_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, lo: int, hi: int,
                      lengths: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Attention of q over tokens [lo, min(hi, len)) returning (O fp32 normalised,
    LSE fp32 natural log); an empty range gives O=0, LSE=-inf.  MHA shapes."""
    qf, kf, vf = q.astype(F32), k.astype(F32), v.astype(F32)
    scale = F32(1.0 / math.sqrt(q.shape[-1]))
    b, h, s, d = k.shape
    o = np.zeros((b, h, d), F32)
    lse = np.full((b, h), -np.inf, F32)
    for bi in range(b):
        e = min(hi, int(lengths[bi]), s)
        if e <= lo:
            continue
        sc = np.einsum("hd,hsd->hs", qf[bi], kf[bi, :, lo:e]) * scale
        m = sc.max(-1, keepdims=True)
        w = np.exp(sc - m)
        l = w.sum(-1, keepdims=True)
        o[bi] = np.einsum("hs,hsd->hd", w / l, vf[bi, :, lo:e])
        lse[bi] = (m + np.log(l))[:, 0]
    return o, lse


def merge_partials(o: np.ndarray, lse: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge of N partials (the combine math of triton_fused.py:487-503,
    expressed on (O, LSE) pairs): o [N,...,D], lse [N,...] -> fp32 [...,D]; all-empty
    rows give 0 (triton_utils.py:181-186)."""
    m = lse.max(axis=0)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    w = np.where(np.isfinite(lse), np.exp(lse - m_safe[None]), 0.0)
    den = w.sum(axis=0)
    num = (w[..., None] * o).sum(axis=0)
    return np.where(den[..., None] > 0, num / np.where(den > 0, den, 1.0)[..., None], 0.0).astype(F32)


# ---------------------------------------------------------------------------
# tree-attention verify -- doc/TODO.MD:186-237 (planned in the reference, not implemented)
# ---------------------------------------------------------------------------


def tree_mask(parents: np.ndarray) -> np.ndarray:
    """Dense tree mask [B, N, N]: mask[b, i, j] is True when draft node j is node i or
    one of its ancestors (parents[b, i] < i, -1 = root hangs off the committed prefix)."""
    b, n = parents.shape
    m = np.zeros((b, n, n), bool)
    for bi in range(b):
        for i in range(n):
            j = i
            while j >= 0:
                m[bi, i, j] = True
                j = int(parents[bi, j])
    return m


def tree_verify_attention(q: np.ndarray, cache: OPagedCache, tree_k: np.ndarray, tree_v: np.ndarray,
                          parents: np.ndarray) -> np.ndarray:
    """The dense-mask statement of tree verify: node i of request b attends to the
    committed prefix (the first lengths[b] tokens of the paged cache, dequantized as the
    reference's to_dense does) and to the draft tokens the tree mask allows, fp32 softmax
    with scale 1/sqrt(D), output cast to q's dtype.  q [B, N, Hq, D], tree_k/v
    [B, N, Hkv, D]; GQA as elsewhere (q head h reads kv head h // (Hq / Hkv))."""
    b, n, hq, d = q.shape
    kd, vd = paged_to_dense(cache)  # [B, Hkv, S, D]
    hkv = kd.shape[1]
    g = hq // hkv
    s = kd.shape[2]
    mask = tree_mask(parents)
    out = np.zeros(q.shape, np.float32)
    scale = F32(1.0 / math.sqrt(d))
    for bi in range(b):
        L = min(int(cache.lengths[bi]), s)
        for h in range(hq):
            kh = h // g
            keys = np.concatenate([kd[bi, kh, :L], tree_k[bi, :, kh].astype(F32)], 0)  # [L + N, D]
            vals = np.concatenate([vd[bi, kh, :L], tree_v[bi, :, kh].astype(F32)], 0)
            sc = (keys @ q[bi, :, h].astype(F32).T).T * scale  # [N, L + N]
            allowed = np.concatenate([np.ones((n, L), bool), mask[bi]], 1)
            sc = np.where(allowed, sc, -np.inf)
            w = np.exp(sc - sc.max(1, keepdims=True))
            out[bi, :, h] = (w / w.sum(1, keepdims=True)) @ vals
    return out.astype(q.dtype)


# ---------------------------------------------------------------------------
# symmetric per-token INT8 -- the format of the benchmark configurations' wording; the
# reference lists it as future work (doc/TODO.MD:241-255), so this is the specification
# restated: s = max(absmax / 127, 1e-8) per (token, head), q = clamp(rint(x / s), +-127)
# ---------------------------------------------------------------------------


def quantize_symmetric(x: np.ndarray):
    """x [..., S, D] -> (values int8 [..., S, D], scale fp32 [..., S]), each step fp32."""
    xf = np.asarray(x, F32)
    s = np.maximum(np.abs(xf).max(-1) / F32(127.0), _SCALE_FLOOR).astype(F32)
    q = np.clip(np.rint(xf / s[..., None]), -127, 127).astype(np.int8)
    return q, s


def symmetric_paged_attention(q: np.ndarray, k_values: np.ndarray, k_scale: np.ndarray, v_values: np.ndarray,
                              v_scale: np.ndarray, table: np.ndarray, lengths: np.ndarray, max_seq_len: int) -> np.ndarray:
    """Paged attention over a symmetric pool (values [P, Hkv, page, D], scales
    [P, Hkv, page]): dequantize (values * scale), gather by table.clamp_min(0), masked
    reference attention -- the reference's paged path (attention.py:171-223) with this
    format's dequantization."""
    b, cols = table.shape
    t = np.maximum(table, 0)

    def dense(vals, sc):
        x = vals.astype(F32) * sc[..., None]  # [P, H, page, D]
        g = x[t]  # [B, cols, H, page, D]
        return g.transpose(0, 2, 1, 3, 4).reshape(b, x.shape[1], -1, x.shape[-1])[..., :max_seq_len, :]

    return _gqa_attention(q, dense(k_values, k_scale), dense(v_values, v_scale), lengths)


def algorithmic_bytes_paged(batch: int, q_heads: int, kv_heads: int, head_dim: int, lengths: Sequence[int],
                            page: int = 16, table_cols: Optional[int] = None, q_bytes: int = 2) -> int:
    """Algorithmic bytes of one paged decode call: for every referenced (page, kv
    head): K+V int8 values + fp32 scale + int16 zp; plus q and out (fp16), the int64
    table and lengths."""
    pages = sum((int(n) + page - 1) // page for n in lengths)
    kv = pages * kv_heads * 2 * (page * head_dim + 4 + 2)
    cols = table_cols if table_cols is not None else max((int(n) + page - 1) // page for n in lengths)
    return kv + 2 * batch * q_heads * head_dim * q_bytes + batch * cols * 8 + batch * 8
