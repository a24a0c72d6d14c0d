"""Paged INT8 KV cache and a device-resident page allocator.

``PagedKVCache`` has the fields and layouts of the reference class
(src/flashspec/paged.py:258-300): pool values [P, H, 1, bs, D] int8 with qparams
[P, H, 1, 1, 1], block_table int64 [B, cols] (-1 = unallocated), lengths int64 [B].

``PagedKVAllocator`` reproduces the reference allocator (paged.py:17-255) -- same
methods, same lowest-page-first free list, same stale-row semantics of reused pages --
with the pool in HBM and every page write done by one batched ``fs_page_update``
launch (dequantize page -> insert rows -> requantize, bit-exact).
"""

from __future__ import annotations

import ctypes as C
import heapq
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from .quant import (QuantizedTensor, dequantize_int8_per_block, dtype_code, estimate_quantized_bytes,
                    quantize_int8_per_block, require_cuda, stream_of)

ITEM_DTYPE = np.dtype([("page", "<i8"), ("src_b", "<i4"), ("src_t", "<i4"), ("dst_row", "<i4"),
                       ("n_rows", "<i4"), ("from_zero", "<i4"), ("reserved", "<i4")])
assert ITEM_DTYPE.itemsize == C.sizeof(_lib.FsPageUpdate)

_SCALE_FLOOR = float(np.float32(1.0e-8))


class _PinnedRing:
    """Reusable pinned staging buffers for small per-step uploads (page-update items,
    table changes): a buffer is refilled only after the copy that last read it has
    completed on the GPU, so no pinned allocation happens per call."""

    def __init__(self, n: int = 8):
        self.bufs = [None] * n
        self.events = [None] * n
        self.i = 0

    def upload(self, arr: np.ndarray, device: torch.device) -> torch.Tensor:
        raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        k = self.i
        self.i = (self.i + 1) % len(self.bufs)
        if self.events[k] is not None:
            self.events[k].synchronize()
        if self.bufs[k] is None or self.bufs[k].numel() < raw.size:
            self.bufs[k] = torch.empty(max(raw.size, 4096), dtype=torch.uint8).pin_memory()
        host = self.bufs[k][: raw.size]
        host.numpy()[:] = raw
        dev = host.to(device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(device))
        self.events[k] = ev
        return dev


_RING = _PinnedRing()


def _upload(arr: np.ndarray, device: torch.device) -> torch.Tensor:
    return _RING.upload(arr, device)


def page_update(items: np.ndarray, k_src: torch.Tensor, v_src: torch.Tensor, dst_k: QuantizedTensor,
                dst_v: QuantizedTensor, src_k: Optional[QuantizedTensor] = None,
                src_v: Optional[QuantizedTensor] = None) -> None:
    """Launch ``fs_page_update`` for ``items`` (ITEM_DTYPE records).  k_src/v_src are
    [Bsrc, H, T, D] token sources; pools are [P, H, 1, bs, D]; src_* default to the
    destination (in-place update)."""
    if items.size == 0:
        return
    src_k = src_k or dst_k
    src_v = src_v or dst_v
    device = dst_k.values.device
    if k_src.stride(-1) != 1:
        k_src = k_src.contiguous()
    if v_src.stride(-1) != 1:
        v_src = v_src.contiguous()
    if k_src.stride() != v_src.stride() or k_src.dtype != v_src.dtype:
        k_src, v_src = k_src.contiguous(), v_src.to(k_src.dtype).contiguous()
    dev_items = _upload(items, device)
    a = _lib.FsPageUpdateArgs()
    a.items = dev_items.data_ptr()
    a.n_items = int(items.size)
    a.k_src, a.v_src = k_src.data_ptr(), v_src.data_ptr()
    a.src_dtype = dtype_code(k_src)
    a.src_stride_b, a.src_stride_h, a.src_stride_t = k_src.stride(0), k_src.stride(1), k_src.stride(2)
    a.heads = int(dst_k.values.shape[1])
    a.head_dim = int(dst_k.values.shape[-1])
    a.block_size = int(dst_k.values.shape[-2])
    a.num_pages = int(dst_k.values.shape[0])
    a.k_values_in, a.k_scale_in, a.k_zero_in = src_k.values.data_ptr(), src_k.scale.data_ptr(), src_k.zero_point.data_ptr()
    a.v_values_in, a.v_scale_in, a.v_zero_in = src_v.values.data_ptr(), src_v.scale.data_ptr(), src_v.zero_point.data_ptr()
    a.k_values_out, a.k_scale_out, a.k_zero_out = dst_k.values.data_ptr(), dst_k.scale.data_ptr(), dst_k.zero_point.data_ptr()
    a.v_values_out, a.v_scale_out, a.v_zero_out = dst_v.values.data_ptr(), dst_v.scale.data_ptr(), dst_v.zero_point.data_ptr()
    with torch.cuda.device(device):
        _lib.check(_lib.load().fs_page_update(C.byref(a), stream_of(device)), "fs_page_update")
    # keep the uploaded item buffer alive until the kernel has consumed it
    dev_items.record_stream(torch.cuda.current_stream(device))


def empty_pool(pages: int, heads: int, block_size: int, head_dim: int, device) -> QuantizedTensor:
    """A pool of quantized all-zero pages, bit-identical to quantize_int8_per_block of
    zeros (values -128, scale 1e-8, zero point 0) as the reference allocator starts
    (paged.py:48-55)."""
    values = torch.full((pages, heads, 1, block_size, head_dim), -128, dtype=torch.int8, device=device)
    scale = torch.full((pages, heads, 1, 1, 1), _SCALE_FLOOR, dtype=torch.float32, device=device)
    zp = torch.zeros((pages, heads, 1, 1, 1), dtype=torch.int16, device=device)
    return QuantizedTensor(values, scale, zp, block_size, (pages, heads, block_size, head_dim))


@dataclass(frozen=True)
class PagedKVCache:
    """Same fields and semantics as the reference PagedKVCache (paged.py:258-300)."""

    k_quant: QuantizedTensor
    v_quant: QuantizedTensor
    block_table: torch.Tensor
    lengths: torch.Tensor
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

    @classmethod
    def from_dense(cls, k: torch.Tensor, v: torch.Tensor, block_size: int = 16, *,
                   lengths: Optional[torch.Tensor] = None, block_table_pattern: str = "contiguous",
                   layout_seed: int = 0, perm: Optional[torch.Tensor] = None) -> "PagedKVCache":
        """paged.py:303-419 on the GPU: pad, split into pages (batch-major physical
        order), optionally permute (``shuffled``: seeded randperm on k's device, or an
        explicit ``perm``; ``interleaved``: logical-block-major), quantize the pool with
        the CUDA quantizer.  The table is the inverse permutation."""
        require_cuda(k, "k")
        if k.ndim != 4 or v.ndim != 4:
            raise ValueError("k and v must have shape [batch, heads, seq_len, head_dim]")
        if k.shape != v.shape:
            raise ValueError("k and v shapes differ")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        b, h, s, d = k.shape
        bps = (s + block_size - 1) // block_size
        total = b * bps
        pad = bps * block_size - s

        def phys(x):
            if pad:
                x = torch.cat([x, x.new_zeros((b, h, pad, d))], dim=2)
            return x.reshape(b, h, bps, block_size, d).permute(0, 2, 1, 3, 4).reshape(total, h, block_size, d)

        pk, pv = phys(k), phys(v)
        table = torch.arange(total, dtype=torch.int64, device=k.device).reshape(b, bps)
        pattern = block_table_pattern.strip().lower()
        if pattern not in {"contiguous", "", "shuffled", "random", "interleaved"}:
            raise ValueError("block_table_pattern must be contiguous, shuffled or interleaved")
        if pattern in {"shuffled", "random"}:
            if perm is None:
                gen = torch.Generator(device=k.device)
                gen.manual_seed(int(layout_seed))
                perm = torch.randperm(total, generator=gen, device=k.device)
        elif pattern == "interleaved":
            perm = torch.arange(total, dtype=torch.int64, device=k.device).reshape(b, bps).t().reshape(-1)
        else:
            perm = None
        if perm is not None:
            perm = perm.to(device=k.device, dtype=torch.int64)
            pk, pv = pk[perm].contiguous(), pv[perm].contiguous()
            inv = torch.empty_like(perm)
            inv[perm] = torch.arange(total, dtype=torch.int64, device=k.device)
            table = inv.reshape(b, bps)
        if lengths is None:
            lens = torch.full((b,), s, dtype=torch.int64, device=k.device)
        else:
            lens = lengths.to(device=k.device, dtype=torch.int64).contiguous()
            if lens.ndim != 1 or lens.shape[0] != b:
                raise ValueError("lengths must have shape [batch]")
            if bool((lens < 0).any()) or bool((lens > s).any()):
                raise ValueError("lengths must lie in [0, seq_len]")
        return cls(quantize_int8_per_block(pk, block_size), quantize_int8_per_block(pv, block_size), table, lens,
                   block_size, s)

    def to_dense(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """paged.py:421-461 (inspection utility; attention never calls it): dense fp32
        K/V [B, H, max_seq_len, D], unallocated table entries read page 0 as in the
        reference (``table.clamp_min(0)``).  With one quantization block per page, only
        the pages the table references are dequantized (``fs_dequantize_pages``, gathered
        by the kernel); otherwise the whole pool is dequantized with torch ops."""
        table = self.block_table.clamp_min(0)
        kq, vq = self.k_quant, self.v_quant
        page = int(self.block_size)
        if int(kq.block_size) == page and kq.values.is_cuda:
            from . import _lib
            from .quant import stream_of

            pages = table.reshape(-1).to(torch.int64).contiguous()
            b, cols = table.shape

            def gather(qt):
                out = torch.empty((pages.numel(), self.num_heads, page, self.head_dim), dtype=torch.float32,
                                  device=qt.values.device)
                with torch.cuda.device(qt.values.device):
                    _lib.check(_lib.load().fs_dequantize_pages(
                        qt.values.contiguous().data_ptr(), qt.scale.contiguous().data_ptr(),
                        qt.zero_point.contiguous().data_ptr(), pages.data_ptr(), pages.numel(),
                        int(qt.values.shape[0]), self.num_heads, page, self.head_dim, out.data_ptr(),
                        stream_of(qt.values.device)), "fs_dequantize_pages")
                return (out.view(b, cols, self.num_heads, page, self.head_dim).permute(0, 2, 1, 3, 4)
                        .reshape(b, self.num_heads, -1, self.head_dim)[..., : self.max_seq_len, :])

            return gather(kq), gather(vq)
        pk = dequantize_int8_per_block(kq, dtype=torch.float32)
        pv = dequantize_int8_per_block(vq, dtype=torch.float32)

        def gather_t(p):
            return (p[table].permute(0, 2, 1, 3, 4).contiguous()
                    .reshape(self.batch_size, self.num_heads, -1, self.head_dim)[..., : self.max_seq_len, :])

        return gather_t(pk), gather_t(pv)

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> "PagedKVCache":
        """Functional append (paged.py:463-557) on the GPU, bit-exact: every page of the
        store is dequantized and requantized (the reference re-quantizes the whole
        store), new tokens go to their tail pages, missing pages are appended at the end
        of the store in (batch, token) order starting from zeros."""
        if k_new.ndim != 4 or v_new.ndim != 4:
            raise ValueError("k_new and v_new must have shape [batch, heads, tokens, head_dim]")
        if k_new.shape != v_new.shape:
            raise ValueError("k_new and v_new shapes differ")
        if k_new.shape[0] != self.batch_size or k_new.shape[1] != self.num_heads or k_new.shape[3] != self.head_dim:
            raise ValueError("new KV batch / heads / head_dim must match the cache")
        t_new = int(k_new.shape[2])
        if t_new <= 0:
            raise ValueError("append needs at least one token")
        if k_new.device != self.block_table.device or v_new.device != self.block_table.device:
            raise ValueError("new KV must be on the cache's device")
        require_cuda(k_new, "k_new")
        bs = self.block_size
        table = self.block_table.cpu().numpy().copy()
        lengths = self.lengths.cpu().numpy().copy()
        n_old = int(self.k_quant.values.shape[0])
        req_cols = int(((lengths + t_new + bs - 1) // bs).max())
        if req_cols > table.shape[1]:
            table = np.concatenate([table, np.full((table.shape[0], req_cols - table.shape[1]), -1, np.int64)], 1)
        rows: Dict[int, Tuple[int, int, int, int]] = {}  # page -> (src_b, src_t, dst_row, n_rows)
        n_new = 0
        for bi in range(table.shape[0]):
            start = int(lengths[bi])
            for ti in range(t_new):
                pos = start + ti
                lb, off = pos // bs, pos % bs
                p = int(table[bi, lb])
                if p < 0:
                    p = n_old + n_new
                    n_new += 1
                    table[bi, lb] = p
                if p in rows:
                    sb, st, dr, nr = rows[p]
                    if sb != bi or dr + nr != off or st + nr != ti:
                        raise ValueError("append rows into one page must be consecutive tokens of one request")
                    rows[p] = (sb, st, dr, nr + 1)
                else:
                    rows[p] = (bi, ti, off, 1)
        total = n_old + n_new
        items = np.zeros(total, ITEM_DTYPE)
        items["page"] = np.arange(total)
        items["from_zero"][n_old:] = 1
        for p, (sb, st, dr, nr) in rows.items():
            items[p]["src_b"], items[p]["src_t"], items[p]["dst_row"], items[p]["n_rows"] = sb, st, dr, nr
        h, d = self.num_heads, self.head_dim
        dev = self.k_quant.values.device
        nk, nv = empty_pool(total, h, bs, d, dev), empty_pool(total, h, bs, d, dev)
        page_update(items, k_new, v_new, nk, nv, _as_pool(self.k_quant), _as_pool(self.v_quant))
        new_lengths = lengths + t_new
        return PagedKVCache(nk, nv, torch.from_numpy(table).to(dev), torch.from_numpy(new_lengths).to(dev), bs,
                            int(new_lengths.max()))

    def estimated_bytes(self) -> int:
        """paged.py:559-577."""
        return (estimate_quantized_bytes(self.k_quant) + estimate_quantized_bytes(self.v_quant)
                + self.block_table.numel() * self.block_table.element_size()
                + self.lengths.numel() * self.lengths.element_size())


def _as_pool(qt) -> QuantizedTensor:
    return QuantizedTensor(qt.values.contiguous(), qt.scale.contiguous(), qt.zero_point.contiguous(),
                           int(qt.block_size), tuple(qt.original_shape))


class _Request:
    """Host record of one live request: its row in the allocator's page table and its
    token count."""

    __slots__ = ("slot", "length", "_owner")

    def __init__(self, slot: int, length: int, owner: "PagedKVAllocator"):
        self.slot, self.length, self._owner = slot, length, owner

    @property
    def pages(self) -> List[int]:
        o = self._owner
        return o._ptab[self.slot, : o._npages[self.slot]].tolist()


class PagedKVAllocator:
    """Device-resident version of the reference PagedKVAllocator (paged.py:17-255).

    The pool lives in HBM; the bookkeeping is on the host: a min-heap free list
    (allocation takes the lowest free page, which is what the reference's sorted list +
    pop(0) does) and a slot-indexed numpy page table (row = live request, -1 padded), so
    ``to_cache`` and single-token ``append_batch`` are a few numpy operations rather than
    a Python loop per request.  Every data write is one batched ``fs_page_update``."""

    def __init__(self, *, capacity_blocks: int, heads: int, head_dim: int, block_size: int = 16,
                 device="cuda", dtype: torch.dtype = torch.float32) -> None:
        if capacity_blocks <= 0:
            raise ValueError("capacity_blocks must be positive")
        if heads <= 0 or head_dim <= 0:
            raise ValueError("heads and head_dim must be positive")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        self.capacity_blocks, self.heads, self.head_dim, self.block_size = (
            int(capacity_blocks), int(heads), int(head_dim), int(block_size))
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("PagedKVAllocator keeps its pool on a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self.k_quant = empty_pool(self.capacity_blocks, self.heads, self.block_size, self.head_dim, self.device)
        self.v_quant = empty_pool(self.capacity_blocks, self.heads, self.block_size, self.head_dim, self.device)
        self._free: List[int] = list(range(self.capacity_blocks))  # a valid min-heap
        self._requests: Dict[int, _Request] = {}
        self._ptab = np.full((16, 16), -1, np.int64)  # [slot, logical page] -> physical page
        self._npages = np.zeros(16, np.int64)
        self._lens = np.zeros(16, np.int64)
        self._free_slots: List[int] = list(range(16))
        # device copy of the slot-indexed table and lengths, updated by the changes since
        # the last to_cache (entries (slot, col) and slots whose length changed)
        self._dtab: Optional[torch.Tensor] = None
        self._dlens: Optional[torch.Tensor] = None
        self._dirty_e: List[Tuple[np.ndarray, np.ndarray]] = []
        self._dirty_l: List[np.ndarray] = []

    # -- bookkeeping ----------------------------------------------------------------
    @property
    def live_request_ids(self) -> List[int]:
        return list(self._requests.keys())

    @property
    def free_blocks(self) -> List[int]:
        """The free list in the reference's order (ascending)."""
        return sorted(self._free)

    def _allocate_block(self) -> int:
        if not self._free:
            raise RuntimeError("PagedKVAllocator is out of physical pages")
        return heapq.heappop(self._free)

    def _new_slot(self, pages_hint: int) -> int:
        if not self._free_slots:
            n = self._ptab.shape[0]
            self._ptab = np.concatenate([self._ptab, np.full((n, self._ptab.shape[1]), -1, np.int64)], 0)
            self._npages = np.concatenate([self._npages, np.zeros(n, np.int64)])
            self._lens = np.concatenate([self._lens, np.zeros(n, np.int64)])
            self._free_slots = list(range(2 * n - 1, n - 1, -1))
        self._ensure_cols(pages_hint)
        return self._free_slots.pop()

    def _ensure_cols(self, cols: int) -> None:
        if cols > self._ptab.shape[1]:
            new = max(cols, 2 * self._ptab.shape[1])
            pad = np.full((self._ptab.shape[0], new - self._ptab.shape[1]), -1, np.int64)
            self._ptab = np.concatenate([self._ptab, pad], 1)

    def _validate_kv(self, k: torch.Tensor, v: torch.Tensor, *, batch_expected: Optional[int]) -> None:
        """paged.py:201-219."""
        if k.ndim != 4 or v.ndim != 4:
            raise ValueError("KV must have shape [batch, heads, tokens, head_dim]")
        if k.shape != v.shape:
            raise ValueError("K/V shapes differ")
        if batch_expected is not None and k.shape[0] != batch_expected:
            raise ValueError("KV batch must match request_ids")
        if k.shape[1] != self.heads or k.shape[3] != self.head_dim:
            raise ValueError("KV heads/head_dim must match the allocator")
        if k.shape[2] <= 0:
            raise ValueError("KV token dimension is empty")
        if k.device != self.device or v.device != self.device:
            raise ValueError("KV tensors must be on the allocator's device")

    def _get(self, request_id: int) -> _Request:
        try:
            return self._requests[int(request_id)]
        except KeyError as exc:
            raise KeyError(f"unknown request_id: {request_id}") from exc

    # -- writes -----------------------------------------------------------------------
    def add_request(self, request_id: int, k: torch.Tensor, v: torch.Tensor, *, length: Optional[int] = None) -> None:
        """paged.py:66-106: prompt pages, zero padded, quantized page by page."""
        request_id = int(request_id)
        if request_id in self._requests:
            raise ValueError(f"request_id {request_id} already exists")
        self._validate_kv(k, v, batch_expected=None)
        if k.shape[0] != 1:
            raise ValueError("add_request takes one request (batch dim 1)")
        seq = int(k.shape[2])
        eff = seq if length is None else int(length)
        if eff < 0 or eff > seq:
            raise ValueError("length must lie in [0, seq_len]")
        need = (eff + self.block_size - 1) // self.block_size
        if len(self._free) < need:
            raise RuntimeError("PagedKVAllocator is out of physical pages")
        slot = self._new_slot(need)
        pages = [self._allocate_block() for _ in range(need)]
        self._ptab[slot, :] = -1
        self._ptab[slot, :need] = pages
        self._npages[slot] = need
        self._lens[slot] = eff
        self._dirty_e.append((np.full(need, slot, np.int64), np.arange(need, dtype=np.int64)))
        self._dirty_l.append(np.array([slot], np.int64))
        if need:
            items = np.zeros(need, ITEM_DTYPE)
            starts = np.arange(need) * self.block_size
            items["page"] = pages
            items["src_t"] = starts
            items["n_rows"] = np.minimum(self.block_size, eff - starts)
            items["from_zero"] = 1
            page_update(items, k, v, self.k_quant, self.v_quant)
        self._requests[request_id] = _Request(slot, eff, self)

    def append_request(self, request_id: int, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """paged.py:108-136."""
        self._validate_kv(k_new, v_new, batch_expected=1)
        self.append_batch([request_id], k_new, v_new)

    def append_batch(self, request_ids: Sequence[int], k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """paged.py:138-144, batched: every touched page of every request is rewritten by
        one kernel launch.  Pages are allocated in the reference's order (requests in
        order, tokens in order)."""
        ids = [int(r) for r in request_ids]
        self._validate_kv(k_new, v_new, batch_expected=len(ids))
        t = int(k_new.shape[2])
        reqs = [self._get(r) for r in ids]
        slots = np.fromiter((r.slot for r in reqs), np.int64, len(reqs))
        lens = self._lens[slots]
        npg = self._npages[slots]
        bs = self.block_size
        need_pages = np.maximum(0, (lens + t + bs - 1) // bs - npg)
        if int(need_pages.sum()) > len(self._free):
            raise RuntimeError("PagedKVAllocator is out of physical pages")
        self._ensure_cols(int(((lens + t + bs - 1) // bs).max()) if len(ids) else 0)
        if t == 1:  # decode step: one row into each tail page
            off = lens % bs
            lb = lens // bs
            grown = np.nonzero(need_pages)[0]
            for i in grown:  # new tail pages, lowest free first, request order
                self._ptab[slots[i], lb[i]] = self._allocate_block()
            if len(grown):
                self._dirty_e.append((slots[grown].astype(np.int64), lb[grown].astype(np.int64)))
            self._npages[slots] = np.maximum(npg, lb + 1)
            items = np.zeros(len(ids), ITEM_DTYPE)
            items["page"] = self._ptab[slots, lb]
            items["src_b"] = np.arange(len(ids))
            items["dst_row"] = off
            items["n_rows"] = 1
        else:
            recs = []
            for bi, slot in enumerate(slots):
                ti, ln = 0, int(self._lens[slot])
                while ti < t:
                    lb_, off_ = divmod(ln + ti, bs)
                    if lb_ == self._npages[slot]:
                        self._ptab[slot, lb_] = self._allocate_block()
                        self._npages[slot] += 1
                        self._dirty_e.append((np.array([slot], np.int64), np.array([lb_], np.int64)))
                    n = min(t - ti, bs - off_)
                    recs.append((int(self._ptab[slot, lb_]), bi, ti, off_, n, 0, 0))
                    ti += n
            items = np.array(recs, ITEM_DTYPE)
        self._lens[slots] += t
        self._dirty_l.append(slots.astype(np.int64))
        for r in reqs:
            r.length += t
        page_update(items, k_new, v_new, self.k_quant, self.v_quant)

    def release_request(self, request_id: int) -> None:
        """paged.py:146-151: the pages return to the free list (not zeroed)."""
        req = self._requests.pop(int(request_id))
        for p in self._ptab[req.slot, : self._npages[req.slot]].tolist():
            heapq.heappush(self._free, p)
        n_old = int(self._npages[req.slot])
        self._dirty_e.append((np.full(n_old, req.slot, np.int64), np.arange(n_old, dtype=np.int64)))
        self._dirty_l.append(np.array([req.slot], np.int64))
        self._ptab[req.slot, :] = -1
        self._npages[req.slot] = 0
        self._lens[req.slot] = 0
        self._free_slots.append(req.slot)

    # -- views ---------------------------------------------------------------------------
    def block_table_numpy(self, request_ids: Sequence[int]) -> Tuple[np.ndarray, np.ndarray]:
        slots = np.fromiter((self._get(r).slot for r in request_ids), np.int64, len(request_ids))
        cols = max(1, int(self._npages[slots].max()) if len(slots) else 0)
        return self._ptab[slots, :cols].copy(), self._lens[slots].copy()

    def to_cache(self, request_ids: Optional[Sequence[int]] = None) -> PagedKVCache:
        """paged.py:153-179: table/lengths in the given request order, -1 padded.

        The slot-indexed table and lengths live on the device; a call uploads only what
        changed since the previous one (new page entries, entries of released requests
        reset to -1, changed lengths) together with the batch's slot list, in one pinned
        copy, and gathers the batch's rows on the device.  The first call, and any call
        after the host table grew, uploads the whole table."""
        ids = self.live_request_ids if request_ids is None else [int(r) for r in request_ids]
        if not ids:
            raise ValueError("to_cache needs at least one live request")
        slots = np.fromiter((self._get(r).slot for r in ids), np.int64, len(ids))
        cols = max(1, int(self._npages[slots].max()))
        max_len = int(self._lens[slots].max())
        b = len(ids)
        if self._dtab is None or tuple(self._dtab.shape) != self._ptab.shape:
            packed = np.concatenate([self._lens, self._ptab.reshape(-1), slots])
            dev = _upload(packed, self.device).view(torch.int64)
            rows = self._ptab.shape[0]
            self._dlens = dev[:rows].clone()
            self._dtab = dev[rows: rows + self._ptab.size].view(self._ptab.shape).clone()
            slots_dev = dev[rows + self._ptab.size:]
        else:
            es = np.concatenate([e[0] for e in self._dirty_e]) if self._dirty_e else np.zeros(0, np.int64)
            ec = np.concatenate([e[1] for e in self._dirty_e]) if self._dirty_e else np.zeros(0, np.int64)
            ls = np.unique(np.concatenate(self._dirty_l)) if self._dirty_l else np.zeros(0, np.int64)
            ne, nl = es.size, ls.size
            packed = np.concatenate([es, ec, self._ptab[es, ec], ls, self._lens[ls], slots])
            dev = _upload(packed, self.device).view(torch.int64)
            if ne:
                self._dtab.index_put_((dev[:ne], dev[ne:2 * ne]), dev[2 * ne:3 * ne])
            if nl:
                self._dlens.index_put_((dev[3 * ne:3 * ne + nl],), dev[3 * ne + nl:3 * ne + 2 * nl])
            slots_dev = dev[3 * ne + 2 * nl:]
        self._dirty_e.clear()
        self._dirty_l.clear()
        table = self._dtab[:, :cols].index_select(0, slots_dev)
        lengths = self._dlens.index_select(0, slots_dev)
        assert table.shape == (b, cols)
        return PagedKVCache(self.k_quant, self.v_quant, table, lengths, self.block_size, max_len)

    def stats(self) -> Dict[str, float]:
        """paged.py:181-199."""
        allocated = self.capacity_blocks - len(self._free)
        used = sum(r.length for r in self._requests.values())
        at = allocated * self.block_size
        cap = self.capacity_blocks * self.block_size
        waste = max(0, at - used)
        return {
            "allocated_blocks": float(allocated), "free_blocks": float(len(self._free)),
            "live_requests": float(len(self._requests)), "used_tokens": float(used),
            "capacity_tokens": float(cap), "block_utilization": used / max(1, at),
            "capacity_utilization": used / max(1, cap), "padding_waste": float(waste),
            "fragmentation": waste / max(1, at),
        }


def paged_cache_symmetric(k: torch.Tensor, v: torch.Tensor, page: int = 16, *, lengths: Optional[torch.Tensor] = None,
                          perm: Optional[torch.Tensor] = None) -> PagedKVCache:
    """Dense fp16/bf16 K/V [B, Hkv, S, D] -> a PagedKVCache in the symmetric per-token
    format (FS_KV_SYMMETRIC): pool values [P, Hkv, page, D] int8 and scales [P, Hkv, page]
    fp32, P = B * ceil(S / page) pages, physical page perm[j] holding logical page j of
    the batch-major order (identity when perm is None); the table is the inverse map."""
    from .quant import quantize_int8_symmetric_per_token

    if k.ndim != 4 or k.shape != v.shape:
        raise ValueError("k and v must be [batch, heads, seq_len, head_dim] of one shape")
    b, h, s_, d = (int(x) for x in k.shape)
    bps = (s_ + page - 1) // page
    total = b * bps
    pad = bps * page - s_

    def pool(x):
        if pad:
            x = torch.cat([x, x.new_zeros((b, h, pad, d))], dim=2)
        x = x.reshape(b, h, bps, page, d).permute(0, 2, 1, 3, 4).reshape(total, h, page, d)
        if perm is not None:
            x = torch.empty_like(x).index_copy_(0, perm.to(x.device), x)
        return quantize_int8_symmetric_per_token(x, page)

    table = torch.arange(total, device=k.device).view(b, bps)
    if perm is not None:
        table = perm.to(k.device).view(b, bps)
    lens = torch.full((b,), s_, dtype=torch.int64, device=k.device) if lengths is None else lengths.to(torch.int64)
    return PagedKVCache(pool(k), pool(v), table, lens, page, s_)
