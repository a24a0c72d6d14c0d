"""Decode-attention backends ``cuda_fused`` and ``cuda_paged``.

Drop-in for the reference entry points ``fused_dequant_attention_triton``
(src/flashspec/triton_fused.py:764-791) and ``paged_quant_attention_triton``
(src/flashspec/triton_paged.py:453-490): same arguments, same output dtype/shape,
same ``return_stats`` dictionary keys, same ValueError/RuntimeError split for
bad shapes / bad devices.  Differences: there is no CPU/Triton fallback (non-CUDA
inputs raise), and GQA is accepted (q heads a multiple of kv heads; q head h
reads kv head h // (Hq/Hkv)).  The math runs in ``libflashspec_b200.so``.
"""

from __future__ import annotations

import ctypes as C
import math
import os
from typing import Dict, Optional, Tuple

import torch

from . import _lib
from .quant import (QuantizedTensor, SymQuantizedTensor, build_compression_stats, estimate_quantized_bytes,
                    require_cuda, stream_of)

PAGE_TOKENS = 16  # tokens per kernel step (one page / quant block)
NUM_WARPS = 4
_workspaces: Dict[Tuple[int, int], torch.Tensor] = {}
_tickets: Dict[Tuple[int, int], torch.Tensor] = {}
_plans: Dict[tuple, Tuple[int, int]] = {}
# environment knobs the library's plan reads (decode.cu): part of the plan cache key
_PLAN_KNOBS = ("FLASHSPEC_DECODE_KERNEL", "FLASHSPEC_KERNEL_SHAPE", "FLASHSPEC_NUM_WARPS", "FLASHSPEC_TIER_SKEW",
               "FLASHSPEC_PIECE_COST")


def _workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Per (device, stream) scratch for split-K partials (contents irrelevant).  Calls
    on one stream are ordered, so they can share it."""
    key = (device.index, stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def _ticket_buffer(device: torch.device, stream: int, count: int) -> torch.Tensor:
    """Per (device, stream) split-merge counters: zero filled when allocated, and every
    completed call leaves them zero."""
    key = (device.index, stream)
    t = _tickets.get(key)
    if t is None or t.numel() < count:
        t = torch.zeros(max(count, 4096), dtype=torch.int32, device=device)
        _tickets[key] = t
    return t


def reset_workspaces() -> None:
    """Drop cached workspaces and tickets (needed after a call reported FS_DEV_TIMEOUT,
    which can leave tickets non-zero)."""
    _workspaces.clear()
    _tickets.clear()


def _env_splits() -> int:
    """FLASHSPEC_NUM_SPLITS override, as in the reference (triton_fused.py:560-601)."""
    v = os.environ.get("FLASHSPEC_NUM_SPLITS")
    if v is None:
        return 0
    try:
        n = int(v)
    except ValueError:
        return 0
    return n if n >= 1 else 0


def _validate_query(q: torch.Tensor, name: str) -> None:
    """validate_decode_query (src/flashspec/triton_utils.py:33-45)."""
    if q.ndim != 3:
        raise ValueError("q must have shape [batch, heads, head_dim]")
    if q.device.type != "cuda":
        raise RuntimeError(f"CUDA {name} attention needs a CUDA q tensor")
    if q.shape[-1] > 256:
        raise ValueError(f"CUDA {name} attention supports head_dim <= 256")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("CUDA decode attention takes fp16 or bf16 q")


def _check_gqa(hq: int, hkv: int) -> int:
    if hkv <= 0 or hq % hkv:
        raise ValueError("q heads must be a positive multiple of the kv heads")
    return hq // hkv


def _i64(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int64 and t.is_contiguous() else t.to(torch.int64).contiguous()


def _run(entry: str, args: _lib.FsDecodeArgs, device: torch.device, splits_hint: int, xargs=None) -> int:
    """Plan (cached), workspace and launch of one decode call; ``xargs`` (FsExchangeArgs)
    selects fs_paged_decode_exchange and its own plan."""
    if torch.cuda.current_device() != device.index:
        with torch.cuda.device(device):
            return _run(entry, args, device, splits_hint, xargs)
    lib = _lib.load()
    stream = stream_of(device)
    args.num_splits = splits_hint
    # the plan (workspace bytes, splits) depends on the shape fields and the env knobs
    key = (device.index, args.layout, args.batch, args.q_heads, args.kv_heads, args.head_dim, args.block_size,
           args.page_size, args.num_blocks, args.table_cols, args.max_seq_len, args.num_splits, args.page_begin,
           args.page_end, bool(args.shard_o), args.q_dtype, args.kv_format, entry,
           tuple(os.environ.get(k) for k in _PLAN_KNOBS))
    plan = _plans.get(key)
    if plan is None:
        nbytes = C.c_size_t(0)
        splits = C.c_int32(0)
        size_fn = lib.fs_paged_decode_exchange_workspace_size if xargs is not None else lib.fs_decode_workspace_size
        _lib.check(size_fn(C.byref(args), C.byref(nbytes), C.byref(splits)), entry)
        plan = _plans[key] = (nbytes.value, splits.value)
        if len(_plans) > 256:
            _plans.pop(next(iter(_plans)))
    nbytes = C.c_size_t(plan[0])
    splits = C.c_int32(plan[1])
    if nbytes.value:
        ws = _workspace(device, stream, nbytes.value)
        args.workspace = ws.data_ptr()
        args.workspace_bytes = ws.numel()
        tk = _ticket_buffer(device, stream, args.batch * args.kv_heads)
        args.tickets = tk.data_ptr()
        args.ticket_count = tk.numel()
    if xargs is not None:
        _lib.check(getattr(lib, entry)(C.byref(args), C.byref(xargs), stream), entry)
    else:
        _lib.check(getattr(lib, entry)(C.byref(args), stream), entry)
    return splits.value


def _decode_args(layout, q, kq, vq, out, lengths, table, num_blocks, max_seq_len, hkv, status,
                 page_size: int = 0) -> _lib.FsDecodeArgs:
    a = _lib.FsDecodeArgs()
    a.layout = layout
    a.q = q.data_ptr()
    sym = bool(getattr(kq, "symmetric", False))
    if sym != bool(getattr(vq, "symmetric", False)):
        raise ValueError("K and V must use the same quantization format")
    a.kv_format = _lib.FS_KV_SYMMETRIC if sym else _lib.FS_KV_AFFINE_BLOCK
    a.k_values, a.k_scale = kq.values.data_ptr(), kq.scale.data_ptr()
    a.v_values, a.v_scale = vq.values.data_ptr(), vq.scale.data_ptr()
    if not sym:
        a.k_zero, a.v_zero = kq.zero_point.data_ptr(), vq.zero_point.data_ptr()
    a.block_table = table.data_ptr() if table is not None else None
    a.lengths = lengths.data_ptr() if lengths is not None else None
    a.out = out.data_ptr() if out is not None else None
    a.batch, a.q_heads, a.kv_heads, a.head_dim = q.shape[0], q.shape[1], hkv, q.shape[2]
    a.block_size = int(kq.block_size)
    a.num_blocks = num_blocks
    a.table_cols = table.shape[1] if table is not None else 0
    a.max_seq_len = max_seq_len
    a.sm_scale = 1.0 / math.sqrt(float(q.shape[2]))
    a.device_status = status.data_ptr() if status is not None else None
    a.q_dtype = _lib.FS_BF16 if q.dtype == torch.bfloat16 else _lib.FS_F16
    a.page_size = int(page_size)
    return a


def _contig_quant(qt):
    if getattr(qt, "symmetric", False):
        return SymQuantizedTensor(qt.values.contiguous(), qt.scale.contiguous(), int(qt.block_size),
                                  tuple(qt.original_shape))
    return QuantizedTensor(qt.values.contiguous(), qt.scale.contiguous(), qt.zero_point.contiguous(),
                           int(qt.block_size), tuple(qt.original_shape))


def fused_dequant_attention_cuda(q: torch.Tensor, k_quant, v_quant, lengths: Optional[torch.Tensor] = None,
                                 return_stats: bool = False, *, num_splits: Optional[int] = None,
                                 device_status: Optional[torch.Tensor] = None):
    """Contiguous INT8 KV decode attention (backend ``cuda_fused``).

    q [B, Hq, D] fp16 or bf16 (out has q's dtype); k_quant/v_quant quantized from
    [B, Hkv, S, D] (head_dim 32/64/128/256, quant block up to 64 tokens); optional
    lengths int64 [B] (None = every request uses S).
    Validation follows _validate_triton_fused_inputs (triton_fused.py:506-548)."""
    _validate_query(q, "fused")
    if len(k_quant.original_shape) != 4 or len(v_quant.original_shape) != 4:
        raise ValueError("k_quant and v_quant must come from [batch, heads, seq_len, head_dim] tensors")
    if tuple(k_quant.original_shape) != tuple(v_quant.original_shape):
        raise ValueError("k_quant and v_quant original_shape differ")
    b, hkv, seq, d = (int(x) for x in k_quant.original_shape)
    if q.shape[0] != b or q.shape[2] != d:
        raise ValueError("q batch / head_dim must match the quantized K/V")
    _check_gqa(q.shape[1], hkv)
    if k_quant.values.device != q.device or v_quant.values.device != q.device:
        raise RuntimeError("q, k_quant and v_quant must be on the same CUDA device")
    if lengths is not None:
        if lengths.ndim != 1 or lengths.shape[0] != b:
            raise ValueError("lengths must have shape [batch]")
        if lengths.device != q.device:
            raise RuntimeError("lengths must be on q's CUDA device")
        lengths = _i64(lengths)
    kq, vq = _contig_quant(k_quant), _contig_quant(v_quant)
    # quant blocks per (request, kv head); the symmetric format stores [.., S_pad, D]
    nblk = (int(kq.values.shape[-2]) // int(kq.block_size) if getattr(kq, "symmetric", False)
            else int(kq.values.shape[-3]))
    qc = q.contiguous()
    out = torch.empty_like(qc)
    a = _decode_args(_lib.FS_LAYOUT_CONTIGUOUS, qc, kq, vq, out, lengths, None, nblk, seq, hkv, device_status)
    splits = _run("fs_fused_decode", a, q.device, num_splits or _env_splits())
    if not return_stats:
        return out
    dense = 2 * b * hkv * seq * d * qc.element_size()
    quant = estimate_quantized_bytes(kq) + estimate_quantized_bytes(vq)
    return out, build_compression_stats(dense, quant, materializes_dense_kv=False, num_splits=splits,
                                        block_n=int(kq.block_size), num_warps=NUM_WARPS)


def paged_quant_attention_cuda(q: torch.Tensor, cache, return_stats: bool = False, *,
                               num_splits: Optional[int] = None, page_range: Optional[Tuple[int, int]] = None,
                               partial_out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                               device_status: Optional[torch.Tensor] = None, exchange=None):
    """Paged INT8 KV decode attention (backend ``cuda_paged``).

    ``cache`` is a PagedKVCache (this package's or the reference's): pool
    [P, Hkv, page / qb, qb, D] int8 + fp32/int16 qparams per quant block of qb tokens
    (the page a multiple of qb), block_table int64 [B, cols] (-1 = unallocated),
    lengths int64 [B], max_seq_len; q fp16 or bf16.  Validation follows
    _validate_triton_paged_inputs (triton_paged.py:302-335).

    Extensions used by sequence sharding: ``page_range=(lo, hi)`` restricts every
    request to logical pages [lo, hi); ``partial_out=(O fp32 [B,Hq,D], LSE fp32
    [B,Hq])`` receives the normalised partial result and its log-sum-exp instead
    of the fp16 output (None is returned then); ``exchange=(FsExchangeArgs, out)``
    runs the window's decode with the fused exchange epilogue
    (``fs_paged_decode_exchange``): every rank's rows are merged into ``out`` (fp16 or
    fp32 [B, Hq, D]), which is returned."""
    _validate_query(q, "paged")
    kq, vq = cache.k_quant, cache.v_quant
    hkv = int(kq.original_shape[1])
    d = int(kq.original_shape[-1])
    if q.shape[0] != cache.block_table.shape[0] or q.shape[2] != d:
        raise ValueError("q batch / head_dim must match the PagedKVCache")
    _check_gqa(q.shape[1], hkv)
    if tuple(kq.original_shape) != tuple(vq.original_shape):
        raise ValueError("cache.k_quant and cache.v_quant original_shape differ")
    if len(kq.original_shape) != 4:
        raise ValueError("PagedKVCache k_quant/v_quant must come from [physical, heads, block, head_dim] tensors")
    if int(kq.original_shape[2]) != int(cache.block_size):
        raise ValueError("physical block sequence length must equal cache.block_size")
    if int(kq.block_size) != int(vq.block_size):
        raise ValueError("K/V quantization block_size differ")
    if int(cache.block_size) % int(kq.block_size) != 0:
        raise ValueError("cache.block_size must be a multiple of the quantization block_size")
    if kq.values.device != q.device or vq.values.device != q.device:
        raise RuntimeError("q and the cache's quantized K/V must be on the same CUDA device")
    if cache.block_table.device != q.device or cache.lengths.device != q.device:
        raise RuntimeError("block_table and lengths must be on q's CUDA device")
    kq, vq = _contig_quant(kq), _contig_quant(vq)
    table = _i64(cache.block_table)
    lengths = _i64(cache.lengths)
    qc = q.contiguous()
    num_pages = int(kq.values.shape[0])
    out = None
    if exchange is not None:
        if partial_out is not None:
            raise ValueError("exchange and partial_out are exclusive")
        xargs, out = exchange
        if tuple(out.shape) != tuple(qc.shape) or out.dtype not in (torch.float16, torch.float32) \
                or not out.is_contiguous() or out.device != q.device:
            raise ValueError("exchange output must be a contiguous fp16/fp32 [B, Hq, D] tensor on q's device")
        xargs.out = out.data_ptr()
        xargs.out_dtype = _lib.FS_F16 if out.dtype == torch.float16 else _lib.FS_F32
    elif partial_out is None:
        out = torch.empty_like(qc)
    a = _decode_args(_lib.FS_LAYOUT_PAGED, qc, kq, vq, out, lengths, table, num_pages, int(cache.max_seq_len),
                     hkv, device_status, page_size=int(cache.block_size))
    if page_range is not None:
        a.page_begin, a.page_end = int(page_range[0]), int(page_range[1])
    if partial_out is not None:
        o, lse = partial_out
        if o.dtype != torch.float32 or lse.dtype != torch.float32 or not (o.is_contiguous() and lse.is_contiguous()):
            raise ValueError("partial_out must be contiguous fp32 tensors")
        if tuple(o.shape) != tuple(qc.shape) or tuple(lse.shape) != tuple(qc.shape[:2]):
            raise ValueError("partial_out shapes must be [B, Hq, D] and [B, Hq]")
        a.shard_o, a.shard_lse = o.data_ptr(), lse.data_ptr()
    if exchange is not None:
        a.out = None
        splits = _run("fs_paged_decode_exchange", a, q.device, num_splits or _env_splits(), exchange[0])
    else:
        splits = _run("fs_paged_decode", a, q.device, num_splits or _env_splits())
    if not return_stats:
        return out
    dense = 2 * q.shape[0] * hkv * int(cache.max_seq_len) * d * qc.element_size()
    stats = build_compression_stats(dense, cache.estimated_bytes(), materializes_dense_kv=False,
                                    physical_blocks=float(cache.block_table.ge(0).sum().item()),
                                    num_splits=splits, block_n=int(kq.block_size), num_warps=NUM_WARPS)
    return out, stats


def merge_partials(o_parts: torch.Tensor, lse_parts: torch.Tensor, out_dtype: torch.dtype = torch.float16):
    """LSE merge of stacked partials o [N, ..., D] fp32 / lse [N, ...] fp32 (split-K or
    per-GPU shards) -> [..., D]; same math as _combine_splits_kernel
    (triton_fused.py:446-503)."""
    require_cuda(o_parts, "o_parts")
    if o_parts.dtype != torch.float32 or lse_parts.dtype != torch.float32:
        raise ValueError("partials must be fp32")
    n, d = o_parts.shape[0], o_parts.shape[-1]
    if tuple(lse_parts.shape) != tuple(o_parts.shape[:-1]):
        raise ValueError("lse_parts must match o_parts without the last dim")
    rows = lse_parts[0].numel()
    oc, lc = o_parts.contiguous(), lse_parts.contiguous()
    out = torch.empty(o_parts.shape[1:], dtype=out_dtype, device=o_parts.device)
    code = {torch.float16: _lib.FS_F16, torch.bfloat16: _lib.FS_BF16, torch.float32: _lib.FS_F32}[out_dtype]
    with torch.cuda.device(o_parts.device):
        _lib.check(_lib.load().fs_merge_partials(oc.data_ptr(), lc.data_ptr(), n, rows, d, 0, out.data_ptr(), code,
                                                 stream_of(o_parts.device)), "fs_merge_partials")
    return out


BACKENDS = {
    "cuda_fused": fused_dequant_attention_cuda,
    "cuda_paged": paged_quant_attention_cuda,
}


def register_backend(name: str, fn) -> None:
    """Add an attention backend under ``name`` (the microbench --backend key)."""
    BACKENDS[name] = fn


def get_backend(name: str):
    try:
        return BACKENDS[name]
    except KeyError:
        raise ValueError(f"unknown backend {name!r}; known: {sorted(BACKENDS)}") from None
