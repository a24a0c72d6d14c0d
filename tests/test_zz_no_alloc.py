"""The allocation-free paged decode entry point, called through the C ABI.

fs_paged_decode_noalloc exists for callers that cannot give the library device
memory and must not see it allocate any (a plugin whose host owns all device
allocations, a loop that cannot afford cudaMalloc's implicit synchronisation).  It
must give the same result as fs_paged_decode with a caller-provided workspace, call
after call, although its scratch array keeps the previous call's contents.

This file is named to be collected last, so a run that stops at the first failure
has already run every other test."""

from __future__ import annotations

import ctypes as C
import math

import numpy as np
import pytest
import torch

ATOL, RTOL = 2e-3, 1e-2


def _args(q, cache, out, num_splits):
    from flashspec_b200 import _lib

    a = _lib.FsDecodeArgs()
    a.layout = _lib.FS_LAYOUT_PAGED
    a.q = q.data_ptr()
    kq, vq = cache["k"], cache["v"]
    a.k_values, a.k_scale, a.k_zero = kq[0].data_ptr(), kq[1].data_ptr(), kq[2].data_ptr()
    a.v_values, a.v_scale, a.v_zero = vq[0].data_ptr(), vq[1].data_ptr(), vq[2].data_ptr()
    a.block_table = cache["table"].data_ptr()
    a.lengths = cache["lengths"].data_ptr()
    a.out = out.data_ptr()
    a.batch, a.q_heads, a.kv_heads, a.head_dim, a.block_size = q.shape[0], q.shape[1], kq[0].shape[1], 128, 16
    a.num_blocks = kq[0].shape[0]
    a.table_cols = cache["table"].shape[1]
    a.max_seq_len = cache["max_seq_len"]
    a.num_splits = num_splits
    a.sm_scale = 1.0 / math.sqrt(128.0)
    return a


def _workload(seed=3, b=5, hq=8, hkv=4):
    import flashspec_b200 as fs

    g = torch.Generator(device="cuda").manual_seed(seed)
    lengths = [700, 33, 512, 129, 1]
    pages = [(n + 15) // 16 for n in lengths]
    pool = sum(pages) + 7
    kq = fs.quantize_int8_per_block(torch.randn(pool, hkv, 16, 128, generator=g, device="cuda",
                                                dtype=torch.float16), 16)
    vq = fs.quantize_int8_per_block(torch.randn(pool, hkv, 16, 128, generator=g, device="cuda",
                                                dtype=torch.float16), 16)
    perm = torch.randperm(pool, generator=torch.Generator().manual_seed(seed))
    table = torch.full((b, max(pages)), -1, dtype=torch.int64)
    pos = 0
    for i, n in enumerate(pages):
        table[i, :n] = perm[pos:pos + n]
        pos += n
    q = torch.randn(b, hq, 128, generator=g, device="cuda", dtype=torch.float16)
    cache = {"k": (kq.values, kq.scale, kq.zero_point), "v": (vq.values, vq.scale, vq.zero_point),
             "table": table.cuda(), "lengths": torch.tensor(lengths, dtype=torch.int64, device="cuda"),
             "max_seq_len": max(lengths)}
    return q, cache


def _close(got, ref):
    ref = torch.as_tensor(np.asarray(ref, dtype=np.float32)) if not torch.is_tensor(ref) else ref.float().cpu()
    err = (got.float().cpu() - ref).abs()
    assert bool(torch.all(err <= ATOL + RTOL * ref.abs())), f"max abs err {err.max().item():.3e}"


def _oracle(q, cache):
    """The CPU oracle's paged attention on the same quantized pool and table."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
    import flashspec_oracle as O

    def oq(t):
        v, s, z = (x.cpu().numpy() for x in t)
        return O.OQuant(v, s, z, 16, (v.shape[0], v.shape[1], 16, 128))

    oc = O.OPagedCache(oq(cache["k"]), oq(cache["v"]), cache["table"].cpu().numpy(),
                       cache["lengths"].cpu().numpy(), 16, cache["max_seq_len"])
    return O.paged_quant_attention(q.cpu().numpy(), oc)


def _noalloc_twice(lib, q, cache, splits):
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):  # the second call sees the first call's leftovers in the scratch
        out = torch.full_like(q, float("nan"))
        assert lib.fs_paged_decode_noalloc(C.byref(_args(q, cache, out, splits)), stream) == 0
        outs.append(out)
    torch.cuda.synchronize()
    return outs


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from flashspec_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    q, cache = _workload()
    splits = 4  # forces the split-K path, i.e. the scratch memory
    expected = _oracle(q, cache)

    ref = torch.empty_like(q)
    a = _args(q, cache, ref, splits)
    nbytes, s = C.c_size_t(0), C.c_int32(0)
    assert lib.fs_decode_workspace_size(C.byref(a), C.byref(nbytes), C.byref(s)) == 0
    assert s.value == splits and nbytes.value > 0
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    tickets = torch.zeros(q.shape[0] * 4, dtype=torch.int32, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.tickets, a.ticket_count = tickets.data_ptr(), tickets.numel()
    assert lib.fs_paged_decode(C.byref(a), stream) == 0
    torch.cuda.synchronize()
    _close(ref, expected)

    for out in _noalloc_twice(lib, q, cache, splits):
        assert not torch.isnan(out).any()
        _close(out, ref)
        _close(out, expected)
    # the library's automatic split count goes through the same scratch
    (out, _) = _noalloc_twice(lib, q, cache, 0)
    _close(out, expected)


@pytest.mark.gpu
def test_noalloc_balanced_kernel_vs_oracle(monkeypatch):
    """The balanced (stream-K) kernel merges the pieces of pairs that several warps
    share through the same counters; through the fixed scratch it must clear them
    itself before every call."""
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from flashspec_b200 import _lib

    lib = _lib.load()
    q, cache = _workload(seed=11, b=5, hq=16, hkv=2)
    expected = _oracle(q, cache)
    monkeypatch.setenv("FLASHSPEC_DECODE_KERNEL", "balanced")
    a = _args(q, cache, torch.empty_like(q), 0)
    nbytes, s = C.c_size_t(0), C.c_int32(0)
    assert lib.fs_decode_workspace_size(C.byref(a), C.byref(nbytes), C.byref(s)) == 0
    assert s.value == 0 and nbytes.value > 0  # the balanced plan
    # a split call first leaves its own partials behind in the shared scratch
    _noalloc_twice(lib, q, cache, 7)
    for out in _noalloc_twice(lib, q, cache, 0):
        assert not torch.isnan(out).any()
        _close(out, expected)


def test_noalloc_rejects_requests_beyond_its_scratch():
    """Checked before any CUDA call, so this runs without a GPU."""
    from flashspec_b200 import _lib

    lib = _lib.load()
    a = _lib.FsDecodeArgs()
    a.layout = _lib.FS_LAYOUT_PAGED
    a.batch, a.q_heads, a.kv_heads, a.head_dim, a.block_size = 64, 32, 8, 128, 16
    a.num_splits = 64  # 64*8*64*4 partial rows * 516 B > 8 MiB
    assert lib.fs_paged_decode_noalloc(C.byref(a), None) == 6
    assert b"scratch" in lib.fs_status_string(6)
    a.batch, a.kv_heads, a.q_heads, a.num_splits = 70000, 1, 1, 1  # more counters than it holds
    assert lib.fs_paged_decode_noalloc(C.byref(a), None) == 6
