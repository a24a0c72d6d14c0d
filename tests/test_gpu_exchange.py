"""The peer-memory exchange of sequence-sharded decode steps (fs_exchange_*).

On one GPU: a one-rank exchange must give exactly fs_merge_partials' result, call
after call, and a two-rank exchange whose peer never arrives must give up within its
time limit, say so in the status word and write NaN (the GPU stays usable).  With two
GPUs: two ranks (child processes, gloo for the handle exchange) decode their page
windows and merge through the exchange, eagerly and as CUDA-graph replays, and must
match the CPU oracle on the whole sequence."""

from __future__ import annotations

import ctypes as C
import os
import socket
import sys
import tempfile
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
ATOL, RTOL = 2e-3, 1e-2

pytestmark = pytest.mark.gpu


def _need_gpu(n=1):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} CUDA device(s)")


def _partial(seed=0):
    import flashspec_b200 as fs
    from flashspec_b200 import configs

    wl = configs.paged_workload("xch", 2, 16, 2, [900, 301], seed=seed, device="cuda")
    o = torch.empty(wl.q.shape, dtype=torch.float32, device="cuda")
    lse = torch.empty(wl.q.shape[:2], dtype=torch.float32, device="cuda")
    fs.paged_quant_attention_cuda(wl.q, wl.cache, partial_out=(o, lse))
    return wl, o, lse


def _create(lib, slot):
    from flashspec_b200 import _lib

    buf, h = C.c_void_p(), (C.c_char * _lib.EXCHANGE_HANDLE_BYTES)()
    assert lib.fs_exchange_create(slot, C.byref(buf), h) == 0
    return buf.value


def test_one_rank_exchange_equals_merge_partials_on_consecutive_calls():
    _need_gpu()
    import flashspec_b200 as fs
    from flashspec_b200 import _lib

    lib = _lib.load()
    wl, o, lse = _partial()
    rows, d = lse.numel(), o.shape[-1]
    slot = (rows * (d + 1) + 63) // 64 * 64
    ref = fs.merge_partials(o[None], lse[None], torch.float16)
    buf = _create(lib, slot)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        a = _lib.FsExchangeArgs()
        a.world, a.rank = 1, 0
        a.bufs[0] = buf
        a.slot_floats, a.rows, a.head_dim = slot, rows, d
        a.o_mine, a.lse_mine = o.data_ptr(), lse.data_ptr()
        a.out_dtype, a.timeout_ns, a.device_status = _lib.FS_F16, 10**9, status.data_ptr()
        stream = torch.cuda.current_stream().cuda_stream
        for _ in range(3):  # the call counter advances; every call must be complete
            out = torch.full_like(wl.q, float("nan"))
            a.out = out.data_ptr()
            assert lib.fs_exchange_merge(C.byref(a), stream) == 0
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert torch.equal(out, ref)
    finally:
        torch.cuda.synchronize()
        lib.fs_exchange_destroy(buf)


def test_missing_peer_times_out_and_reports():
    """Rank 0 of a two-rank exchange whose rank 1 never runs: the kernel waits for the
    peer's tagged words, which nothing writes, gives up after 20 ms, sets FS_DEV_TIMEOUT
    and writes NaN rather than a partial merge; a second call on the same buffers does
    the same (its epoch has moved on, the peer's has not), and the device stays usable."""
    _need_gpu()
    from flashspec_b200 import _lib

    lib = _lib.load()
    wl, o, lse = _partial()
    rows, d = lse.numel(), o.shape[-1]
    slot = (rows * (d + 1) + 63) // 64 * 64
    mine, silent_peer = _create(lib, slot), _create(lib, slot)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        a = _lib.FsExchangeArgs()
        a.world, a.rank = 2, 0
        a.bufs[0], a.bufs[1] = mine, silent_peer
        a.slot_floats, a.rows, a.head_dim = slot, rows, d
        a.o_mine, a.lse_mine = o.data_ptr(), lse.data_ptr()
        a.out_dtype = _lib.FS_F16
        a.timeout_ns, a.device_status = 20 * 10**6, status.data_ptr()
        for _ in range(2):
            status.zero_()
            out = torch.zeros_like(wl.q)
            a.out = out.data_ptr()
            assert lib.fs_exchange_merge(C.byref(a), torch.cuda.current_stream().cuda_stream) == 0
            torch.cuda.synchronize()
            assert int(status.item()) & _lib.FS_DEV_TIMEOUT
            assert bool(torch.isnan(out).all()), "a timed-out merge must not return values"
        assert float(torch.ones(4, device="cuda").sum()) == 4.0  # context still usable
        # a slot size other than the buffers were created with is refused before launch
        a.slot_floats = slot + 64
        assert lib.fs_exchange_merge(C.byref(a), torch.cuda.current_stream().cuda_stream) == 1
    finally:
        torch.cuda.synchronize()
        lib.fs_exchange_destroy(mine)
        lib.fs_exchange_destroy(silent_peer)


def _fused_call(lib, wl, bufs, rank, slot, out, status, timeout_ns, num_splits):
    """fs_paged_decode_exchange through the C ABI: the whole window (every page) of wl."""
    import flashspec_b200 as fs
    from flashspec_b200 import _lib

    x = _lib.FsExchangeArgs()
    x.world, x.rank = len(bufs), rank
    for r, b in enumerate(bufs):
        x.bufs[r] = b
    x.slot_floats, x.timeout_ns, x.device_status = slot, timeout_ns, status.data_ptr()
    fs.paged_quant_attention_cuda(wl.q, wl.cache, num_splits=num_splits, exchange=(x, out))


@pytest.mark.parametrize("num_splits", [1, 3])
def test_fused_one_rank_exchange_equals_paged_decode(num_splits):
    """With one rank the fused decode + exchange epilogue merges a single partial with
    weight 1, so its fp16 output must equal fs_paged_decode's bit for bit (same splits),
    call after call as the per-pair epoch advances; fp32 output must round to it."""
    _need_gpu()
    import flashspec_b200 as fs
    from flashspec_b200 import _lib

    lib = _lib.load()
    wl, o, lse = _partial()
    rows, d = lse.numel(), o.shape[-1]
    slot = (rows * (d + 1) + 63) // 64 * 64
    ref = fs.paged_quant_attention_cuda(wl.q, wl.cache, num_splits=num_splits)
    buf = _create(lib, slot)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        for _ in range(3):
            out = torch.full_like(wl.q, float("nan"))
            _fused_call(lib, wl, [buf], 0, slot, out, status, 10**9, num_splits)
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert torch.equal(out, ref)
        out32 = torch.full(wl.q.shape, float("nan"), dtype=torch.float32, device="cuda")
        _fused_call(lib, wl, [buf], 0, slot, out32, status, 10**9, num_splits)
        torch.cuda.synchronize()
        assert torch.equal(out32.half(), ref)
    finally:
        torch.cuda.synchronize()
        lib.fs_exchange_destroy(buf)


def test_fused_missing_peer_times_out_and_reports():
    """Rank 0 of a two-rank fused step whose rank 1 never runs: each pair's epilogue
    waits for the peer's tagged words, which nothing writes, gives up after 20 ms, sets
    FS_DEV_TIMEOUT and writes NaN; again on a second call; the device stays usable, and
    buffers of another slot size are refused before launch."""
    _need_gpu()
    from flashspec_b200 import _lib

    lib = _lib.load()
    wl, o, lse = _partial()
    rows, d = lse.numel(), o.shape[-1]
    slot = (rows * (d + 1) + 63) // 64 * 64
    mine, silent_peer = _create(lib, slot), _create(lib, slot)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        for _ in range(2):
            status.zero_()
            out = torch.zeros_like(wl.q)
            _fused_call(lib, wl, [mine, silent_peer], 0, slot, out, status, 20 * 10**6, 2)
            torch.cuda.synchronize()
            assert int(status.item()) & _lib.FS_DEV_TIMEOUT
            assert bool(torch.isnan(out).all()), "a timed-out step must not return values"
        assert float(torch.ones(4, device="cuda").sum()) == 4.0
        with pytest.raises(ValueError, match="status 1"):
            _fused_call(lib, wl, [mine, silent_peer], 0, slot + 64, torch.zeros_like(wl.q), status, 20 * 10**6, 2)
    finally:
        torch.cuda.synchronize()
        lib.fs_exchange_destroy(mine)
        lib.fs_exchange_destroy(silent_peer)


def test_decoder_check_raises_after_a_timeout():
    """PeerExchange.check() turns FS_DEV_TIMEOUT into an exception on the host."""
    _need_gpu()
    from flashspec_b200 import _lib
    from flashspec_b200.dist import PeerExchange

    x = PeerExchange.__new__(PeerExchange)
    x.rank = 0
    x.status = torch.tensor([_lib.FS_DEV_TIMEOUT], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="timed out"):
        x.check()
    x.status.zero_()
    x.check()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, transport):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    from flashspec_b200 import configs
    from flashspec_b200.dist import SequenceShardedDecoder

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path.insert(0, str(ROOT / "oracle"))
    import flashspec_oracle as O

    wl = configs.paged_workload("xch2", 2, 16, 2, [3000, 1301], seed=5, device=f"cuda:{rank}")
    n_pages = int(wl.cache.block_table.shape[1])

    def oq(t):
        return O.OQuant(t.values.cpu().numpy(), t.scale.cpu().numpy(), t.zero_point.cpu().numpy(), 16,
                        tuple(t.original_shape))

    oc = O.OPagedCache(oq(wl.cache.k_quant), oq(wl.cache.v_quant), wl.cache.block_table.cpu().numpy(),
                       wl.cache.lengths.cpu().numpy(), 16, int(wl.cache.max_seq_len))
    full = torch.from_numpy(O.paged_quant_attention(wl.q.cpu().numpy(), oc).astype("float32")).to(wl.q.device)
    dec = SequenceShardedDecoder(transport=transport)
    errs = []
    for _ in range(3):
        out = dec(wl.q, wl.cache, n_pages)
        errs.append(float(((out.float() - full.float()).abs() - RTOL * full.float().abs()).max()))
    replay, gout = dec.capture(wl.q, wl.cache, n_pages)
    for _ in range(3):
        replay()
        torch.cuda.synchronize()
        errs.append(float(((gout.float() - full.float()).abs() - RTOL * full.float().abs()).max()))
    torch.cuda.synchronize()
    status = [int(x.status.item()) for x in dec._xch.values()]
    modes = sorted({k[2] for k in dec._xch})
    assert modes == (["fused"] if transport == "p2p" else ["kernel"]), modes
    (Path(out_dir) / f"rank{rank}.txt").write_text(f"{max(errs)} {max(status)}")
    dec.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["p2p", "p2p_kernel"])
def test_two_ranks_match_the_oracle(transport):
    """Two ranks (one GPU each) decode their page windows and exchange; rank r's merged
    output must match the CPU oracle on the whole sequence, eagerly and replayed from a
    CUDA graph, with the fused epilogue ("p2p") and with the separate exchange kernel."""
    _need_gpu(2)
    import torch.multiprocessing as mp

    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_rank_main, args=(r, 2, port, d, transport)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            if p.is_alive():
                p.kill()
        assert [p.exitcode for p in procs] == [0, 0]
        for r in range(2):
            err, status = (Path(d) / f"rank{r}.txt").read_text().split()
            assert float(err) <= ATOL and int(status) == 0, (r, err, status)
