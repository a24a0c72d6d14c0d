"""Multi-GPU decode: one process per GPU, torch.distributed for the plumbing.

Two strategies (the reference has no multi-GPU path):

* request x kv-head sharding (configs 0, 1, 2, 4): every rank owns whole requests
  and runs the single-GPU kernel on them.  No communication; see ``request_shard``.
* sequence sharding of long requests (config 3): rank r owns the contiguous logical
  pages ``page_window(n_pages, r, N)`` of every request and only those pages are
  resident on it.  By default one kernel per step (``fs_paged_decode_exchange``): the
  decode of the rank's window whose epilogue -- the CTA that finishes a (request, kv
  head) pair -- stores the pair's normalised (O, LSE) rows into every rank's exchange
  buffer over NVLink and merges all ranks' rows with the log-sum-exp rule, the same
  math as the split-K combine (src/flashspec/triton_fused.py:446-503) applied across
  GPUs.  ``transport="p2p_kernel"`` runs the decode into (O, LSE) and a separate
  exchange kernel (``fs_exchange_merge``); ``transport="nccl"`` an all-gather +
  ``fs_merge_partials``.
"""

from __future__ import annotations

import os

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def page_window(n_pages: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous logical page range [lo, hi) of ``rank`` (balanced to one page)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    return (n_pages * rank) // world, (n_pages * (rank + 1)) // world


def request_shard(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Assign requests to ranks balancing tokens (greedy longest first), the
    communication-free sharding of ragged batches."""
    order = sorted(range(len(lengths)), key=lambda i: -int(lengths[i]))
    load = [0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(x) for x in out]


def _cuda_partial(q, cache, window):
    from .attention import paged_quant_attention_cuda

    o = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.empty(q.shape[:2], dtype=torch.float32, device=q.device)
    paged_quant_attention_cuda(q, cache, page_range=window, partial_out=(o, lse))
    return o, lse


def _cuda_merge(o_parts, lse_parts, out_dtype):
    from .attention import merge_partials

    return merge_partials(o_parts, lse_parts, out_dtype)


class PeerExchange:
    """The exchange buffers of one group of ranks (one process per GPU of a node): this
    rank's own, created by the library, and every peer's, mapped through its CUDA IPC
    handle (handles travel once through ``torch.distributed.all_gather_object``).
    ``merge`` runs ``fs_exchange_merge``: this rank's partial rows go to every rank over
    NVLink and the merged rows come back in ``out``, with no collective-library call."""

    def __init__(self, group, device: torch.device, slot_floats: int, timeout_ns: int):
        import ctypes as C

        from . import _lib

        self._lib = _lib.load()
        self.device = device
        self.slot_floats = slot_floats
        self.timeout_ns = timeout_ns
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _lib.EXCHANGE_MAX_RANKS:
            raise ValueError(f"the peer exchange serves at most {_lib.EXCHANGE_MAX_RANKS} ranks")
        own = C.c_void_p()
        handle = (C.c_char * _lib.EXCHANGE_HANDLE_BYTES)()
        with torch.cuda.device(device):
            _lib.check(self._lib.fs_exchange_create(slot_floats, C.byref(own), handle), "fs_exchange_create")
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._peers = []
        bufs = []
        with torch.cuda.device(device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bufs.append(self._own)
                    continue
                hb = (C.c_char * _lib.EXCHANGE_HANDLE_BYTES).from_buffer_copy(h)
                p = C.c_void_p()
                _lib.check(self._lib.fs_exchange_open(hb, C.byref(p)), "fs_exchange_open")
                self._peers.append(p.value)
                bufs.append(p.value)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self._args = _lib.FsExchangeArgs()
        self._args.world, self._args.rank = self.world, self.rank
        for r, b in enumerate(bufs):
            self._args.bufs[r] = b
        self._args.slot_floats = slot_floats
        self._args.timeout_ns = timeout_ns
        self._args.device_status = self.status.data_ptr()

    def merge(self, o: torch.Tensor, lse: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        import ctypes as C

        from . import _lib
        from .quant import stream_of

        a = self._args
        a.o_mine, a.lse_mine = o.data_ptr(), lse.data_ptr()
        a.rows, a.head_dim = lse.numel(), o.shape[-1]
        a.out = out.data_ptr()
        a.out_dtype = {torch.float16: _lib.FS_F16, torch.float32: _lib.FS_F32}[out.dtype]
        _lib.check(self._lib.fs_exchange_merge(C.byref(a), stream_of(self.device)), "fs_exchange_merge")
        return out

    def decode(self, q: torch.Tensor, cache, window: Tuple[int, int], out: torch.Tensor) -> torch.Tensor:
        """The whole step in one kernel (``fs_paged_decode_exchange``): decode of this
        rank's page window whose epilogue stores the rows to every rank and merges them
        into ``out``.  A set of buffers serves either this or ``merge``, not both."""
        from .attention import paged_quant_attention_cuda

        return paged_quant_attention_cuda(q, cache, page_range=window, exchange=(self._args, out))

    def check(self) -> None:
        """Raise if any merge so far gave up waiting for a peer (FS_DEV_TIMEOUT in the
        status word).  Waits for this device's queued work.  A timed-out call wrote NaN
        to the rows it could not merge, and the ranks' call counters may now disagree,
        so the group must close its exchange (collectively) and create a new one."""
        from . import _lib

        st = int(self.status.item())
        if st & _lib.FS_DEV_TIMEOUT:
            raise RuntimeError(f"peer exchange on rank {self.rank} timed out waiting for a peer (status {st}); "
                               "close the decoder's exchange on every rank and recreate it")

    def close_peers(self) -> None:
        """Unmap the peers' buffers (this rank stops addressing them)."""
        with torch.cuda.device(self.device):
            for p in self._peers:
                self._lib.fs_exchange_close(p)
        self._peers = []

    def destroy(self) -> None:
        """Free this rank's own buffer: only after every peer has unmapped it."""
        with torch.cuda.device(self.device):
            if self._own:
                self._lib.fs_exchange_destroy(self._own)
                self._own = None

    def close(self) -> None:
        """Single-process teardown (no peer holds this rank's buffer)."""
        self.close_peers()
        self.destroy()


class SequenceShardedDecoder:
    """Decode one batch whose KV pages are split across the ranks of ``group``.

    Default (CUDA) path per call, with more than one rank: transport "p2p" runs the
    decode of the rank's window with the fused exchange epilogue (one kernel; shapes it
    does not take fall back to "p2p_kernel"); "p2p_kernel" writes the rank's partial
    (O, LSE) into a preallocated [O | LSE] fp32 buffer and the peer-memory exchange
    (``PeerExchange.merge``) delivers every rank's rows to every rank and merges them
    into the fp16 output; or (transport "nccl", also
    ``FLASHSPEC_EXCHANGE=nccl``) an out-of-place ``all_gather_into_tensor`` collects the
    slots and ``fs_merge_partials`` merges them.  ``capture`` records the whole step as a
    CUDA graph (single-rank groups, or any group on the p2p transports).

    ``partial_fn(q, cache, (lo, hi)) -> (O, LSE)`` and ``merge_fn(O[N], LSE[N], dtype)``
    replace the CUDA steps (then the generic list all-gather is used); tests run the
    collective logic on CPU ranks (gloo) that way."""

    def __init__(self, group: Optional[dist.ProcessGroup] = None,
                 partial_fn: Optional[Callable] = None, merge_fn: Optional[Callable] = None,
                 transport: Optional[str] = None, timeout_ms: float = 2000.0, check_every: int = 0):
        self.group = group
        # check_every > 0: read the exchange status word every that many calls (a host
        # synchronisation); 0 leaves it to check() and close()
        self.check_every = int(check_every)
        self._calls = 0
        self.partial_fn = partial_fn
        self.merge_fn = merge_fn
        # multi-rank CUDA steps: "p2p" (decode with the fused exchange epilogue),
        # "p2p_kernel" (decode, then the exchange kernel) or "nccl" (all-gather)
        self.transport = transport or os.environ.get("FLASHSPEC_EXCHANGE", "p2p")
        if self.transport not in ("p2p", "p2p_kernel", "nccl"):
            raise ValueError("transport must be 'p2p', 'p2p_kernel' or 'nccl'")
        self.timeout_ns = int(timeout_ms * 1e6)
        self._bufs = {}
        self._xch = {}
        self._unfusable = set()

    @property
    def world(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    @property
    def rank(self) -> int:
        return dist.get_rank(self.group) if dist.is_initialized() else 0

    def window(self, n_pages: int) -> Tuple[int, int]:
        return page_window(n_pages, self.rank, self.world)

    def __call__(self, q: torch.Tensor, cache, n_pages: int, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        if self.partial_fn is None and self.merge_fn is None and q.is_cuda:
            return self._cuda_call(q, cache, n_pages, out_dtype)
        pf = self.partial_fn or _cuda_partial
        mf = self.merge_fn or _cuda_merge
        o, lse = pf(q, cache, self.window(n_pages))
        if self.world == 1:
            return mf(o[None], lse[None], out_dtype)
        o_all = [torch.empty_like(o) for _ in range(self.world)]
        lse_all = [torch.empty_like(lse) for _ in range(self.world)]
        dist.all_gather(o_all, o.contiguous(), group=self.group)
        dist.all_gather(lse_all, lse.contiguous(), group=self.group)
        return mf(torch.stack(o_all), torch.stack(lse_all), out_dtype)

    def _cuda_call(self, q, cache, n_pages, out_dtype):
        import ctypes as C

        from . import _lib
        from .attention import paged_quant_attention_cuda
        from .quant import stream_of

        b, hq, d = q.shape
        rows = b * hq
        slot = (rows * d + rows + 63) // 64 * 64  # floats per rank: O then LSE, 256-byte aligned
        key = (q.device, b, hq, d, self.world)
        bufs = self._bufs.get(key)
        if bufs is None:
            mine = torch.empty((slot,), dtype=torch.float32, device=q.device)
            gather = torch.empty((self.world, slot), dtype=torch.float32, device=q.device) if self.world > 1 else None
            bufs = self._bufs[key] = (mine, gather)
        mine, gather = bufs
        o = mine[: rows * d].view(b, hq, d)
        lse = mine[rows * d: rows * d + rows].view(b, hq)
        if self.world > 1 and self.transport in ("p2p", "p2p_kernel"):
            # "p2p": one kernel per step (decode + exchange epilogue) where the shape
            # allows it; otherwise, and with "p2p_kernel", decode then exchange kernel
            fused = self.transport == "p2p" and (q.device, b, hq, d, n_pages) not in self._unfusable
            out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
            if fused:
                xch = self._exchange(q.device, slot, "fused")
                try:
                    xch.decode(q, cache, self.window(n_pages), out)
                except ValueError as e:
                    if "(status 2)" not in str(e):  # FS_ERR_UNSUPPORTED: shape outside the fused kernel
                        raise
                    self._unfusable.add((q.device, b, hq, d, n_pages))
                    fused = False
            if not fused:
                paged_quant_attention_cuda(q, cache, page_range=self.window(n_pages), partial_out=(o, lse))
                xch = self._exchange(q.device, slot, "kernel")
                xch.merge(o, lse, out)
            self._calls += 1
            if self.check_every > 0 and self._calls % self.check_every == 0:
                xch.check()
            return out
        if self.world == 1 and out_dtype == q.dtype:
            # one rank holds the whole window: the plain decode writes the output itself
            return paged_quant_attention_cuda(q, cache, page_range=self.window(n_pages))
        paged_quant_attention_cuda(q, cache, page_range=self.window(n_pages), partial_out=(o, lse))
        if self.world > 1:  # out of place: the send buffer is not a view of the receive buffer
            dist.all_gather_into_tensor(gather.view(-1), mine, group=self.group)
        else:
            gather = mine.view(1, slot)
        out = torch.empty(q.shape, dtype=out_dtype, device=q.device)
        code = {torch.float16: _lib.FS_F16, torch.float32: _lib.FS_F32}[out_dtype]
        base = gather.data_ptr()
        _lib.check(_lib.load().fs_merge_partials(base, base + 4 * rows * d, self.world, rows, d, slot, out.data_ptr(),
                                                 code, stream_of(q.device)), "fs_merge_partials")
        return out

    def _exchange(self, device, slot: int, mode: str) -> "PeerExchange":
        """The group's exchange buffers for one slot size and mode (created collectively
        on first use: every rank reaches it in the same call)."""
        key = (device, slot, mode)
        xch = self._xch.get(key)
        if xch is None:
            xch = self._xch[key] = PeerExchange(self.group, device, slot, self.timeout_ns)
        return xch

    def check(self) -> None:
        """Raise RuntimeError if an exchange of this decoder has timed out (see
        ``PeerExchange.check``); synchronises with the device."""
        for x in self._xch.values():
            x.check()

    def close(self, check: bool = True) -> None:
        """Release the peer-exchange buffers (collectively: every rank calls it, after its
        last step has finished on the GPU; further calls set them up again).  With
        ``check`` the status words are read first and a timeout is raised after the
        buffers are released."""
        failure = None
        if self._xch:
            torch.cuda.synchronize()
            if check:
                try:
                    self.check()
                except RuntimeError as e:
                    failure = e
            multi = dist.is_initialized() and self.world > 1
            if multi:
                dist.barrier(group=self.group)  # every rank's last exchange has finished
            for x in self._xch.values():
                x.close_peers()
            if multi:
                dist.barrier(group=self.group)  # every rank has unmapped its peers' buffers
            for x in self._xch.values():
                x.destroy()
            self._xch.clear()
        if failure is not None:
            raise failure

    def capture(self, q: torch.Tensor, cache, n_pages: int, out_dtype: torch.dtype = torch.float16,
                steps: int = 1):
        """Record ``steps`` consecutive decode steps as one CUDA graph over the given
        tensors; returns ``(replay, out)`` where ``replay()`` re-runs them on the current
        contents of q / cache and refreshes ``out`` (the last step's output).  Several
        steps per graph spare the device the start of a graph launch between steps.
        Multi-rank steps are captured only with the peer-memory exchange (the NCCL step
        runs eagerly); every rank must then replay its graphs the same number of steps."""
        if steps < 1:
            raise ValueError("steps must be >= 1")
        if self.world > 1 and self.transport == "nccl":
            raise ValueError("capture() of a multi-rank step needs a p2p transport; NCCL steps run eagerly")
        side = torch.cuda.Stream(device=q.device)
        side.wait_stream(torch.cuda.current_stream(q.device))
        with torch.cuda.stream(side):
            for _ in range(3):  # workspaces, kernel attributes, NCCL communicator set-up
                self(q, cache, n_pages, out_dtype)
        torch.cuda.current_stream(q.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(steps):
                out = self(q, cache, n_pages, out_dtype)
        return graph.replay, out
