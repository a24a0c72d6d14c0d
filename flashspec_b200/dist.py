"""Multi-GPU decode: one process per GPU, torch.distributed for the plumbing.

Two strategies (the reference has no multi-GPU path; SURVEY of the hot path):

* request x kv-head sharding (configs 0, 1, 2, 4): every rank owns whole requests
  and runs the single-GPU kernel on them.  No communication; see ``request_shard``.
* sequence sharding of long requests (config 3): rank r owns the contiguous logical
  pages ``page_window(n_pages, r, N)`` of every request and only those pages are
  resident on it.  Each rank computes a normalised partial (O fp32, LSE fp32) over
  its window with the page-window mode of the decode kernel, the partials are
  all-gathered (NCCL over NVLink; 2*B*Hq*(D+1)*4 bytes per rank) and merged with the
  log-sum-exp rule of ``fs_merge_partials`` -- the same math as the split-K combine
  (src/flashspec/triton_fused.py:446-503) applied across GPUs.
"""

from __future__ import annotations

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


class SequenceShardedDecoder:
    """Decode one batch whose KV pages are split across the ranks of ``group``.

    ``partial_fn(q, cache, (lo, hi)) -> (O, LSE)`` and ``merge_fn(O[N], LSE[N], dtype)``
    default to the CUDA kernels; they are parameters so the collective logic can run
    on CPU ranks (gloo) in tests."""

    def __init__(self, group: Optional[dist.ProcessGroup] = None,
                 partial_fn: Callable = _cuda_partial, merge_fn: Callable = _cuda_merge):
        self.group = group
        self.partial_fn = partial_fn
        self.merge_fn = merge_fn

    @property
    def world(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    @property
    def rank(self) -> int:
        return dist.get_rank(self.group) if dist.is_initialized() else 0

    def window(self, n_pages: int) -> Tuple[int, int]:
        return page_window(n_pages, self.rank, self.world)

    def __call__(self, q: torch.Tensor, cache, n_pages: int, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        o, lse = self.partial_fn(q, cache, self.window(n_pages))
        if self.world == 1:
            return self.merge_fn(o[None], lse[None], out_dtype)
        o_all = [torch.empty_like(o) for _ in range(self.world)]
        lse_all = [torch.empty_like(lse) for _ in range(self.world)]
        dist.all_gather(o_all, o.contiguous(), group=self.group)
        dist.all_gather(lse_all, lse.contiguous(), group=self.group)
        return self.merge_fn(torch.stack(o_all), torch.stack(lse_all), out_dtype)
