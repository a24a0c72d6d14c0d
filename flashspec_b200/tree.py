"""Tree-attention verify for speculative decoding (the reference's planned "Kernel 3",
doc/TODO.MD:186-237): every node of a draft tree attends to the request's committed
prefix in the paged INT8 cache and to the draft tokens on its own root path.

The prefix half reuses the paged decode kernels: a request's tree nodes are folded into
the query-head axis (up to 8 query rows per kv head and pass), so one read of each prefix
page serves several nodes, and the kernels return normalised partials (O, LSE).  The path
half and the merge run in ``fs_tree_attend``.
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Optional

import torch

from . import _lib
from .attention import paged_quant_attention_cuda
from .quant import stream_of

MAX_ROWS_PER_KV_HEAD = 8  # query rows the decode kernels take per kv head and pass


def validate_tree(parents: torch.Tensor, nodes: int) -> None:
    """parents [B, nodes] integer: parents[b, i] in [-1, i) (nodes in topological order,
    -1 = child of the committed prefix).  Cycles, self loops, forward references and
    orphans (an index outside the tree) raise ValueError."""
    if parents.ndim != 2 or parents.shape[1] != nodes:
        raise ValueError("parents must have shape [batch, nodes]")
    if parents.dtype not in (torch.int32, torch.int64):
        raise ValueError("parents must be an integer tensor")
    idx = torch.arange(nodes, device=parents.device).unsqueeze(0)
    if bool((parents < -1).any()) or bool((parents >= idx).any()):
        raise ValueError("every parent must be -1 or an earlier node (no cycles, no orphans)")


def tree_verify_attention_cuda(q: torch.Tensor, cache, tree_k: torch.Tensor, tree_v: torch.Tensor,
                               parents: torch.Tensor, return_stats: bool = False):
    """q [B, N, Hq, D] fp16/bf16 (one query token per draft node); ``cache`` the committed
    prefix (a PagedKVCache, lengths = committed tokens); tree_k / tree_v [B, N, Hkv, D]
    the draft tokens' K and V (q's dtype); parents [B, N].  Returns out [B, N, Hq, D]:
    node i's attention over the prefix plus its ancestors and itself."""
    if q.ndim != 4:
        raise ValueError("q must have shape [batch, nodes, q_heads, head_dim]")
    b, n, hq, d = q.shape
    if q.device.type != "cuda":
        raise RuntimeError("tree verify needs CUDA tensors")
    hkv = int(cache.k_quant.original_shape[1])
    if hq % hkv:
        raise ValueError("q heads must be a multiple of the kv heads")
    g = hq // hkv
    for t, name in ((tree_k, "tree_k"), (tree_v, "tree_v")):
        if tuple(t.shape) != (b, n, hkv, d):
            raise ValueError(f"{name} must have shape [batch, nodes, kv_heads, head_dim]")
        if t.dtype != q.dtype or t.device != q.device:
            raise ValueError(f"{name} must match q's dtype and device")
    validate_tree(parents, n)
    if cache.block_table.shape[0] != b:
        raise ValueError("the cache batch must match q")

    # ---- prefix: nodes folded into the query-head axis, in chunks the kernels take
    prefix_o = torch.empty((b, n, hq, d), dtype=torch.float32, device=q.device)
    prefix_lse = torch.empty((b, n, hq), dtype=torch.float32, device=q.device)
    per_pass = max(1, MAX_ROWS_PER_KV_HEAD // g)
    if g > MAX_ROWS_PER_KV_HEAD:
        raise ValueError("more than 8 query heads per kv head")
    passes = 0
    for n0 in range(0, n, per_pass):
        n1 = min(n, n0 + per_pass)
        nc = n1 - n0
        qc = (q[:, n0:n1].reshape(b, nc, hkv, g, d).permute(0, 2, 1, 3, 4).reshape(b, hkv * nc * g, d)
              .contiguous())
        o = torch.empty((b, hkv * nc * g, d), dtype=torch.float32, device=q.device)
        lse = torch.empty((b, hkv * nc * g), dtype=torch.float32, device=q.device)
        paged_quant_attention_cuda(qc, cache, partial_out=(o, lse))
        prefix_o[:, n0:n1] = o.view(b, hkv, nc, g, d).permute(0, 2, 1, 3, 4).reshape(b, nc, hq, d)
        prefix_lse[:, n0:n1] = lse.view(b, hkv, nc, g).permute(0, 2, 1, 3).reshape(b, nc, hq)
        passes += 1

    # ---- the draft paths and the merge
    out = torch.empty_like(q)
    qc, kc, vc = q.contiguous(), tree_k.contiguous(), tree_v.contiguous()
    par = parents.to(torch.int32).contiguous()
    a = _lib.FsTreeArgs()
    a.q, a.tree_k, a.tree_v, a.parents = qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), par.data_ptr()
    a.prefix_o, a.prefix_lse, a.out = prefix_o.data_ptr(), prefix_lse.data_ptr(), out.data_ptr()
    a.batch, a.nodes, a.q_heads, a.kv_heads, a.head_dim = b, n, hq, hkv, d
    a.q_dtype = _lib.FS_BF16 if q.dtype == torch.bfloat16 else _lib.FS_F16
    a.sm_scale = 1.0 / math.sqrt(float(d))
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().fs_tree_attend(C.byref(a), stream_of(q.device)), "fs_tree_attend")
    if not return_stats:
        return out
    depth = torch.zeros((b, n), dtype=torch.int64)
    pc = parents.to(torch.int64).cpu()
    for i in range(n):
        depth[:, i] = torch.where(pc[:, i] >= 0, depth.gather(1, pc[:, i].clamp_min(0).unsqueeze(1))[:, 0] + 1, 1)
    leaves = n - int((pc.unsqueeze(2) == torch.arange(n).view(1, 1, n)).any(1).sum(1).float().mean().item())
    return out, {"nodes": float(n), "max_depth": float(depth.max().item()), "leaf_count": float(leaves),
                 "prefix_passes": float(passes), "materializes_dense_kv": 0.0}
