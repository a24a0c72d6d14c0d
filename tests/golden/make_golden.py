"""Generate the golden fixtures in this folder from the reference FlashSpec package.

Run once in a container where the reference source tree is available:

    python tests/golden/make_golden.py /path/to/FlashSpec/src

It imports the reference (pure Python + torch on CPU), drives its public API on
seeded inputs and records inputs and outputs as .npz files.  Nothing at test or
bench time imports the reference; the fixtures are what travel.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _q(qt):
    return dict(values=qt.values.numpy(), scale=qt.scale.numpy(), zero_point=qt.zero_point.numpy(),
                block_size=np.int64(qt.block_size), original_shape=np.array(qt.original_shape, np.int64))


def _save(name, **arrays):
    flat = {}
    for k, v in arrays.items():
        if isinstance(v, dict):
            for kk, vv in v.items():
                flat[f"{k}.{kk}"] = vv
        elif isinstance(v, torch.Tensor):
            flat[k] = v.numpy()
        else:
            flat[k] = np.asarray(v)
    np.savez_compressed(HERE / f"{name}.npz", **flat)
    print(name, sum(a.nbytes for a in flat.values()), "bytes raw")


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    import flashspec as fs  # noqa: the reference package

    g = torch.Generator().manual_seed(20260101)
    rn = lambda *s, dt=torch.float32: torch.randn(*s, generator=g).to(dt)

    # -- quantizer ----------------------------------------------------------
    x = rn(2, 3, 19, 16)
    _save("quant_fp32_b8", x=x, q=_q(fs.quantize_int8_per_block(x, block_size=8)),
          deq=fs.dequantize_int8_per_block(fs.quantize_int8_per_block(x, block_size=8)))
    x = rn(2, 4, 37, 128, dt=torch.float16)
    qt = fs.quantize_int8_per_block(x, block_size=16)
    _save("quant_fp16_b16", x=x, q=_q(qt), deq=fs.dequantize_int8_per_block(qt))
    x = torch.zeros(1, 2, 48, 128)
    x[0, 0, :16] = 0.5  # constant block -> scale floor
    x[0, 1, 16:32] = -3.25
    x[0, 1, 32:48] = rn(16, 128) * 1.0e-9  # tiny range -> floor
    x[0, 0, 32:48] = rn(16, 128) * 1000.0  # wide range
    qt = fs.quantize_int8_per_block(x, block_size=16)
    _save("quant_edge_b16", x=x, q=_q(qt), deq=fs.dequantize_int8_per_block(qt))

    # -- dense reference attention -------------------------------------------
    q, k, v = rn(2, 3, 16), rn(2, 3, 25, 16), rn(2, 3, 25, 16)
    lengths = torch.tensor([25, 9])
    _save("reference_attention_fp32", q=q, k=k, v=v, lengths=lengths,
          out=fs.reference_attention(q, k, v, lengths=lengths))

    # -- fused (contiguous) backend -------------------------------------------
    for name, (b, h, s, lens) in {
        "fused_s129": (2, 4, 129, [129, 113]),
        "fused_s1500": (2, 2, 1500, [1500, 977]),
        "fused_nolen_s200": (3, 2, 200, None),
    }.items():
        q = rn(b, h, 128, dt=torch.float16)
        k = rn(b, h, s, 128, dt=torch.float16)
        v = rn(b, h, s, 128, dt=torch.float16)
        kq, vq = fs.quantize_int8_per_block(k, 16), fs.quantize_int8_per_block(v, 16)
        lt = None if lens is None else torch.tensor(lens, dtype=torch.int64)
        out, stats = fs.fused_dequant_attention(q, kq, vq, lengths=lt, return_stats=True)
        extra = {} if lt is None else {"lengths": lt}
        _save(name, q=q, kq=_q(kq), vq=_q(vq), out=out, quant_kv_bytes=stats["quant_kv_bytes"],
              dense_kv_bytes=stats["dense_kv_bytes"], **extra)

    # -- paged backend: layouts ----------------------------------------------
    for layout in ("contiguous", "shuffled", "interleaved"):
        q = rn(3, 4, 128, dt=torch.float16)
        k = rn(3, 4, 45, 128, dt=torch.float16)
        v = rn(3, 4, 45, 128, dt=torch.float16)
        lens = torch.tensor([45, 30, 7], dtype=torch.int64)
        cache = fs.PagedKVCache.from_dense(k, v, block_size=16, lengths=lens,
                                           block_table_pattern=layout, layout_seed=13)
        out, stats = fs.paged_quant_attention(q, cache, return_stats=True)
        _save(f"paged_{layout}", q=q, k=k, v=v, kq=_q(cache.k_quant), vq=_q(cache.v_quant),
              block_table=cache.block_table, lengths=cache.lengths, max_seq_len=cache.max_seq_len,
              out=out, quant_kv_bytes=stats["quant_kv_bytes"], physical_blocks=stats["physical_blocks"])

    # -- GQA via G reference calls (q heads g::G read kv head j) ---------------
    G = 4
    q = rn(2, 2 * G, 128, dt=torch.float16)
    k = rn(2, 2, 100, 128, dt=torch.float16)
    v = rn(2, 2, 100, 128, dt=torch.float16)
    cache = fs.PagedKVCache.from_dense(k, v, block_size=16, lengths=torch.tensor([100, 61]),
                                       block_table_pattern="shuffled", layout_seed=5)
    out = torch.empty_like(q)
    for gi in range(G):
        out[:, gi::G] = fs.paged_quant_attention(q[:, gi::G].contiguous(), cache)
    _save("paged_gqa4", q=q, kq=_q(cache.k_quant), vq=_q(cache.v_quant), block_table=cache.block_table,
          lengths=cache.lengths, max_seq_len=cache.max_seq_len, out=out)

    # -- functional PagedKVCache.append ----------------------------------------
    k, v = rn(2, 2, 7, 128), rn(2, 2, 7, 128)
    kn, vn = rn(2, 2, 11, 128), rn(2, 2, 11, 128)
    c0 = fs.PagedKVCache.from_dense(k, v, block_size=16, block_table_pattern="shuffled", layout_seed=3)
    c1 = c0.append(kn, vn)
    _save("cache_append", k=k, v=v, k_new=kn, v_new=vn, kq0=_q(c0.k_quant), vq0=_q(c0.v_quant),
          table0=c0.block_table, lengths0=c0.lengths, kq1=_q(c1.k_quant), vq1=_q(c1.v_quant),
          table1=c1.block_table, lengths1=c1.lengths, max_seq_len1=c1.max_seq_len)

    # -- allocator lifecycle (stale page reuse, page-boundary appends) ----------
    H, D, BS, CAP = 2, 128, 16, 24
    alloc = fs.PagedKVAllocator(capacity_blocks=CAP, heads=H, head_dim=D, block_size=BS)
    log = []  # (op, rid list, token arrays)
    tok = {}

    def add(rid, n):
        kk, vv = rn(1, H, n, D, dt=torch.float16), rn(1, H, n, D, dt=torch.float16)
        tok[f"add{rid}_k"], tok[f"add{rid}_v"] = kk, vv
        alloc.add_request(rid, kk, vv)
        log.append(("add", rid, n))

    def app(rids, n, step):
        kk = rn(len(rids), H, n, D, dt=torch.float16)
        vv = rn(len(rids), H, n, D, dt=torch.float16)
        tok[f"app{step}_k"], tok[f"app{step}_v"] = kk, vv
        alloc.append_batch(rids, kk, vv)
        log.append(("app", rids, n))

    add(10, 37)
    add(20, 16)
    add(40, 40)
    app([10], 4, 0)
    step = 1
    for _ in range(20):
        app([10, 20, 40], 1, step)
        step += 1
    alloc.release_request(20)
    log.append(("rel", 20, 0))
    add(30, 5)  # reuses the lowest freed pages (stale contents)
    for _ in range(18):
        app([30, 10], 1, step)
        step += 1
    app([40], 19, step)  # multi-token append across page boundaries
    step += 1
    alloc.release_request(10)
    log.append(("rel", 10, 0))
    add(50, 33)
    for _ in range(6):
        app([50, 30, 40], 1, step)
        step += 1
    ids = [30, 40, 50]
    cache = alloc.to_cache(ids)
    q = rn(len(ids), H, D, dt=torch.float16)
    out = fs.paged_quant_attention(q, cache)
    ops = np.array([(0 if o == "add" else 1 if o == "app" else 2) for o, _, _ in log], np.int64)
    op_ids = [r if isinstance(r, int) else -1 for _, r, _ in log]
    op_n = [n for _, _, n in log]
    op_rids = np.full((len(log), 3), -1, np.int64)
    for i, (_, r, _) in enumerate(log):
        rr = [r] if isinstance(r, int) else r
        op_rids[i, : len(rr)] = rr
    stats = alloc.stats()
    _save("allocator_lifecycle", capacity=CAP, heads=H, head_dim=D, block_size=BS, ops=ops,
          op_rid=np.array(op_ids), op_rids=op_rids, op_n=np.array(op_n),
          kq=_q(alloc.k_quant), vq=_q(alloc.v_quant), free_blocks=np.array(alloc._free_blocks, np.int64),
          table=cache.block_table, lengths=cache.lengths, q=q, out=out,
          stats_keys=np.array(sorted(stats)), stats_vals=np.array([stats[k] for k in sorted(stats)]),
          **{f"tok.{k}": v for k, v in tok.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference/src")
