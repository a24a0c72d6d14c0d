"""Pin the CPU oracle against vectors recorded from the reference itself.

Quantizer, dequantizer, paged layouts and allocator state must match
bit-for-bit; attention outputs (fp16) within 1e-3 abs (fp32 summation order)."""

from __future__ import annotations

import numpy as np
import pytest

import flashspec_oracle as O
from conftest import load_golden


def _same_quant(a: O.OQuant, b: O.OQuant):
    assert a.values.dtype == np.int8 and a.zero_point.dtype == np.int16 and a.scale.dtype == np.float32
    np.testing.assert_array_equal(a.values, b.values)
    np.testing.assert_array_equal(a.scale.view(np.uint32), b.scale.view(np.uint32))
    np.testing.assert_array_equal(a.zero_point, b.zero_point)
    assert tuple(a.original_shape) == tuple(b.original_shape)


@pytest.mark.parametrize("name,bs", [("quant_fp32_b8", 8), ("quant_fp16_b16", 16), ("quant_edge_b16", 16)])
def test_quantize_bit_exact(name, bs):
    g = load_golden(name)
    got = O.quantize_int8_per_block(g["x"], bs)
    _same_quant(got, g.quant("q"))
    deq = O.dequantize_int8_per_block(g.quant("q"))
    np.testing.assert_array_equal(deq.view(np.uint32), g["deq"].view(np.uint32))


def test_reference_attention_fp32():
    g = load_golden("reference_attention_fp32")
    got = O.reference_attention(g["q"], g["k"], g["v"], g["lengths"])
    np.testing.assert_allclose(got, g["out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ["fused_s129", "fused_s1500", "fused_nolen_s200"])
def test_fused_attention(name):
    g = load_golden(name)
    lengths = g.get("lengths")
    got = O.fused_dequant_attention(g["q"], g.quant("kq"), g.quant("vq"), lengths)
    np.testing.assert_allclose(got.astype(np.float32), g["out"].astype(np.float32), atol=1e-3, rtol=0)
    assert O.estimate_quantized_bytes(g.quant("kq")) * 2 == int(g["quant_kv_bytes"])
    # and the quantized inputs are the oracle's own quantization of the fp16 data
    assert g.quant("kq").values.shape[-2] == 16


@pytest.mark.parametrize("layout", ["contiguous", "shuffled", "interleaved"])
def test_paged_layouts_and_attention(layout):
    g = load_golden(f"paged_{layout}")
    perm = None
    if layout == "shuffled":
        table = g["block_table"].reshape(-1)
        perm = np.empty_like(table)
        perm[table] = np.arange(table.size)
    cache = O.paged_from_dense(g["k"], g["v"], 16, lengths=g["lengths"], pattern=layout, perm=perm)
    _same_quant(cache.k_quant, g.quant("kq"))
    _same_quant(cache.v_quant, g.quant("vq"))
    np.testing.assert_array_equal(cache.block_table, g["block_table"])
    out = O.paged_quant_attention(g["q"], cache)
    np.testing.assert_allclose(out.astype(np.float32), g["out"].astype(np.float32), atol=1e-3, rtol=0)
    out2 = O.paged_quant_attention_gathered(g["q"], cache)
    np.testing.assert_array_equal(out, out2)
    assert cache.estimated_bytes() == int(g["quant_kv_bytes"])


def test_paged_gqa():
    g = load_golden("paged_gqa4")
    cache = O.OPagedCache(g.quant("kq"), g.quant("vq"), g["block_table"], g["lengths"], 16, int(g["max_seq_len"]))
    out = O.paged_quant_attention(g["q"], cache)
    np.testing.assert_allclose(out.astype(np.float32), g["out"].astype(np.float32), atol=1e-3, rtol=0)


def test_functional_cache_append_bit_exact():
    g = load_golden("cache_append")
    c0 = O.OPagedCache(g.quant("kq0"), g.quant("vq0"), g["table0"], g["lengths0"], 16, 7)
    c1 = O.paged_cache_append(c0, g["k_new"], g["v_new"])
    _same_quant(c1.k_quant, g.quant("kq1"))
    _same_quant(c1.v_quant, g.quant("vq1"))
    np.testing.assert_array_equal(c1.block_table, g["table1"])
    np.testing.assert_array_equal(c1.lengths, g["lengths1"])
    assert c1.max_seq_len == int(g["max_seq_len1"])


def replay_allocator(g, alloc):
    """Replay the recorded op log of ``allocator_lifecycle`` on ``alloc`` (oracle or
    device allocator); token tensors come from the fixture."""
    step = 0
    for op, rid, rids, n in zip(g["ops"], g["op_rid"], g["op_rids"], g["op_n"]):
        if op == 0:
            alloc.add_request(int(rid), g[f"tok.add{rid}_k"], g[f"tok.add{rid}_v"])
        elif op == 1:
            ids = [int(r) for r in rids if r >= 0]
            alloc.append_batch(ids, g[f"tok.app{step}_k"], g[f"tok.app{step}_v"])
            step += 1
        else:
            alloc.release_request(int(rid))


def test_allocator_lifecycle_bit_exact():
    g = load_golden("allocator_lifecycle")
    a = O.OAllocator(int(g["capacity"]), int(g["heads"]), int(g["head_dim"]), int(g["block_size"]))
    replay_allocator(g, a)
    _same_quant(a.k_quant, g.quant("kq"))
    _same_quant(a.v_quant, g.quant("vq"))
    assert a.free_blocks == [int(x) for x in g["free_blocks"]]
    cache = a.to_cache([30, 40, 50])
    np.testing.assert_array_equal(cache.block_table, g["table"])
    np.testing.assert_array_equal(cache.lengths, g["lengths"])
    st = a.stats()
    for k, v in zip(g["stats_keys"], g["stats_vals"]):
        assert st[str(k)] == pytest.approx(float(v), abs=0, rel=1e-12)
    out = O.paged_quant_attention(g["q"], cache)
    np.testing.assert_allclose(out.astype(np.float32), g["out"].astype(np.float32), atol=1e-3, rtol=0)


def test_merge_partials_equals_full_attention():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 3, 64)).astype(np.float32)
    k = rng.standard_normal((2, 3, 300, 64)).astype(np.float32)
    v = rng.standard_normal((2, 3, 300, 64)).astype(np.float32)
    lengths = np.array([300, 130])
    full = O.reference_attention(q, k, v, lengths)
    parts = [O.partial_attention(q, k, v, lo, lo + 80, lengths) for lo in range(0, 320, 80)]
    o = np.stack([p[0] for p in parts])
    lse = np.stack([p[1] for p in parts])
    np.testing.assert_allclose(O.merge_partials(o, lse), full, atol=2e-6, rtol=1e-5)
    empty = O.merge_partials(np.zeros((2, 1, 4), np.float32), np.full((2, 1), -np.inf, np.float32))
    assert np.all(empty == 0)


def test_algorithmic_bytes_matches_baseline_cfg1():
    assert O.algorithmic_bytes_paged(16, 32, 32, 128, [4096] * 16) == 538_738_816


def test_tree_verify_oracle_equals_path_gather():
    """The dense-mask statement of tree verify agrees with gathering each node's root path
    explicitly (two independent restatements), including a chain, a fork and a node that
    hangs off the prefix."""
    rng = np.random.default_rng(5)
    b, n, hq, hkv, d = 2, 6, 4, 2, 16
    q = rng.standard_normal((b, n, hq, d)).astype(np.float32)
    k = rng.standard_normal((b, hkv, 40, d)).astype(np.float32)
    v = rng.standard_normal((b, hkv, 40, d)).astype(np.float32)
    cache = O.paged_from_dense(k, v, 8, lengths=np.array([40, 13]))
    tk = rng.standard_normal((b, n, hkv, d)).astype(np.float32)
    tv = rng.standard_normal((b, n, hkv, d)).astype(np.float32)
    parents = np.array([[-1, 0, 1, 1, 0, -1], [-1, 0, 1, 2, 3, 4]])
    got = O.tree_verify_attention(q, cache, tk, tv, parents)
    kd, vd = O.paged_to_dense(cache)
    for bi in range(b):
        L = int(cache.lengths[bi])
        for i in range(n):
            path, j = [], i
            while j >= 0:
                path.append(j)
                j = int(parents[bi, j])
            for h in range(hq):
                kh = h // (hq // hkv)
                keys = np.concatenate([kd[bi, kh, :L], tk[bi, path, kh]], 0)
                vals = np.concatenate([vd[bi, kh, :L], tv[bi, path, kh]], 0)
                sc = keys @ q[bi, i, h] / np.sqrt(d)
                w = np.exp(sc - sc.max())
                np.testing.assert_allclose(got[bi, i, h], (w / w.sum()) @ vals, rtol=1e-5, atol=1e-6)
