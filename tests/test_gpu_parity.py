"""GPU parity of the CUDA path against the golden vectors (recorded from the
reference) and the CPU oracle.

Tolerances: attention outputs (fp16) within max-abs 2e-3 and rel 1e-2 of the
reference, i.e. |got - ref| <= 2e-3 + 1e-2 * |ref| elementwise; quantized bytes,
scales, zero points, block tables and allocator state bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import flashspec_oracle as O
from conftest import load_golden

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def fs():
    import flashspec_b200

    return flashspec_b200


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    torch.manual_seed(0)


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def qt_dev(g, prefix):
    f = fs()
    return f.QuantizedTensor(dev(g[f"{prefix}.values"]), dev(g[f"{prefix}.scale"]), dev(g[f"{prefix}.zero_point"]),
                             int(g[f"{prefix}.block_size"]), tuple(int(x) for x in g[f"{prefix}.original_shape"]))


def close(got: torch.Tensor, ref, atol=ATOL, rtol=RTOL):
    ref_t = torch.as_tensor(np.asarray(ref, dtype=np.float32))
    got_f = got.detach().float().cpu()
    err = (got_f - ref_t).abs()
    bound = atol + rtol * ref_t.abs()
    assert torch.all(err <= bound), f"max abs err {err.max().item():.3e}"
    return err.max().item()


def same_quant(qt, oq):
    np.testing.assert_array_equal(qt.values.cpu().numpy(), oq.values)
    np.testing.assert_array_equal(qt.scale.cpu().numpy().view(np.uint32), oq.scale.view(np.uint32))
    np.testing.assert_array_equal(qt.zero_point.cpu().numpy(), oq.zero_point)


# ---------------------------------------------------------------------------------
# quantizer
# ---------------------------------------------------------------------------------


@pytest.mark.parametrize("name,bs", [("quant_fp32_b8", 8), ("quant_fp16_b16", 16), ("quant_edge_b16", 16)])
def test_quantize_matches_reference_bit_exact(name, bs):
    g = load_golden(name)
    q = fs().quantize_int8_per_block(dev(g["x"]), bs)
    same_quant(q, g.quant("q"))
    assert tuple(q.original_shape) == tuple(int(x) for x in g["q.original_shape"])


def test_quantize_random_bf16_and_odd_shapes_vs_oracle():
    rng = np.random.default_rng(1)
    for shape, bs in [((3, 5, 33, 128), 16), ((2, 7, 64), 16), ((4, 1, 17, 96), 4)]:
        x = (rng.standard_normal(shape) * rng.uniform(0.01, 50)).astype(np.float32)
        xt = dev(x).to(torch.bfloat16)
        q = fs().quantize_int8_per_block(xt, bs)
        same_quant(q, O.quantize_int8_per_block(xt.float().cpu().numpy(), bs))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape,bs", [((4, 8, 1000, 128), 16), ((2, 4, 300, 64), 8), ((2, 3, 640, 256), 32),
                                      ((3, 2, 100, 32), 16)])
def test_quantize_vector_kernel_bit_identical_to_division(monkeypatch, dtype, shape, bs):
    """The 16-byte-per-thread quantizer (reciprocal product, division only near a rounding
    boundary) against the per-element division kernel (FLASHSPEC_PAGE_UPDATE_SCALAR), on
    ~4M values of scales 1e-3 .. 1e3 with offsets, ragged tails and a misaligned source."""
    rng = np.random.default_rng(hash((shape, bs)) % 2**32)
    n = int(np.prod(shape))
    x = rng.standard_normal(n).astype(np.float32) * np.repeat(10.0 ** rng.uniform(-3, 3, n // shape[-1]), shape[-1])
    x += np.repeat(rng.standard_normal(n // shape[-1]) * 5, shape[-1])
    flat = torch.empty(n + 3, dtype=dtype, device="cuda")
    flat[3:] = dev(x).to(dtype)
    xt = flat[3:].view(shape)  # 3 elements off the allocation: misaligned rows take scalar loads
    outs = []
    for scalar in (False, True):
        if scalar:
            monkeypatch.setenv("FLASHSPEC_PAGE_UPDATE_SCALAR", "1")
        q = fs().quantize_int8_per_block(xt, bs)
        q2 = fs().quantize_int8_per_block(xt.contiguous().clone(), bs)
        torch.cuda.synchronize()
        outs.append((q, q2))
    (a, a2), (b, b2) = outs
    for x1, x2 in ((a, b), (a2, b2), (a, a2)):
        assert torch.equal(x1.values, x2.values)
        assert torch.equal(x1.scale, x2.scale)
        assert torch.equal(x1.zero_point, x2.zero_point)
    small = xt[:1, :1].float().cpu().numpy()
    same_quant(fs().quantize_int8_per_block(xt[:1, :1].contiguous(), bs), O.quantize_int8_per_block(small, bs))


# ---------------------------------------------------------------------------------
# contiguous backend
# ---------------------------------------------------------------------------------


@pytest.mark.parametrize("name", ["fused_s129", "fused_s1500", "fused_nolen_s200"])
def test_fused_matches_reference_golden(name):
    g = load_golden(name)
    lengths = dev(g["lengths"]) if "lengths" in g else None
    out, stats = fs().fused_dequant_attention_cuda(dev(g["q"]), qt_dev(g, "kq"), qt_dev(g, "vq"), lengths,
                                                   return_stats=True)
    assert out.dtype == torch.float16 and tuple(out.shape) == g["q"].shape
    close(out, g["out"])
    assert stats["materializes_dense_kv"] == 0.0
    assert stats["quant_kv_bytes"] == float(g["quant_kv_bytes"])


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 64])
def test_fused_split_k_invariance(splits):
    g = load_golden("fused_s1500")
    out = fs().fused_dequant_attention_cuda(dev(g["q"]), qt_dev(g, "kq"), qt_dev(g, "vq"), dev(g["lengths"]),
                                            num_splits=splits)
    close(out, g["out"])


# ---------------------------------------------------------------------------------
# paged backend
# ---------------------------------------------------------------------------------


def paged_from_golden(g, key_table="block_table"):
    return fs().PagedKVCache(qt_dev(g, "kq"), qt_dev(g, "vq"), dev(g[key_table]), dev(g["lengths"]), 16,
                             int(g["max_seq_len"]))


@pytest.mark.parametrize("layout", ["contiguous", "shuffled", "interleaved"])
def test_paged_matches_reference_golden(layout):
    g = load_golden(f"paged_{layout}")
    out, stats = fs().paged_quant_attention_cuda(dev(g["q"]), paged_from_golden(g), return_stats=True)
    close(out, g["out"])
    assert stats["physical_blocks"] == float(g["physical_blocks"])
    assert stats["quant_kv_bytes"] == float(g["quant_kv_bytes"])
    assert stats["materializes_dense_kv"] == 0.0


def test_paged_gqa_matches_reference_golden():
    g = load_golden("paged_gqa4")
    out = fs().paged_quant_attention_cuda(dev(g["q"]), paged_from_golden(g))
    close(out, g["out"])


def test_paged_from_dense_on_gpu_matches_reference_layout():
    g = load_golden("paged_shuffled")
    table = g["block_table"].reshape(-1)
    perm = np.empty_like(table)
    perm[table] = np.arange(table.size)
    cache = fs().PagedKVCache.from_dense(dev(g["k"]), dev(g["v"]), 16, lengths=dev(g["lengths"]),
                                         block_table_pattern="shuffled", perm=dev(perm))
    same_quant(cache.k_quant, g.quant("kq"))
    same_quant(cache.v_quant, g.quant("vq"))
    np.testing.assert_array_equal(cache.block_table.cpu().numpy(), g["block_table"])


def test_paged_accepts_foreign_cache_objects_built_by_the_reference():
    """The golden pools were built by the reference's own PagedKVCache.from_dense
    (src/flashspec/paged.py:303-419).  Wrapped in stand-in classes that carry only the
    reference dataclasses' fields (QuantizedTensor quant.py:9-43, PagedKVCache
    paged.py:258-300; the reference cannot be imported on a GPU box), the backend must
    read them by duck typing and give the reference's output."""
    from dataclasses import dataclass
    from typing import Tuple

    @dataclass(frozen=True)
    class ForeignQuant:
        values: torch.Tensor
        scale: torch.Tensor
        zero_point: torch.Tensor
        block_size: int
        original_shape: Tuple[int, ...]

    @dataclass(frozen=True)
    class ForeignPagedCache:
        k_quant: ForeignQuant
        v_quant: ForeignQuant
        block_table: torch.Tensor
        lengths: torch.Tensor
        block_size: int
        max_seq_len: int

        @property
        def num_heads(self) -> int:
            return int(self.k_quant.original_shape[1])

        def estimated_bytes(self) -> int:
            qb = lambda t: t.values.numel() + 4 * t.scale.numel() + 2 * t.zero_point.numel()
            return qb(self.k_quant) + qb(self.v_quant) + 8 * self.block_table.numel() + 8 * self.lengths.numel()

    for name in ("paged_shuffled", "paged_gqa4"):
        g = load_golden(name)

        def fq(prefix):
            return ForeignQuant(dev(g[f"{prefix}.values"]), dev(g[f"{prefix}.scale"]), dev(g[f"{prefix}.zero_point"]),
                                int(g[f"{prefix}.block_size"]), tuple(int(x) for x in g[f"{prefix}.original_shape"]))

        cache = ForeignPagedCache(fq("kq"), fq("vq"), dev(g["block_table"]), dev(g["lengths"]), 16,
                                  int(g["max_seq_len"]))
        out, stats = fs().paged_quant_attention_cuda(dev(g["q"]), cache, return_stats=True)
        close(out, g["out"])
        if "quant_kv_bytes" in g:
            assert stats["quant_kv_bytes"] == float(g["quant_kv_bytes"])


@pytest.mark.parametrize("layout", ["shuffled", "interleaved"])
def test_to_dense_matches_reference_bit_exact(layout):
    """PagedKVCache.to_dense (fs_dequantize_pages gathering the referenced pages) against
    the reference's to_dense recorded in the golden (paged.py:421-461): bit-identical."""
    g = load_golden(f"paged_{layout}")
    cache = paged_from_golden(g)
    k, v = cache.to_dense()
    ok, ov = O.paged_to_dense(O.OPagedCache(g.quant("kq"), g.quant("vq"), g["block_table"], g["lengths"], 16,
                                            int(g["max_seq_len"])))
    np.testing.assert_array_equal(k.cpu().numpy().view(np.uint32), ok.astype(np.float32).view(np.uint32))
    np.testing.assert_array_equal(v.cpu().numpy().view(np.uint32), ov.astype(np.float32).view(np.uint32))
    # unallocated entries read page 0, as the reference's clamp_min(0) gather does
    t = cache.block_table.clone()
    t[0, -1] = -1
    c2 = fs().PagedKVCache(cache.k_quant, cache.v_quant, t, cache.lengths, 16, cache.max_seq_len)
    k2, _ = c2.to_dense()
    ok2, _ = O.paged_to_dense(O.OPagedCache(g.quant("kq"), g.quant("vq"), t.cpu().numpy(), g["lengths"], 16,
                                            int(g["max_seq_len"])))
    np.testing.assert_array_equal(k2.cpu().numpy(), ok2.astype(np.float32))


def _random_paged(rng, b, hq, hkv, lens, slack=3, layout="shuffled"):
    smax = max(max(lens), 1)
    q = rng.standard_normal((b, hq, 128)).astype(np.float16)
    k = rng.standard_normal((b, hkv, smax, 128)).astype(np.float16)
    v = rng.standard_normal((b, hkv, smax, 128)).astype(np.float16)
    bps = (smax + 15) // 16
    total = b * bps + slack
    perm = rng.permutation(total)[: b * bps] if layout == "shuffled" else np.arange(b * bps)
    oc = O.paged_from_dense(k, v, 16, lengths=np.array(lens), pattern="contiguous")
    # scatter logical pages to physical slots `perm` of a pool with slack pages
    pool_k = O.quantize_int8_per_block(np.zeros((total, hkv, 16, 128), np.float32), 16)
    pool_v = O.quantize_int8_per_block(np.zeros((total, hkv, 16, 128), np.float32), 16)
    for src, dst in enumerate(perm):
        for pool, part in ((pool_k, oc.k_quant), (pool_v, oc.v_quant)):
            pool.values[dst] = part.values[src]
            pool.scale[dst] = part.scale[src]
            pool.zero_point[dst] = part.zero_point[src]
    table = perm.reshape(b, bps).astype(np.int64)
    ocache = O.OPagedCache(pool_k, pool_v, table, np.array(lens, np.int64), 16, smax)
    return q, ocache


def _cache_dev(oc):
    f = fs()
    qk = f.QuantizedTensor(dev(oc.k_quant.values), dev(oc.k_quant.scale), dev(oc.k_quant.zero_point), 16,
                           oc.k_quant.original_shape)
    qv = f.QuantizedTensor(dev(oc.v_quant.values), dev(oc.v_quant.scale), dev(oc.v_quant.zero_point), 16,
                           oc.v_quant.original_shape)
    return f.PagedKVCache(qk, qv, dev(oc.block_table), dev(oc.lengths), 16, oc.max_seq_len)


@pytest.mark.parametrize("hq,hkv", [(4, 4), (8, 4), (8, 2), (16, 2), (8, 1)])
@pytest.mark.parametrize("splits", [0, 1, 5])
def test_paged_random_ragged_gqa_vs_oracle(hq, hkv, splits):
    rng = np.random.default_rng(hq * 100 + hkv * 10 + splits)
    lens = [1, 16, 17, 250, 31, 512, 100]
    q, oc = _random_paged(rng, len(lens), hq, hkv, lens)
    out = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc), num_splits=splits or None)
    close(out, O.paged_quant_attention(q, oc))


def test_paged_zero_length_outputs_zero():
    rng = np.random.default_rng(3)
    q, oc = _random_paged(rng, 3, 4, 4, [40, 0, 7])
    oc.lengths[1] = 0
    out = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc), num_splits=4)
    assert torch.all(out[1] == 0)
    ref = O.paged_quant_attention(q, oc)
    close(out[[0, 2]], ref[[0, 2]])


def test_paged_unallocated_table_entries_are_masked():
    rng = np.random.default_rng(4)
    q, oc = _random_paged(rng, 2, 4, 4, [64, 20])
    # request 1 only needs 2 pages: the rest of its row is -1 in a real allocator
    oc.block_table[1, 2:] = -1
    out = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc))
    close(out, O.paged_quant_attention(q, oc))


def test_paged_bad_page_index_is_reported_not_read():
    rng = np.random.default_rng(5)
    q, oc = _random_paged(rng, 2, 4, 4, [64, 64])
    ok = O.paged_quant_attention(q, oc)
    n_pages = oc.k_quant.values.shape[0]
    oc.block_table[0, 1] = n_pages + 1000  # beyond the pool: the kernel must skip it
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc), device_status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1
    close(out[1], ok[1])


def test_paged_layout_invariance_is_bit_exact():
    """The same logical pages in a different physical order give identical bits."""
    rng = np.random.default_rng(6)
    q, oc_a = _random_paged(rng, 3, 8, 2, [300, 129, 77], layout="contiguous")
    perm = rng.permutation(oc_a.k_quant.values.shape[0])
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size)
    sh = lambda qt: O.OQuant(qt.values[perm], qt.scale[perm], qt.zero_point[perm], 16, qt.original_shape)
    oc_b = O.OPagedCache(sh(oc_a.k_quant), sh(oc_a.v_quant), inv[oc_a.block_table], oc_a.lengths, 16,
                         oc_a.max_seq_len)
    a = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc_a), num_splits=3)
    b = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc_b), num_splits=3)
    assert torch.equal(a, b)
    c = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc_a), num_splits=3)
    assert torch.equal(a, c)  # deterministic rerun


def test_paged_page_windows_and_merge_equal_full():
    rng = np.random.default_rng(7)
    q, oc = _random_paged(rng, 2, 16, 2, [700, 333])
    cache = _cache_dev(oc)
    full = fs().paged_quant_attention_cuda(dev(q), cache)
    bounds = [0, 5, 19, 30, 44]
    os_, ls_ = [], []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        o = torch.empty(q.shape, dtype=torch.float32, device="cuda")
        lse = torch.empty(q.shape[:2], dtype=torch.float32, device="cuda")
        fs().paged_quant_attention_cuda(dev(q), cache, page_range=(lo, hi), partial_out=(o, lse))
        os_.append(o)
        ls_.append(lse)
    merged = fs().merge_partials(torch.stack(os_), torch.stack(ls_))
    close(merged, full.float().cpu().numpy(), atol=1e-3, rtol=1e-3)
    close(merged, O.paged_quant_attention(q, oc))
    # a window past every request's end is empty: LSE -inf, O = 0
    o = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    lse = torch.empty(q.shape[:2], dtype=torch.float32, device="cuda")
    fs().paged_quant_attention_cuda(dev(q), cache, page_range=(100, 200), partial_out=(o, lse))
    assert torch.all(torch.isneginf(lse)) and torch.all(o == 0)


def test_validation_errors():
    f = fs()
    g = load_golden("paged_contiguous")
    cache = paged_from_golden(g)
    with pytest.raises(RuntimeError):
        f.paged_quant_attention_cuda(torch.zeros(3, 4, 128, dtype=torch.float16), cache)
    with pytest.raises(ValueError):
        f.paged_quant_attention_cuda(dev(g["q"])[:2], cache)
    with pytest.raises(ValueError):
        f.paged_quant_attention_cuda(dev(g["q"])[:, :3], cache)  # 3 q heads over 4 kv heads


# ---------------------------------------------------------------------------------
# append / allocator
# ---------------------------------------------------------------------------------


def test_functional_cache_append_bit_exact():
    g = load_golden("cache_append")
    f = fs()
    c0 = f.PagedKVCache(qt_dev(g, "kq0"), qt_dev(g, "vq0"), dev(g["table0"]), dev(g["lengths0"]), 16, 7)
    c1 = c0.append(dev(g["k_new"]), dev(g["v_new"]))
    same_quant(c1.k_quant, g.quant("kq1"))
    same_quant(c1.v_quant, g.quant("vq1"))
    np.testing.assert_array_equal(c1.block_table.cpu().numpy(), g["table1"])
    np.testing.assert_array_equal(c1.lengths.cpu().numpy(), g["lengths1"])
    assert c1.max_seq_len == int(g["max_seq_len1"])


class _DevTokens(dict):
    def __getitem__(self, k):
        v = dict.__getitem__(self, k)
        return dev(v) if isinstance(v, np.ndarray) and k.startswith("tok.") else v


def test_allocator_lifecycle_bit_exact():
    from test_oracle_golden import replay_allocator

    g = load_golden("allocator_lifecycle")
    f = fs()
    a = f.PagedKVAllocator(capacity_blocks=int(g["capacity"]), heads=int(g["heads"]), head_dim=int(g["head_dim"]),
                           block_size=int(g["block_size"]), device="cuda")
    replay_allocator(_DevTokens(g), a)
    same_quant(a.k_quant, g.quant("kq"))
    same_quant(a.v_quant, g.quant("vq"))
    assert a.free_blocks == [int(x) for x in g["free_blocks"]]
    cache = a.to_cache([30, 40, 50])
    np.testing.assert_array_equal(cache.block_table.cpu().numpy(), g["table"])
    np.testing.assert_array_equal(cache.lengths.cpu().numpy(), g["lengths"])
    st = a.stats()
    for k, v in zip(g["stats_keys"], g["stats_vals"]):
        assert st[str(k)] == pytest.approx(float(v), abs=0, rel=1e-12)
    # H=2, D=128: attention over the allocator's cache
    out = f.paged_quant_attention_cuda(dev(g["q"]), cache)
    close(out, g["out"])


@pytest.mark.parametrize("D,bs", [(128, 16),   # the serving shape: register-resident page update
                                  (64, 8),     # E = 512, the smallest vector block
                                  (256, 32),   # E = 8192
                                  (32, 8)])    # E = 256: the shared-memory page update
def test_allocator_random_decode_loop_matches_oracle(D, bs):
    rng = np.random.default_rng(11 + D + bs)
    f = fs()
    H, cap = 4, 64
    ga = f.PagedKVAllocator(capacity_blocks=cap, heads=H, head_dim=D, block_size=bs, device="cuda")
    oa = O.OAllocator(cap, H, D, bs)
    live = []
    nxt = 0
    for step in range(60):
        if len(live) < 5 and rng.random() < 0.5:
            n = int(rng.integers(1, 70))
            k = rng.standard_normal((1, H, n, D)).astype(np.float16)
            v = rng.standard_normal((1, H, n, D)).astype(np.float16)
            if len(oa.free_blocks) >= (n + bs - 1) // bs + 8:
                ga.add_request(nxt, dev(k), dev(v))
                oa.add_request(nxt, k, v)
                live.append(nxt)
                nxt += 1
        if live and len(oa.free_blocks) > 8:
            t = int(rng.integers(1, 3))
            k = rng.standard_normal((len(live), H, t, D)).astype(np.float16)
            v = rng.standard_normal((len(live), H, t, D)).astype(np.float16)
            ga.append_batch(live, dev(k), dev(v))
            oa.append_batch(live, k, v)
        if live and rng.random() < 0.2:
            r = live.pop(int(rng.integers(0, len(live))))
            ga.release_request(r)
            oa.release_request(r)
    same_quant(ga.k_quant, oa.k_quant)
    same_quant(ga.v_quant, oa.v_quant)
    assert ga.free_blocks == oa.free_blocks
    if live:
        q = rng.standard_normal((len(live), H, D)).astype(np.float16)
        close(f.paged_quant_attention_cuda(dev(q), ga.to_cache(live)), O.paged_quant_attention(q, oa.to_cache(live)))


@pytest.mark.parametrize("D,bs,chunks", [(128, 16, "1"), (128, 16, "2"), (128, 16, "4"), (64, 64, "2"),
                                         (64, 8, "2")])
def test_page_update_vector_and_scalar_kernels_bit_identical(monkeypatch, D, bs, chunks):
    """The same prefill + append + reuse sequence through the register-resident page
    update (whose quantizer replaces the division by a reciprocal product except near a
    rounding boundary) and through the shared-memory one with the plain correctly
    rounded division (forced by FLASHSPEC_PAGE_UPDATE_SCALAR): identical bytes, scales and
    zero points, for fp16, bf16 and fp32 token sources and value ranges from 1e-3 to 1e3
    (about 4M quantized elements, a few thousand of them near a half-integer)."""
    rng = np.random.default_rng(21)
    f = fs()
    H, cap = 4, 700
    pools = []
    for scalar in (False, True):
        monkeypatch.setenv("FLASHSPEC_PAGE_UPDATE_CHUNKS", chunks)
        if scalar:
            monkeypatch.setenv("FLASHSPEC_PAGE_UPDATE_SCALAR", "1")
        r = np.random.default_rng(21)
        a = f.PagedKVAllocator(capacity_blocks=cap, heads=H, head_dim=D, block_size=bs, device="cuda")
        sizes = [(37, torch.float16, 3.0), (16, torch.bfloat16, 1e-3), (90, torch.float32, 1e3),
                 (64 * bs, torch.float32, 1.0), (64 * bs + 5, torch.float16, 30.0)]
        for i, (n, dt, sc) in enumerate(sizes):
            off = r.standard_normal((1, H, 1, D)).astype(np.float32) * sc
            k = torch.from_numpy(r.standard_normal((1, H, n, D)).astype(np.float32) * sc + off).to(dt)
            v = torch.from_numpy(r.standard_normal((1, H, n, D)).astype(np.float32) * sc).to(dt)
            a.add_request(i, k.cuda(), v.cuda())
        for _ in range(20):
            k = torch.from_numpy(r.standard_normal((len(sizes), H, 1, D)).astype(np.float16)).cuda()
            a.append_batch(list(range(len(sizes))), k, k * 0.5)
        a.release_request(1)
        a.add_request(9, k[:1].repeat(1, 1, 5, 1), k[:1].repeat(1, 1, 5, 1))
        torch.cuda.synchronize()
        pools.append([t.clone() for qt in (a.k_quant, a.v_quant) for t in (qt.values, qt.scale, qt.zero_point)])
        monkeypatch.delenv("FLASHSPEC_PAGE_UPDATE_SCALAR", raising=False)
    for x, y in zip(*pools):
        assert torch.equal(x, y)


# ---------------------------------------------------------------------------------
# balanced (stream-K) kernel, forced through FLASHSPEC_DECODE_KERNEL
# ---------------------------------------------------------------------------------


@pytest.mark.parametrize("kernel", ["balanced", "split"])
@pytest.mark.parametrize("lens,hq,hkv", [([1, 16, 17, 250, 31, 512, 100], 8, 4),
                                         ([2000, 3], 16, 2),      # few pairs: many warps share a pair
                                         ([0, 40, 0, 7], 4, 4),   # empty requests
                                         ([4096], 8, 8)])
def test_decode_kernels_vs_oracle(monkeypatch, kernel, lens, hq, hkv):
    monkeypatch.setenv("FLASHSPEC_DECODE_KERNEL", kernel)
    rng = np.random.default_rng(sum(lens) + hq)
    q, oc = _random_paged(rng, len(lens), hq, hkv, [max(n, 1) for n in lens])
    oc.lengths[:] = lens
    out = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc))
    ref = O.paged_quant_attention(q, oc)
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.all(out[i] == 0)
        else:
            close(out[i], ref[i])


def test_balanced_kernel_deterministic_and_matches_split(monkeypatch):
    rng = np.random.default_rng(21)
    q, oc = _random_paged(rng, 5, 8, 2, [900, 13, 1500, 64, 333])
    cache = _cache_dev(oc)
    monkeypatch.setenv("FLASHSPEC_DECODE_KERNEL", "balanced")
    a = fs().paged_quant_attention_cuda(dev(q), cache)
    b = fs().paged_quant_attention_cuda(dev(q), cache)
    assert torch.equal(a, b)
    monkeypatch.setenv("FLASHSPEC_DECODE_KERNEL", "split")
    c = fs().paged_quant_attention_cuda(dev(q), cache)
    close(a, c.float().cpu().numpy(), atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("skew,cost", [(0, 0), (256, 0), (0, 64), (200, 17)])
def test_balanced_share_division_variants(monkeypatch, skew, cost):
    """Tier weights and per-pair piece costs only move the share boundaries of the
    balanced kernel: any setting gives the oracle's result.  The batch is large enough
    for a full grid (three CTA tiers per SM) and mixes empty requests, one-token requests
    and pairs shorter than a share."""
    monkeypatch.setenv("FLASHSPEC_DECODE_KERNEL", "balanced")
    monkeypatch.setenv("FLASHSPEC_TIER_SKEW", str(skew))
    monkeypatch.setenv("FLASHSPEC_PIECE_COST", str(cost))
    lens = [3000, 0, 1, 17, 450, 0, 2049, 96, 5, 1200] * 3
    rng = np.random.default_rng(skew + cost)
    q, oc = _random_paged(rng, len(lens), 16, 8, [max(n, 1) for n in lens])
    oc.lengths[:] = lens
    out = fs().paged_quant_attention_cuda(dev(q), _cache_dev(oc))
    ref = O.paged_quant_attention(q, oc)
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.all(out[i] == 0)
        else:
            close(out[i], ref[i])


def test_balanced_page_windows_merge_equal_full(monkeypatch):
    monkeypatch.setenv("FLASHSPEC_DECODE_KERNEL", "balanced")
    rng = np.random.default_rng(8)
    q, oc = _random_paged(rng, 3, 8, 8, [700, 333, 1200])
    cache = _cache_dev(oc)
    os_, ls_ = [], []
    for lo, hi in [(0, 7), (7, 40), (40, 80)]:
        o = torch.empty(q.shape, dtype=torch.float32, device="cuda")
        lse = torch.empty(q.shape[:2], dtype=torch.float32, device="cuda")
        fs().paged_quant_attention_cuda(dev(q), cache, page_range=(lo, hi), partial_out=(o, lse))
        os_.append(o)
        ls_.append(lse)
    close(fs().merge_partials(torch.stack(os_), torch.stack(ls_)), O.paged_quant_attention(q, oc))


def test_fused_balanced_vs_golden(monkeypatch):
    monkeypatch.setenv("FLASHSPEC_DECODE_KERNEL", "balanced")
    for name in ["fused_s129", "fused_s1500", "fused_nolen_s200"]:
        g = load_golden(name)
        lengths = dev(g["lengths"]) if "lengths" in g else None
        close(fs().fused_dequant_attention_cuda(dev(g["q"]), qt_dev(g, "kq"), qt_dev(g, "vq"), lengths), g["out"])


def test_sequence_sharded_decoder_single_rank_and_graph_replay():
    from flashspec_b200.dist import SequenceShardedDecoder

    rng = np.random.default_rng(12)
    q, oc = _random_paged(rng, 2, 16, 2, [900, 301])
    cache = _cache_dev(oc)
    qd = dev(q)
    dec = SequenceShardedDecoder()
    out = dec(qd, cache, cache.block_table.shape[1])
    close(out, O.paged_quant_attention(q, oc))
    replay, gout = dec.capture(qd, cache, cache.block_table.shape[1])
    qd.copy_(dev(rng.standard_normal(q.shape).astype(np.float16)))  # new query, same graph
    replay()
    torch.cuda.synchronize()
    close(gout, O.paged_quant_attention(qd.cpu().numpy(), oc))
