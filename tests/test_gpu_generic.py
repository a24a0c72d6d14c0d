"""GPU parity of the generic decode kernel: the cache shapes outside the tuned kernels.

The reference accepts head_dim up to 256, any quantization block, and pages that hold
several quantization blocks (src/flashspec/triton_paged.py:242-246); its own CUDA parity
tests run head_dim 64 with lengths [129, 113] (tests/test_flashspec.py:92-105,177-198).
Every case here goes through the public entry points and is checked against the CPU
oracle at |got - ref| <= 2e-3 + 1e-2 |ref| (fp16 or bf16 output)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import flashspec_oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")


def fs():
    import flashspec_b200

    return flashspec_b200


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def close(got, ref):
    ref_t = torch.as_tensor(np.asarray(ref, dtype=np.float32))
    err = (got.detach().float().cpu() - ref_t).abs()
    bad = err > ATOL + RTOL * ref_t.abs()
    assert not bool(bad.any()), f"{int(bad.sum())} out of tolerance, max abs err {err.max().item():.3e}"


def qt_dev(oq):
    return fs().QuantizedTensor(dev(oq.values), dev(oq.scale), dev(oq.zero_point), int(oq.block_size),
                                tuple(oq.original_shape))


def make_paged(rng, b, hq, hkv, d, lens, page, qb, slack=3):
    """Pool of pages of `page` tokens quantized in blocks of `qb` tokens (values
    [P, Hkv, page / qb, qb, D]), pages of the requests scattered over the pool."""
    smax = max(max(lens), 1)
    ppr = (smax + page - 1) // page
    total = b * ppr + slack
    q = rng.standard_normal((b, hq, d)).astype(np.float32)
    pool_k = np.zeros((total, hkv, page, d), np.float32)
    pool_v = np.zeros((total, hkv, page, d), np.float32)
    perm = rng.permutation(total)[: b * ppr]
    table = perm.reshape(b, ppr).astype(np.int64)
    for i in range(b):
        for j in range(ppr):
            pool_k[table[i, j]] = rng.standard_normal((hkv, page, d))
            pool_v[table[i, j]] = rng.standard_normal((hkv, page, d))
    kq = O.quantize_int8_per_block(pool_k.astype(np.float16), qb)
    vq = O.quantize_int8_per_block(pool_v.astype(np.float16), qb)
    oc = O.OPagedCache(kq, vq, table, np.array(lens, np.int64), page, smax)
    return q, oc


def cache_dev(oc):
    return fs().PagedKVCache(qt_dev(oc.k_quant), qt_dev(oc.v_quant), dev(oc.block_table), dev(oc.lengths),
                             int(oc.block_size), int(oc.max_seq_len))


def test_fused_head_dim_64_reference_shape():
    """tests/test_flashspec.py:92-105 of the reference: B2 H3 S129 D64, lengths [129, 113]."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 3, 64)).astype(np.float16)
    k = rng.standard_normal((2, 3, 129, 64)).astype(np.float16)
    v = rng.standard_normal((2, 3, 129, 64)).astype(np.float16)
    lengths = np.array([129, 113], np.int64)
    kq, vq = O.quantize_int8_per_block(k, 16), O.quantize_int8_per_block(v, 16)
    out, stats = fs().fused_dequant_attention_cuda(dev(q), qt_dev(kq), qt_dev(vq), dev(lengths), return_stats=True)
    assert out.dtype == torch.float16
    close(out, O.fused_dequant_attention(q, kq, vq, lengths))
    assert stats["materializes_dense_kv"] == 0.0


def test_paged_head_dim_64_reference_shape():
    """tests/test_flashspec.py:177-198 of the reference: from_dense with 16-token pages."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal((2, 3, 64)).astype(np.float16)
    k = rng.standard_normal((2, 3, 129, 64)).astype(np.float16)
    v = rng.standard_normal((2, 3, 129, 64)).astype(np.float16)
    perm = rng.permutation(2 * 9)
    oc = O.paged_from_dense(k, v, 16, lengths=np.array([129, 113]), pattern="shuffled", perm=perm)
    close(fs().paged_quant_attention_cuda(dev(q), cache_dev(oc)), O.paged_quant_attention(q, oc))


@pytest.mark.parametrize("d,page,qb,hq,hkv", [
    (128, 16, 8, 8, 8),     # quant block 8
    (128, 32, 32, 8, 4),    # quant block 32
    (128, 32, 16, 8, 8),    # a page holds two quant blocks
    (64, 64, 16, 4, 4),     # four quant blocks per page
    (256, 16, 16, 8, 2),    # head_dim 256, GQA 4
    (32, 8, 8, 16, 2),      # head_dim 32, GQA 8
    (128, 64, 64, 4, 4),    # 64-token quant blocks
])
def test_paged_generic_shapes_vs_oracle(d, page, qb, hq, hkv):
    rng = np.random.default_rng(d + page + qb + hq)
    lens = [1, page, page + 1, 250, 31, 0, 7 * page - 3]
    q, oc = make_paged(rng, len(lens), hq, hkv, d, [max(n, 1) for n in lens], page, qb)
    oc.lengths[:] = lens
    q16 = q.astype(np.float16)
    out = fs().paged_quant_attention_cuda(dev(q16), cache_dev(oc))
    ref = O.paged_quant_attention(q16, oc)
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.all(out[i] == 0)
        else:
            close(out[i], ref[i])


@pytest.mark.parametrize("splits", [1, 3, 8])
def test_generic_split_counts(splits):
    rng = np.random.default_rng(50 + splits)
    lens = [700, 33, 512, 1]
    q, oc = make_paged(rng, len(lens), 8, 4, 64, lens, 32, 16)
    q16 = q.astype(np.float16)
    out = fs().paged_quant_attention_cuda(dev(q16), cache_dev(oc), num_splits=splits)
    close(out, O.paged_quant_attention(q16, oc))


def test_bf16_query_on_the_tuned_shape():
    """bf16 q with D=128 and 16-token pages: the output comes back in bf16."""
    rng = np.random.default_rng(7)
    lens = [300, 17, 1024]
    q, oc = make_paged(rng, len(lens), 8, 4, 128, lens, 16, 16)
    qb = torch.from_numpy(q).to(torch.bfloat16)
    out = fs().paged_quant_attention_cuda(qb.cuda(), cache_dev(oc))
    assert out.dtype == torch.bfloat16
    close(out, O.paged_quant_attention(qb.float().numpy(), oc))


def test_bf16_fused_head_dim_64():
    rng = np.random.default_rng(8)
    q = torch.from_numpy(rng.standard_normal((3, 4, 64)).astype(np.float32)).to(torch.bfloat16)
    k = rng.standard_normal((3, 4, 200, 64)).astype(np.float16)
    v = rng.standard_normal((3, 4, 200, 64)).astype(np.float16)
    kq, vq = O.quantize_int8_per_block(k, 8), O.quantize_int8_per_block(v, 8)
    lengths = np.array([200, 1, 99], np.int64)
    out = fs().fused_dequant_attention_cuda(q.cuda(), qt_dev(kq), qt_dev(vq), dev(lengths))
    assert out.dtype == torch.bfloat16
    close(out, O.fused_dequant_attention(q.float().numpy(), kq, vq, lengths))


def test_generic_page_windows_merge_to_the_whole():
    """Sequence-shard windows (partial O, LSE) of the generic path merge to the full result."""
    rng = np.random.default_rng(9)
    lens = [900, 301]
    q, oc = make_paged(rng, len(lens), 8, 2, 64, lens, 32, 16)
    q16 = dev(q.astype(np.float16))
    cache = cache_dev(oc)
    cols = int(cache.block_table.shape[1])
    os_, ls_ = [], []
    for lo, hi in [(0, 5), (5, 11), (11, cols)]:
        o = torch.empty(q16.shape, dtype=torch.float32, device="cuda")
        lse = torch.empty(q16.shape[:2], dtype=torch.float32, device="cuda")
        fs().paged_quant_attention_cuda(q16, cache, page_range=(lo, hi), partial_out=(o, lse))
        os_.append(o)
        ls_.append(lse)
    close(fs().merge_partials(torch.stack(os_), torch.stack(ls_)), O.paged_quant_attention(q.astype(np.float16), oc))


def test_generic_masks_unallocated_and_reports_bad_pages():
    rng = np.random.default_rng(10)
    lens = [120, 90]
    q, oc = make_paged(rng, len(lens), 4, 4, 64, lens, 32, 8)
    q16 = q.astype(np.float16)
    oc.lengths[1] = 60  # request 1 needs 2 of its 3 pages
    oc.block_table[1, 2] = -1
    ref = O.paged_quant_attention(q16, oc)
    cache = cache_dev(oc)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    close(fs().paged_quant_attention_cuda(dev(q16), cache, device_status=status), ref)
    assert int(status.item()) == 0
    bad = cache.block_table.clone()
    bad[1, 0] = 10**6  # outside the pool: the page is skipped and reported
    bad_cache = fs().PagedKVCache(cache.k_quant, cache.v_quant, bad, cache.lengths, cache.block_size,
                                  cache.max_seq_len)
    out = fs().paged_quant_attention_cuda(dev(q16), bad_cache, device_status=status)
    torch.cuda.synchronize()
    close(out[0], ref[0])
    assert int(status.item()) & 1


def test_unsupported_shapes_raise():
    rng = np.random.default_rng(11)
    q, oc = make_paged(rng, 2, 4, 4, 64, [40, 40], 16, 16)
    q32 = dev(q)  # fp32 q
    with pytest.raises(ValueError):
        fs().paged_quant_attention_cuda(q32, cache_dev(oc))
