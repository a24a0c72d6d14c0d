"""GPU parity of tree-attention verify (speculative decoding) against the dense
tree-mask oracle: chains, forks of several depths and branch factors, GQA with the
nodes split over several prefix passes, an empty prefix, bf16, and the single-path case
matching the plain paged decode.  Tolerance |got - ref| <= 2e-3 + 1e-2 |ref|."""

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


def prefix_cache(rng, b, hkv, d, lens, page=16):
    smax = max(max(lens), 1)
    k = rng.standard_normal((b, hkv, smax, d)).astype(np.float16)
    v = rng.standard_normal((b, hkv, smax, d)).astype(np.float16)
    bps = (smax + page - 1) // page
    oc = O.paged_from_dense(k, v, page, lengths=np.array(lens), pattern="shuffled", perm=rng.permutation(b * bps))
    dc = fs().PagedKVCache(*(fs().QuantizedTensor(dev(t.values), dev(t.scale), dev(t.zero_point), page,
                                                  tuple(t.original_shape)) for t in (oc.k_quant, oc.v_quant)),
                           dev(oc.block_table), dev(oc.lengths), page, smax)
    return oc, dc


def random_tree(rng, b, n, branch):
    """parents[b, i] in [-1, i): node i hangs off one of the last `branch` nodes (or the
    prefix), which gives chains for branch 1 and bushier trees for larger ones."""
    par = np.full((b, n), -1, np.int64)
    for bi in range(b):
        for i in range(1, n):
            par[bi, i] = rng.integers(max(-1, i - branch), i)
    return par


@pytest.mark.parametrize("n,branch,hq,hkv,d", [(1, 1, 8, 8, 128), (8, 1, 4, 4, 128), (12, 3, 8, 2, 128),
                                               (16, 4, 32, 8, 128), (7, 2, 4, 4, 64)])
def test_tree_verify_vs_dense_mask(n, branch, hq, hkv, d):
    rng = np.random.default_rng(n * 10 + branch + d)
    b = 3
    lens = [300, 17, 1]
    oc, dc = prefix_cache(rng, b, hkv, d, lens)
    q = rng.standard_normal((b, n, hq, d)).astype(np.float16)
    tk = rng.standard_normal((b, n, hkv, d)).astype(np.float16)
    tv = rng.standard_normal((b, n, hkv, d)).astype(np.float16)
    par = random_tree(rng, b, n, branch)
    out, stats = fs().tree_verify_attention_cuda(dev(q), dc, dev(tk), dev(tv), dev(par), return_stats=True)
    close(out, O.tree_verify_attention(q, oc, tk, tv, par))
    assert stats["nodes"] == n and stats["prefix_passes"] >= 1


def test_tree_verify_empty_prefix_and_bf16():
    rng = np.random.default_rng(3)
    b, n, hq, hkv, d = 2, 5, 8, 4, 128
    oc, dc = prefix_cache(rng, b, hkv, d, [64, 1])
    oc.lengths[1] = 0
    dc = fs().PagedKVCache(dc.k_quant, dc.v_quant, dc.block_table, dev(oc.lengths), 16, dc.max_seq_len)
    q = torch.from_numpy(rng.standard_normal((b, n, hq, d)).astype(np.float32)).to(torch.bfloat16)
    tk = torch.from_numpy(rng.standard_normal((b, n, hkv, d)).astype(np.float32)).to(torch.bfloat16)
    tv = torch.from_numpy(rng.standard_normal((b, n, hkv, d)).astype(np.float32)).to(torch.bfloat16)
    par = np.array([[-1, 0, 0, 1, 2], [-1, -1, 1, 2, 0]])
    out = fs().tree_verify_attention_cuda(q.cuda(), dc, tk.cuda(), tv.cuda(), dev(par))
    assert out.dtype == torch.bfloat16
    close(out, O.tree_verify_attention(q.float().numpy(), oc, tk.float().numpy(), tv.float().numpy(), par))


def test_single_path_matches_paged_decode():
    """A chain of T draft tokens whose K/V are the last T tokens of a cache: the chain's
    last node sees exactly what a paged decode of the whole cache sees."""
    rng = np.random.default_rng(4)
    b, hq, hkv, d, T = 2, 8, 4, 128, 5
    oc, dc = prefix_cache(rng, b, hkv, d, [200, 77])
    kd, vd = O.paged_to_dense(oc)
    q_last = rng.standard_normal((b, hq, d)).astype(np.float16)
    full = fs().paged_quant_attention_cuda(dev(q_last), dc)
    # the prefix: the same cache T tokens shorter; the draft tokens: the dequantized last T
    short = fs().PagedKVCache(dc.k_quant, dc.v_quant, dc.block_table, dc.lengths - T, 16, dc.max_seq_len)
    tk = np.zeros((b, T, hkv, d), np.float32)
    tv = np.zeros((b, T, hkv, d), np.float32)
    for bi in range(b):
        L = int(oc.lengths[bi])
        tk[bi] = kd[bi, :, L - T:L].transpose(1, 0, 2)
        tv[bi] = vd[bi, :, L - T:L].transpose(1, 0, 2)
    q = np.repeat(q_last[:, None], T, axis=1)
    par = np.tile(np.arange(-1, T - 1), (b, 1))
    out = fs().tree_verify_attention_cuda(dev(q), short, dev(tk.astype(np.float16)), dev(tv.astype(np.float16)),
                                          dev(par))
    close(out[:, -1], full.float().cpu().numpy())


@pytest.mark.parametrize("bad", [[[-1, 1, 0]], [[-1, 0, 3]], [[-2, 0, 1]], [[0, 0, 1]]])
def test_invalid_trees_raise(bad):
    rng = np.random.default_rng(6)
    oc, dc = prefix_cache(rng, 1, 2, 64, [40])
    q = dev(rng.standard_normal((1, 3, 2, 64)).astype(np.float16))
    t = dev(rng.standard_normal((1, 3, 2, 64)).astype(np.float16))
    with pytest.raises(ValueError):
        fs().tree_verify_attention_cuda(q, dc, t, t, dev(np.array(bad)))
