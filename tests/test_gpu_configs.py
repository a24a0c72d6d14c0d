"""GPU parity at the benchmarked configurations, through the same plans ``bench.py`` runs.

Every GPU call here is the full-size call of its configuration (cfg0 B8 H32 S2048
contiguous; cfg1 B16 H32 S4096 over a 4506-page pool with a shuffled table; cfg2 B64
32q/8kv ragged with round-robin pages, at the configured S=4 and with the default
balanced plan; cfg3 B2 64q/8kv S131072 on one GPU, whole and as two page windows
merged).  The CPU oracle then checks a subset of the requests of that call (their pages
only), which keeps the CPU time to seconds while the GPU side exercises the large-size
index arithmetic, the pool with slack, the big tables and the plans' share arithmetic.

Tolerance: |got - oracle| <= 2e-3 + 1e-2 * |oracle| elementwise (fp16 output)."""

from __future__ import annotations

import ctypes as C

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


def close(got: torch.Tensor, ref: np.ndarray):
    ref_t = torch.as_tensor(np.asarray(ref, dtype=np.float32))
    err = (got.detach().float().cpu() - ref_t).abs()
    bad = err > ATOL + RTOL * ref_t.abs()
    assert not bool(bad.any()), f"{int(bad.sum())} elements out of tolerance, max abs err {err.max().item():.3e}"
    return err.max().item()


def oracle_paged_subset(q: torch.Tensor, cache, reqs):
    """The oracle's paged attention on requests ``reqs`` of a device cache: only the
    pages their table rows reference are copied to the host (the oracle would otherwise
    dequantize the whole pool, slack included, for pages that never enter the result)."""
    idx = torch.tensor(reqs, dtype=torch.long, device=cache.block_table.device)
    table = cache.block_table.index_select(0, idx)
    used = torch.unique(table[table >= 0])
    remap = torch.full((int(cache.k_quant.values.shape[0]),), -1, dtype=torch.int64, device=table.device)
    remap[used] = torch.arange(used.numel(), device=table.device)
    sub_table = torch.where(table >= 0, remap[table.clamp_min(0)], torch.full_like(table, -1))

    def sub(qt):
        return O.OQuant(qt.values[used].cpu().numpy(), qt.scale[used].cpu().numpy(),
                        qt.zero_point[used].cpu().numpy(), 16, (int(used.numel()),) + tuple(qt.original_shape[1:]))

    lengths = cache.lengths.index_select(0, idx).cpu().numpy()
    oc = O.OPagedCache(sub(cache.k_quant), sub(cache.v_quant), sub_table.cpu().numpy(), lengths, 16,
                       int(cache.max_seq_len))
    return O.paged_quant_attention(q.index_select(0, idx).cpu().numpy(), oc)


def plan_of(q, cache, num_splits=0):
    """(workspace bytes, splits) the library's plan picks for this call; splits 0 = the
    balanced kernel."""
    from flashspec_b200 import _lib
    from flashspec_b200.attention import _decode_args

    a = _decode_args(_lib.FS_LAYOUT_PAGED, q, cache.k_quant, cache.v_quant, q, cache.lengths, cache.block_table,
                     int(cache.k_quant.values.shape[0]), int(cache.max_seq_len), int(cache.k_quant.original_shape[1]),
                     None)
    a.num_splits = num_splits
    nbytes, splits = C.c_size_t(0), C.c_int32(0)
    assert _lib.load().fs_decode_workspace_size(C.byref(a), C.byref(nbytes), C.byref(splits)) == 0
    return nbytes.value, splits.value


@pytest.fixture(scope="module")
def cfg1():
    from flashspec_b200 import configs

    wl = configs.cfg1()
    yield wl
    del wl
    torch.cuda.empty_cache()


@pytest.fixture(scope="module")
def cfg2():
    from flashspec_b200 import configs

    wl = configs.cfg2()
    yield wl
    del wl
    torch.cuda.empty_cache()


def test_cfg0_fused_full_call_vs_oracle():
    import flashspec_b200 as fs
    from flashspec_b200 import configs

    wl = configs.cfg0()
    out = fs.fused_dequant_attention_cuda(wl.q, wl.k_quant, wl.v_quant)
    torch.cuda.synchronize()
    reqs = [0, 5, 7]

    def sub(qt):
        v = qt.values[reqs].cpu().numpy()
        return O.OQuant(v, qt.scale[reqs].cpu().numpy(), qt.zero_point[reqs].cpu().numpy(), 16,
                        (len(reqs),) + tuple(qt.original_shape[1:]))

    ref = O.fused_dequant_attention(wl.q[reqs].cpu().numpy(), sub(wl.k_quant), sub(wl.v_quant))
    close(out[reqs], ref)
    assert not torch.isnan(out).any()


def test_cfg1_bench_plan_vs_oracle(cfg1):
    import flashspec_b200 as fs

    wl = cfg1
    assert wl.cache.k_quant.values.shape[0] == 4506  # 4096 pages + 10% slack
    _, splits = plan_of(wl.q, wl.cache)
    assert splits == 0, "cfg1 is benchmarked on the balanced kernel"
    out = fs.paged_quant_attention_cuda(wl.q, wl.cache)
    torch.cuda.synchronize()
    reqs = [0, 7, 15]
    close(out[reqs], oracle_paged_subset(wl.q, wl.cache, reqs))
    assert not torch.isnan(out).any()


def test_cfg1_split_kernel_vs_oracle(cfg1, monkeypatch):
    """The same call forced onto the split kernel (the plan for fewer pairs than CTAs)."""
    import flashspec_b200 as fs

    wl = cfg1
    monkeypatch.setenv("FLASHSPEC_DECODE_KERNEL", "split")
    out = fs.paged_quant_attention_cuda(wl.q, wl.cache)
    torch.cuda.synchronize()
    reqs = [3, 12]
    close(out[reqs], oracle_paged_subset(wl.q, wl.cache, reqs))


@pytest.mark.parametrize("num_splits", [4, 0])
def test_cfg2_ragged_gqa_vs_oracle(cfg2, num_splits):
    """num_splits=4 is the configured split-K; 0 is the library's default plan (balanced)."""
    import flashspec_b200 as fs

    wl = cfg2
    _, splits = plan_of(wl.q, wl.cache, num_splits)
    assert splits == (4 if num_splits == 4 else 0)
    out = fs.paged_quant_attention_cuda(wl.q, wl.cache, num_splits=num_splits or None)
    torch.cuda.synchronize()
    reqs = [0, 21, 42, 63]  # longest (8192) ... shortest (128)
    close(out[reqs], oracle_paged_subset(wl.q, wl.cache, reqs))
    assert not torch.isnan(out).any()


def test_cfg3_long_context_full_and_two_windows_vs_oracle():
    """cfg3 on one GPU: the whole 131072-token requests with the default plan (the
    one-wave split kernel), and the same call as two logical page windows whose (O, LSE)
    partials are merged -- the single-GPU form of the sequence-sharded step."""
    import flashspec_b200 as fs
    from flashspec_b200 import configs

    wl = configs.cfg3()
    q, cache = wl.q, wl.cache
    n_pages = int(cache.block_table.shape[1])
    assert n_pages == 8192
    _, splits = plan_of(q, cache)
    assert splits > 1
    out = fs.paged_quant_attention_cuda(q, cache)
    parts_o, parts_l = [], []
    for lo, hi in [(0, 4096), (4096, n_pages)]:
        o = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        lse = torch.empty(q.shape[:2], dtype=torch.float32, device=q.device)
        fs.paged_quant_attention_cuda(q, cache, page_range=(lo, hi), partial_out=(o, lse))
        parts_o.append(o)
        parts_l.append(lse)
    merged = fs.merge_partials(torch.stack(parts_o), torch.stack(parts_l), torch.float16)
    torch.cuda.synchronize()
    ref = oracle_paged_subset(q, cache, [1])
    close(out[1:2], ref)
    close(merged[1:2], ref)
    del wl, q, cache
    torch.cuda.empty_cache()
