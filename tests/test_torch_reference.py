"""Pin the torch-CPU reference arm (``oracle/torch_reference.py``) against the vectors
recorded from the reference itself: the quantizer bit-exact, attention outputs of the
``fused`` / ``paged`` backends within 1e-3 abs (fp16 outputs; only the summation order
of the fp32 einsums may differ), the configuration builders' algorithmic bytes."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torch_reference as T
from conftest import load_golden


def tq(g, prefix):
    return T.TQuant(torch.from_numpy(g[f"{prefix}.values"]), torch.from_numpy(g[f"{prefix}.scale"]),
                    torch.from_numpy(g[f"{prefix}.zero_point"]), int(g[f"{prefix}.block_size"]),
                    tuple(int(x) for x in g[f"{prefix}.original_shape"]))


@pytest.mark.parametrize("name,bs", [("quant_fp32_b8", 8), ("quant_fp16_b16", 16), ("quant_edge_b16", 16)])
def test_quantizer_bit_exact(name, bs):
    g = load_golden(name)
    got = T.quantize_int8_per_block(torch.from_numpy(g["x"]), bs)
    np.testing.assert_array_equal(got.values.numpy(), g["q.values"])
    np.testing.assert_array_equal(got.scale.numpy().view(np.uint32), g["q.scale"].view(np.uint32))
    np.testing.assert_array_equal(got.zero_point.numpy(), g["q.zero_point"])
    deq = T.dequantize_int8_per_block(tq(g, "q")).numpy()
    np.testing.assert_array_equal(deq.view(np.uint32), g["deq"].view(np.uint32))


@pytest.mark.parametrize("name", ["fused_s129", "fused_s1500", "fused_nolen_s200"])
def test_fused_backend(name):
    g = load_golden(name)
    lengths = torch.from_numpy(g["lengths"]) if "lengths" in g else None
    got = T.fused_dequant_attention(torch.from_numpy(g["q"]), tq(g, "kq"), tq(g, "vq"), lengths)
    np.testing.assert_allclose(got.float().numpy(), g["out"].astype(np.float32), atol=1e-3, rtol=0)


@pytest.mark.parametrize("name", ["paged_contiguous", "paged_shuffled", "paged_interleaved", "paged_gqa4"])
def test_paged_backend(name):
    g = load_golden(name)
    cache = T.TPagedCache(tq(g, "kq"), tq(g, "vq"), torch.from_numpy(g["block_table"]),
                          torch.from_numpy(g["lengths"]), 16, int(g["max_seq_len"]))
    got = T.paged_quant_attention(torch.from_numpy(g["q"]), cache)
    np.testing.assert_allclose(got.float().numpy(), g["out"].astype(np.float32), atol=1e-3, rtol=0)


def test_reference_attention_fp32():
    g = load_golden("reference_attention_fp32")
    got = T.reference_attention(torch.from_numpy(g["q"]), torch.from_numpy(g["k"]), torch.from_numpy(g["v"]),
                                torch.from_numpy(g["lengths"]))
    np.testing.assert_allclose(got.numpy(), g["out"], rtol=1e-5, atol=1e-6)


def test_host_builders_match_the_benchmark_bytes():
    assert T.algorithmic_bytes(16, 32, 32, [4096] * 16, table_cols=256) == 538_738_816
    assert T.algorithmic_bytes(8, 32, 32, [2048] * 8, with_lengths=False) == 134_742_016
    lens = T.cfg2_lengths()
    assert lens[0] == 8192 and lens[-1] == 128 and len(lens) == 64


def test_small_host_workload_runs_and_matches_numpy_oracle():
    """A scaled-down paged workload through both CPU restatements (torch and numpy)."""
    import flashspec_oracle as O

    wl = T.paged_host_workload("tiny", 3, 8, 2, [100, 37, 64], seed=4)
    got = wl.call()

    def oq(t):
        return O.OQuant(t.values.numpy(), t.scale.numpy(), t.zero_point.numpy(), 16, t.original_shape)

    c = wl.cache
    oc = O.OPagedCache(oq(c.k_quant), oq(c.v_quant), c.block_table.numpy(), c.lengths.numpy(), 16, c.max_seq_len)
    ref = O.paged_quant_attention(wl.q.numpy(), oc)
    np.testing.assert_allclose(got.float().numpy(), ref.astype(np.float32), atol=1e-3, rtol=0)


def test_allocator_lifecycle_bit_exact():
    """The torch allocator behind the reduced cfg4 reference loop replays the recorded
    allocator log (prefill, appends incl. stale-page reuse, releases) bit-exactly."""
    g = load_golden("allocator_lifecycle")
    a = T.TAllocator(int(g["capacity"]), int(g["heads"]), int(g["head_dim"]), int(g["block_size"]))
    step = 0
    for op, rid, rids, n in zip(g["ops"], g["op_rid"], g["op_rids"], g["op_n"]):
        if op == 0:
            a.add_request(int(rid), torch.from_numpy(g[f"tok.add{rid}_k"]), torch.from_numpy(g[f"tok.add{rid}_v"]))
        elif op == 1:
            ids = [int(r) for r in rids if r >= 0]
            a.append_batch(ids, torch.from_numpy(g[f"tok.app{step}_k"]), torch.from_numpy(g[f"tok.app{step}_v"]))
            step += 1
        else:
            a.release_request(int(rid))
    for qt, p in ((a.k_quant, "kq"), (a.v_quant, "vq")):
        np.testing.assert_array_equal(qt.values.numpy().reshape(g[f"{p}.values"].shape), g[f"{p}.values"])
        np.testing.assert_array_equal(qt.scale.numpy().reshape(-1).view(np.uint32),
                                      g[f"{p}.scale"].reshape(-1).view(np.uint32))
        np.testing.assert_array_equal(qt.zero_point.numpy().reshape(-1), g[f"{p}.zero_point"].reshape(-1))
    assert a.free_blocks == [int(x) for x in g["free_blocks"]]
    cache = a.to_cache([30, 40, 50])
    np.testing.assert_array_equal(cache.block_table.numpy(), g["table"])
    np.testing.assert_array_equal(cache.lengths.numpy(), g["lengths"])
    out = T.paged_quant_attention(torch.from_numpy(g["q"]), cache)
    np.testing.assert_allclose(out.float().numpy(), g["out"].astype(np.float32), atol=1e-3, rtol=0)


def test_reduced_serving_loop_runs():
    res = T.serving_loop(T.ServingParams(steps=2, max_live=2, prompt_max=256, out_max=80))
    assert res["decode_tokens"] > 0 and res["bytes_moved"] > 0
