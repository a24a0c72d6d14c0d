"""Config-4 serving loop on the GPU, replayed on the CPU oracle allocator: every
attention output within tolerance and the final pool / free list bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import flashspec_oracle as O

pytestmark = pytest.mark.gpu


def test_serving_loop_matches_oracle_allocator():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from flashspec_b200.serving import ServingConfig, run

    cfg = ServingConfig(steps=40, arrival_rate=1.5, max_live=6, prompt_min=5, prompt_max=90, out_min=3, out_max=35,
                        heads=2, head_dim=128, seed=5, capacity_pages=40)
    rec = []
    res = run(cfg, measure=True, recorder=rec)
    assert res["decode_tokens"] > 0 and res["finished"] > 0
    ora = O.OAllocator(cfg.capacity(), cfg.heads, cfg.head_dim, cfg.page)
    n_attn = 0
    for op, a, x, y in rec:
        if op == "add":
            ora.add_request(a, x, y)
        elif op == "append":
            ora.append_batch(a, x, y)
        elif op == "release":
            ora.release_request(a)
        elif op == "attn":
            ref = O.paged_quant_attention(x, ora.to_cache(a)).astype(np.float32)
            err = np.abs(y.astype(np.float32) - ref)
            assert np.all(err <= 2e-3 + 1e-2 * np.abs(ref)), f"max err {err.max()}"
            n_attn += len(a)
        else:  # final device allocator state == oracle state, bit for bit
            dev = a
            np.testing.assert_array_equal(dev.k_quant.values.cpu().numpy(), ora.k_quant.values)
            np.testing.assert_array_equal(dev.v_quant.values.cpu().numpy(), ora.v_quant.values)
            np.testing.assert_array_equal(dev.k_quant.scale.cpu().numpy().view(np.uint32),
                                          ora.k_quant.scale.view(np.uint32))
            np.testing.assert_array_equal(dev.v_quant.zero_point.cpu().numpy(), ora.v_quant.zero_point)
            assert dev.free_blocks == ora.free_blocks
            assert dev.stats() == ora.stats()
    assert n_attn == res["decode_tokens"]


def test_device_table_follows_the_host_table():
    """to_cache keeps the slot table and lengths on the device and uploads only what
    changed; over a random lifecycle (prefills, single and multi-token appends that open
    pages, releases, slot reuse, table growth) every to_cache equals the host table
    (-1 padded) and lengths, in the requested order."""
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    import flashspec_b200 as fs

    rng = np.random.default_rng(2)
    h, d = 2, 128
    alloc = fs.PagedKVAllocator(capacity_blocks=600, heads=h, head_dim=d, device="cuda")
    live, nxt = [], 0
    for step in range(60):
        for _ in range(int(rng.integers(0, 3))):
            n = int(rng.integers(1, 300))
            k = torch.randn(1, h, n, d, device="cuda", dtype=torch.float16)
            alloc.add_request(nxt, k, k)
            live.append(nxt)
            nxt += 1
        if live:
            t = 1 if step % 4 else int(rng.integers(2, 40))
            k = torch.randn(len(live), h, t, d, device="cuda", dtype=torch.float16)
            alloc.append_batch(live, k, k)
            order = list(rng.permutation(live))
            cache = alloc.to_cache(order)
            table, lens = alloc.block_table_numpy(order)
            np.testing.assert_array_equal(cache.block_table.cpu().numpy(), table)
            np.testing.assert_array_equal(cache.lengths.cpu().numpy(), lens)
            assert cache.max_seq_len == int(lens.max())
        for rid in [r for r in live if rng.random() < 0.2]:
            alloc.release_request(rid)
            live.remove(rid)


def test_run_decode_simulation_schema_and_sanity():
    """The reference's simulation API (src/flashspec/serving.py:33-190): same keys."""
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from flashspec_b200.serving import SimulationConfig, run_decode_simulation

    res = run_decode_simulation(SimulationConfig(requests=4, prompt_lens=(40, 130), prompt_length_distribution="bimodal",
                                                 decode_steps=12, request_life_steps=5, heads=4, head_dim=64))
    keys = {"device", "device_name", "dtype", "requests", "prompt_len", "prompt_lens", "prompt_length_distribution",
            "average_prompt_len", "decode_steps", "request_life_steps", "arrivals", "finishes", "prefill_ms",
            "arrival_prefill_ms", "total_prefill_ms", "first_attention_ms", "decode_ms", "ttft_ms", "tpot_ms",
            "tokens_per_second", "generated_tokens", "allocated_blocks", "free_blocks", "live_requests",
            "used_tokens", "capacity_tokens", "block_utilization", "capacity_utilization", "padding_waste",
            "fragmentation"}
    assert keys <= set(res)
    assert res["generated_tokens"] == 4 * 12 and res["finishes"] == 8 and res["arrivals"] == 12
    assert res["average_prompt_len"] == 85.0 and res["ttft_ms"] > 0 and res["tokens_per_second"] > 0
