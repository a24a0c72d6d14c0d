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
