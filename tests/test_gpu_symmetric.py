"""GPU parity of the symmetric per-token INT8 format (FS_KV_SYMMETRIC): the quantizer
bit-exact against the oracle's restatement of the format, and paged / contiguous decode
against the oracle's attention over the dequantized cache at
|got - ref| <= 2e-3 + 1e-2 |ref|."""

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


def close(got, ref):
    ref_t = torch.as_tensor(np.asarray(ref, dtype=np.float32))
    err = (got.detach().float().cpu() - ref_t).abs()
    bad = err > ATOL + RTOL * ref_t.abs()
    assert not bool(bad.any()), f"{int(bad.sum())} out of tolerance, max abs err {err.max().item():.3e}"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_symmetric_quantizer_bit_exact(dtype):
    g = torch.Generator(device="cuda").manual_seed(1)
    x = (torch.randn(3, 4, 37, 128, generator=g, device="cuda") * 3).to(dtype)
    x[0, 0, 5] = 0  # an all-zero token: scale floor 1e-8, values 0
    qt = fs().quantize_int8_symmetric_per_token(x, 16)
    vals, sc = O.quantize_symmetric(x.float().cpu().numpy())
    assert tuple(qt.values.shape) == (3, 4, 48, 128)
    np.testing.assert_array_equal(qt.values[..., :37, :].cpu().numpy(), vals)
    np.testing.assert_array_equal(qt.scale[..., :37].cpu().numpy().view(np.uint32), sc.view(np.uint32))
    assert bool((qt.values[..., 37:, :] == 0).all())


@pytest.mark.parametrize("hq,hkv,d,page", [(32, 32, 128, 16), (8, 2, 128, 32), (4, 4, 64, 16)])
def test_symmetric_paged_decode_vs_oracle(hq, hkv, d, page):
    g = torch.Generator(device="cuda").manual_seed(hq + d + page)
    b, s = 4, 700
    k = torch.randn(b, hkv, s, d, generator=g, device="cuda", dtype=torch.float16)
    v = torch.randn(b, hkv, s, d, generator=g, device="cuda", dtype=torch.float16)
    q = torch.randn(b, hq, d, generator=g, device="cuda", dtype=torch.float16)
    bps = (s + page - 1) // page
    perm = torch.randperm(b * bps, generator=torch.Generator().manual_seed(3))
    lengths = torch.tensor([700, 1, 333, 16], dtype=torch.int64, device="cuda")
    cache = fs().paged_cache_symmetric(k, v, page, lengths=lengths, perm=perm)
    out, stats = fs().paged_quant_attention_cuda(q, cache, return_stats=True)
    kq, vq = cache.k_quant, cache.v_quant
    ref = O.symmetric_paged_attention(q.cpu().numpy(), kq.values.cpu().numpy(), kq.scale.cpu().numpy(),
                                      vq.values.cpu().numpy(), vq.scale.cpu().numpy(), cache.block_table.cpu().numpy(),
                                      lengths.cpu().numpy(), s)
    close(out, ref)
    assert stats["quant_kv_bytes"] > 0


def test_symmetric_fused_decode_vs_oracle():
    g = torch.Generator(device="cuda").manual_seed(9)
    b, h, s, d = 3, 8, 300, 128
    k = torch.randn(b, h, s, d, generator=g, device="cuda", dtype=torch.float16)
    v = torch.randn(b, h, s, d, generator=g, device="cuda", dtype=torch.float16)
    q = torch.randn(b, h, d, generator=g, device="cuda", dtype=torch.float16)
    kq = fs().quantize_int8_symmetric_per_token(k, 16)
    vq = fs().quantize_int8_symmetric_per_token(v, 16)
    lengths = torch.tensor([300, 299, 17], dtype=torch.int64, device="cuda")
    out = fs().fused_dequant_attention_cuda(q, kq, vq, lengths)
    kd = fs().dequantize_int8_symmetric(kq).cpu().numpy()
    vd = fs().dequantize_int8_symmetric(vq).cpu().numpy()
    close(out, O.reference_attention(q.cpu().numpy(), kd, vd, lengths.cpu().numpy()))
