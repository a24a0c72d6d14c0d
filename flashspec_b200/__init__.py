"""flashspec_b200: B200-native (sm_100a) INT8 decode attention for FlashSpec caches.

Public API mirrors the reference package (src/flashspec/__init__.py:3-24) for the
hot path: the cache objects (QuantizedTensor, PagedKVCache, PagedKVAllocator), the
quantizer, and two attention backends that replace the reference's Triton ones:

    fused_dequant_attention_cuda   <-> fused_dequant_attention_triton
    paged_quant_attention_cuda     <-> paged_quant_attention_triton

All compute runs in the in-tree native library ``libflashspec_b200.so`` (C ABI in
include/flashspec_b200.h).  There is no CPU or Triton fallback.
"""

from ._build import build
from .attention import (BACKENDS, fused_dequant_attention_cuda, get_backend, merge_partials,
                        paged_quant_attention_cuda, register_backend, reset_workspaces)
from .paged import PagedKVAllocator, PagedKVCache
from .paged import paged_cache_symmetric
from .quant import (QuantizedTensor, SymQuantizedTensor, build_compression_stats, dequantize_int8_per_block,
                    dequantize_int8_symmetric, estimate_quantized_bytes, quantize_int8_per_block,
                    quantize_int8_symmetric_per_token)
from .tree import tree_verify_attention_cuda

__all__ = [
    "BACKENDS",
    "PagedKVAllocator",
    "PagedKVCache",
    "QuantizedTensor",
    "build",
    "build_compression_stats",
    "dequantize_int8_per_block",
    "estimate_quantized_bytes",
    "fused_dequant_attention_cuda",
    "get_backend",
    "merge_partials",
    "paged_quant_attention_cuda",
    "quantize_int8_per_block",
    "register_backend",
    "SymQuantizedTensor",
    "dequantize_int8_symmetric",
    "paged_cache_symmetric",
    "quantize_int8_symmetric_per_token",
    "reset_workspaces",
    "tree_verify_attention_cuda",
]
