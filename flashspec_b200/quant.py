"""INT8 cache format and the CUDA quantizer.

The format is the reference's (src/flashspec/quant.py:9-43): per block of
``block_size`` tokens x head_dim, an affine uint8 code stored as int8 (u - 128)
with an fp32 scale and an int16 zero point.  ``QuantizedTensor`` has the same
fields, so reference objects (or any object with these attributes) are accepted
by every entry point of this package.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from . import _lib

_DTYPES = {torch.float16: _lib.FS_F16, torch.bfloat16: _lib.FS_BF16, torch.float32: _lib.FS_F32}


@dataclass(frozen=True)
class QuantizedTensor:
    """Same fields and meaning as the reference QuantizedTensor (quant.py:9-43)."""

    values: torch.Tensor  # int8 [..., n_blocks, block_size, head_dim]
    scale: torch.Tensor  # fp32 [..., n_blocks, 1, 1]
    zero_point: torch.Tensor  # int16 [..., n_blocks, 1, 1]
    block_size: int
    original_shape: Tuple[int, ...]

    @property
    def device(self) -> torch.device:
        return self.values.device


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float16, bfloat16 or float32") from None


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise RuntimeError(f"{what} must be a CUDA tensor (flashspec_b200 has no CPU path)")


def quantize_int8_per_block(x: torch.Tensor, block_size: int = 16) -> QuantizedTensor:
    """CUDA version of quantize_int8_per_block (src/flashspec/quant.py:94-165),
    bit-exact: same zero padding of the sequence axis (quant.py:69-91), same fp32
    operation order and round-half-even."""
    require_cuda(x, "x")
    if x.ndim < 2:
        raise ValueError("input needs a sequence and a feature dimension")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    if x.shape[-1] <= 0 or x.shape[-2] <= 0:
        raise ValueError("sequence and feature dimensions must be non-empty")
    original_shape = tuple(int(s) for s in x.shape)
    xc = x.detach().contiguous()
    code = dtype_code(xc)
    lead = original_shape[:-2]
    seq, d = original_shape[-2], original_shape[-1]
    nblk = (seq + block_size - 1) // block_size
    n_lead = 1
    for s in lead:
        n_lead *= s
    values = torch.empty((*lead, nblk, block_size, d), dtype=torch.int8, device=x.device)
    scale = torch.empty((*lead, nblk, 1, 1), dtype=torch.float32, device=x.device)
    zp = torch.empty((*lead, nblk, 1, 1), dtype=torch.int16, device=x.device)
    if n_lead > 0:
        args = _lib.FsQuantizeArgs(xc.data_ptr(), code, n_lead, seq, d, block_size, values.data_ptr(),
                                   scale.data_ptr(), zp.data_ptr())
        with torch.cuda.device(x.device):
            _lib.check(_lib.load().fs_quantize_blocks(C.byref(args), stream_of(x.device)), "fs_quantize_blocks")
    return QuantizedTensor(values, scale, zp, block_size, original_shape)


def dequantize_int8_per_block(q, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Dense dequantization (src/flashspec/quant.py:168-204): (float(v+128) - zp) * scale,
    reshaped to ``original_shape``.  A utility for inspection; the attention
    kernels never materialise dense KV."""
    u = q.values.to(torch.int16) + 128
    x = (u.to(torch.float32) - q.zero_point.to(torch.float32)) * q.scale.to(torch.float32)
    lead = tuple(q.original_shape[:-2])
    seq, d = q.original_shape[-2], q.original_shape[-1]
    x = x.reshape(*lead, -1, d)[..., :seq, :]
    return x.to(dtype=dtype) if dtype is not None else x


def estimate_quantized_bytes(q) -> int:
    """quant.py:232-247: values + 4*scale + 2*zero_point elements (no zero points in the
    symmetric format)."""
    zp = getattr(q, "zero_point", None)
    return int(q.values.numel() + q.scale.numel() * 4 + (zp.numel() * 2 if zp is not None else 0))


@dataclass
class SymQuantizedTensor:
    """Symmetric per-token INT8 (FS_KV_SYMMETRIC): values int8 [..., S_pad, D] =
    clamp(rint(x / s), -127, 127) with s = max(absmax / 127, 1e-8) per token and head,
    scale fp32 [..., S_pad]; S_pad = the sequence padded with zero tokens to a multiple
    of block_size.  No zero points.  The reference has no such format (it lists
    symmetric INT8 as future work, doc/TODO.MD:241-255); the benchmark configurations'
    wording describes it."""

    values: torch.Tensor
    scale: torch.Tensor
    block_size: int
    original_shape: Tuple[int, ...]
    zero_point: Optional[torch.Tensor] = None
    symmetric: bool = True

    @property
    def device(self) -> torch.device:
        return self.values.device


def quantize_int8_symmetric_per_token(x: torch.Tensor, block_size: int = 16) -> SymQuantizedTensor:
    """x [..., S, D] (fp16 / bf16 / fp32, CUDA) -> SymQuantizedTensor; the sequence is
    zero-padded to a multiple of block_size (padded tokens get scale 1e-8, values 0)."""
    require_cuda(x, "x")
    if x.ndim < 2 or x.shape[-1] <= 0 or x.shape[-2] <= 0:
        raise ValueError("input needs non-empty sequence and feature dimensions")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    shape = tuple(int(s) for s in x.shape)
    seq, d = shape[-2], shape[-1]
    pad = (-seq) % block_size
    xc = x.detach()
    if pad:
        xc = torch.cat([xc, xc.new_zeros((*shape[:-2], pad, d))], dim=-2)
    xc = xc.contiguous()
    n_lead = 1
    for s_ in shape[:-2]:
        n_lead *= s_
    values = torch.empty(xc.shape, dtype=torch.int8, device=x.device)
    scale = torch.empty(xc.shape[:-1], dtype=torch.float32, device=x.device)
    args = _lib.FsQuantizeArgs(xc.data_ptr(), dtype_code(xc), n_lead, seq + pad, d, block_size, values.data_ptr(),
                               scale.data_ptr(), None)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().fs_quantize_symmetric(C.byref(args), stream_of(x.device)), "fs_quantize_symmetric")
    return SymQuantizedTensor(values, scale, block_size, shape)


def dequantize_int8_symmetric(q: SymQuantizedTensor, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """values * scale, back to original_shape."""
    x = q.values.to(torch.float32) * q.scale.to(torch.float32).unsqueeze(-1)
    lead, seq, d = tuple(q.original_shape[:-2]), q.original_shape[-2], q.original_shape[-1]
    x = x.reshape(*lead, -1, d)[..., :seq, :]
    return x.to(dtype) if dtype is not None else x


def build_compression_stats(dense_bytes: float, quant_bytes: float, *, materializes_dense_kv: bool,
                            **extra: float) -> Dict[str, float]:
    """quant.py:207-229: the stats dict every attention backend returns."""
    stats = {
        "dense_kv_bytes": float(dense_bytes),
        "quant_kv_bytes": float(quant_bytes),
        "compression_ratio": float(dense_bytes / max(1, quant_bytes)),
        "materializes_dense_kv": 1.0 if materializes_dense_kv else 0.0,
    }
    stats.update({k: float(v) for k, v in extra.items()})
    return stats
