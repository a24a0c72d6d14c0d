"""ctypes binding of the C ABI declared in ``include/flashspec_b200.h``.

The shared library is loaded once.  If it is missing this module raises: the
package has no fallback implementation of any kernel.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libflashspec_b200.so"

FS_OK = 0
FS_ERR_CUDA = 3
FS_F16, FS_BF16, FS_F32 = 0, 1, 2
FS_LAYOUT_CONTIGUOUS, FS_LAYOUT_PAGED = 0, 1
FS_DEV_BAD_PAGE, FS_DEV_TIMEOUT = 1, 2
ABI_VERSION = 3
FS_KV_AFFINE_BLOCK, FS_KV_SYMMETRIC = 0, 1

_STATUS_EXC = {1: ValueError, 2: ValueError, 3: RuntimeError, 4: RuntimeError, 5: ValueError, 6: ValueError}


class FsDecodeArgs(C.Structure):
    _fields_ = [
        ("layout", C.c_int32),
        ("q", C.c_void_p),
        ("k_values", C.c_void_p),
        ("k_scale", C.c_void_p),
        ("k_zero", C.c_void_p),
        ("v_values", C.c_void_p),
        ("v_scale", C.c_void_p),
        ("v_zero", C.c_void_p),
        ("block_table", C.c_void_p),
        ("lengths", C.c_void_p),
        ("out", C.c_void_p),
        ("batch", C.c_int32),
        ("q_heads", C.c_int32),
        ("kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("block_size", C.c_int32),
        ("num_blocks", C.c_int64),
        ("table_cols", C.c_int32),
        ("max_seq_len", C.c_int32),
        ("num_splits", C.c_int32),
        ("sm_scale", C.c_float),
        ("page_begin", C.c_int64),
        ("page_end", C.c_int64),
        ("shard_o", C.c_void_p),
        ("shard_lse", C.c_void_p),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
        ("tickets", C.c_void_p),
        ("ticket_count", C.c_int64),
        ("device_status", C.c_void_p),
        ("q_dtype", C.c_int32),
        ("page_size", C.c_int32),
        ("kv_format", C.c_int32),
    ]


class FsQuantizeArgs(C.Structure):
    _fields_ = [
        ("x", C.c_void_p),
        ("x_dtype", C.c_int32),
        ("n_lead", C.c_int64),
        ("seq_len", C.c_int32),
        ("head_dim", C.c_int32),
        ("block_size", C.c_int32),
        ("values", C.c_void_p),
        ("scale", C.c_void_p),
        ("zero_point", C.c_void_p),
    ]


class FsPageUpdate(C.Structure):
    _fields_ = [
        ("page", C.c_int64),
        ("src_b", C.c_int32),
        ("src_t", C.c_int32),
        ("dst_row", C.c_int32),
        ("n_rows", C.c_int32),
        ("from_zero", C.c_int32),
        ("reserved", C.c_int32),
    ]


class FsPageUpdateArgs(C.Structure):
    _fields_ = [
        ("items", C.c_void_p),
        ("n_items", C.c_int32),
        ("k_src", C.c_void_p),
        ("v_src", C.c_void_p),
        ("src_dtype", C.c_int32),
        ("src_stride_b", C.c_int64),
        ("src_stride_h", C.c_int64),
        ("src_stride_t", C.c_int64),
        ("heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("block_size", C.c_int32),
        ("num_pages", C.c_int64),
        ("k_values_in", C.c_void_p),
        ("k_scale_in", C.c_void_p),
        ("k_zero_in", C.c_void_p),
        ("v_values_in", C.c_void_p),
        ("v_scale_in", C.c_void_p),
        ("v_zero_in", C.c_void_p),
        ("k_values_out", C.c_void_p),
        ("k_scale_out", C.c_void_p),
        ("k_zero_out", C.c_void_p),
        ("v_values_out", C.c_void_p),
        ("v_scale_out", C.c_void_p),
        ("v_zero_out", C.c_void_p),
    ]


EXCHANGE_MAX_RANKS = 8
EXCHANGE_HANDLE_BYTES = 64


class FsExchangeArgs(C.Structure):
    _fields_ = [
        ("world", C.c_int32),
        ("rank", C.c_int32),
        ("bufs", C.c_void_p * EXCHANGE_MAX_RANKS),
        ("slot_floats", C.c_int64),
        ("o_mine", C.c_void_p),
        ("lse_mine", C.c_void_p),
        ("rows", C.c_int64),
        ("head_dim", C.c_int32),
        ("out", C.c_void_p),
        ("out_dtype", C.c_int32),
        ("timeout_ns", C.c_int64),
        ("device_status", C.c_void_p),
    ]


class FsTreeArgs(C.Structure):
    _fields_ = [
        ("q", C.c_void_p),
        ("tree_k", C.c_void_p),
        ("tree_v", C.c_void_p),
        ("parents", C.c_void_p),
        ("prefix_o", C.c_void_p),
        ("prefix_lse", C.c_void_p),
        ("out", C.c_void_p),
        ("batch", C.c_int32),
        ("nodes", C.c_int32),
        ("q_heads", C.c_int32),
        ("kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("q_dtype", C.c_int32),
        ("sm_scale", C.c_float),
    ]


# every symbol the header declares, with its signature
SIGNATURES = {
    "fs_abi_version": (C.c_int, []),
    "fs_status_string": (C.c_char_p, [C.c_int]),
    "fs_last_error_detail": (C.c_char_p, []),
    "fs_decode_workspace_size": (C.c_int, [C.POINTER(FsDecodeArgs), C.POINTER(C.c_size_t), C.POINTER(C.c_int32)]),
    "fs_fused_decode": (C.c_int, [C.POINTER(FsDecodeArgs), C.c_void_p]),
    "fs_paged_decode": (C.c_int, [C.POINTER(FsDecodeArgs), C.c_void_p]),
    "fs_paged_decode_noalloc": (C.c_int, [C.POINTER(FsDecodeArgs), C.c_void_p]),
    "fs_merge_partials": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int64, C.c_int32, C.c_int64, C.c_void_p,
                                    C.c_int32, C.c_void_p]),
    "fs_quantize_blocks": (C.c_int, [C.POINTER(FsQuantizeArgs), C.c_void_p]),
    "fs_quantize_symmetric": (C.c_int, [C.POINTER(FsQuantizeArgs), C.c_void_p]),
    "fs_exchange_create": (C.c_int, [C.c_int64, C.POINTER(C.c_void_p), C.c_void_p]),
    "fs_exchange_open": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "fs_exchange_close": (C.c_int, [C.c_void_p]),
    "fs_exchange_destroy": (C.c_int, [C.c_void_p]),
    "fs_exchange_merge": (C.c_int, [C.POINTER(FsExchangeArgs), C.c_void_p]),
    "fs_paged_decode_exchange_workspace_size": (C.c_int, [C.POINTER(FsDecodeArgs), C.POINTER(C.c_size_t),
                                                          C.POINTER(C.c_int32)]),
    "fs_paged_decode_exchange": (C.c_int, [C.POINTER(FsDecodeArgs), C.POINTER(FsExchangeArgs), C.c_void_p]),
    "fs_page_update": (C.c_int, [C.POINTER(FsPageUpdateArgs), C.c_void_p]),
    "fs_tree_attend": (C.c_int, [C.POINTER(FsTreeArgs), C.c_void_p]),
    "fs_read_bandwidth_probe": (C.c_int, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_int32, C.POINTER(C.c_int32),
                                          C.c_void_p]),
    "fs_dequantize_pages": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                      C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
}

_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def load() -> C.CDLL:
    """Load the native library (once) and bind every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise RuntimeError(
            f"flashspec_b200 native library missing at {_LIB_PATH}; build it with "
            "`python -m flashspec_b200._build` (there is no non-CUDA fallback)")
    lib = C.CDLL(os.fspath(_LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.fs_abi_version() != ABI_VERSION:
        raise RuntimeError("flashspec_b200 native library ABI mismatch; rebuild it")
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != FS_OK:
        msg = load().fs_status_string(status).decode()
        if status == FS_ERR_CUDA:
            msg += f" [{load().fs_last_error_detail().decode()}]"
        raise _STATUS_EXC.get(status, RuntimeError)(f"{what} failed: {msg} (status {status})")
