"""CPU checks of the C-ABI boundary: the native library loads without a GPU,
exports every function include/flashspec_b200.h declares, and the ctypes
structures match the C layout (compiled with gcc from the header)."""

from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "flashspec_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(fs_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from flashspec_b200 import _lib

    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert lib.fs_abi_version() == _lib.ABI_VERSION
    assert lib.fs_status_string(0) == b"ok"


def test_calls_without_gpu_fail_cleanly():
    from flashspec_b200 import _lib

    lib = _lib.load()
    assert lib.fs_page_update(None, None) == 1  # invalid argument, no CUDA call
    assert lib.fs_merge_partials(None, None, 1, 1, 1, 0, None, 0, None) == 1
    a = _lib.FsDecodeArgs()
    assert lib.fs_paged_decode(C.byref(a), None) == 1


def test_ctypes_layouts_match_c(tmp_path):
    from flashspec_b200 import _lib

    structs = {"FsDecodeArgs": _lib.FsDecodeArgs, "FsQuantizeArgs": _lib.FsQuantizeArgs,
               "FsPageUpdate": _lib.FsPageUpdate, "FsPageUpdateArgs": _lib.FsPageUpdateArgs,
               "FsExchangeArgs": _lib.FsExchangeArgs, "FsTreeArgs": _lib.FsTreeArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for name, cls in structs.items():
        lines.append(f'printf("{name} %zu\\n", sizeof({name}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{name}.{fname} %zu\\n", offsetof({name}, {fname}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", str(src), "-o", str(exe)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines())
    for name, cls in structs.items():
        assert int(got[name]) == C.sizeof(cls), name
        for fname, _ in cls._fields_:
            assert int(got[f"{name}.{fname}"]) == getattr(cls, fname).offset, f"{name}.{fname}"


def test_cuda_entry_points_refuse_cpu_tensors():
    import torch

    import flashspec_b200 as f

    with pytest.raises(RuntimeError):
        f.quantize_int8_per_block(torch.zeros(2, 16, 8))


def test_cuda_failure_reports_the_failing_call():
    """A valid decode description queried without a usable GPU fails with FS_ERR_CUDA,
    and fs_last_error_detail names the CUDA call and its error; with a GPU the query
    succeeds and the detail is not consulted."""
    from flashspec_b200 import _lib

    lib = _lib.load()
    a = _lib.FsDecodeArgs()
    a.layout = _lib.FS_LAYOUT_PAGED
    a.q = a.k_values = a.v_values = a.k_scale = a.v_scale = a.k_zero = a.v_zero = 4096
    a.block_table = a.lengths = a.out = 4096
    a.batch, a.q_heads, a.kv_heads, a.head_dim, a.block_size = 2, 8, 8, 128, 16
    a.num_blocks, a.table_cols, a.max_seq_len = 64, 4, 64
    a.sm_scale = 128 ** -0.5
    n, s = C.c_size_t(0), C.c_int32(0)
    st = lib.fs_decode_workspace_size(C.byref(a), C.byref(n), C.byref(s))
    if st == 0:
        pytest.skip("a GPU is usable here: no CUDA failure to report")
    assert st == 3  # FS_ERR_CUDA
    detail = lib.fs_last_error_detail().decode()
    assert "cuda" in detail.lower() and ":" in detail, detail
