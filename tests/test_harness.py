"""Harness checks on CPU: microbench JSON schema (dense backend), ncu CSV parsing /
back-fill (synthetic fixture), profile-matrix manifest (dry run).  Mirrors the
reference's schema and NcuBackfill tests (tests/test_flashspec.py:263-324, 397-425)."""

from __future__ import annotations

import csv
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_microbench_json_schema_on_cpu():
    env = {k: v for k, v in os.environ.items() if not k.startswith("FLASHSPEC_")}
    proc = subprocess.run([sys.executable, "-m", "flashspec_b200.harness.microbench", "--backend", "dense",
                           "--batch", "1", "--heads", "1", "--seq-len", "4", "--head-dim", "8", "--iters", "1",
                           "--warmup", "0", "--repeats", "1", "--device", "cpu", "--dtype", "float32", "--json"],
                          check=True, capture_output=True, text=True, env=env, cwd=ROOT)
    data = json.loads(proc.stdout)
    for key in ("backend", "seq_len", "head_dim", "block_size", "num_splits", "block_n", "env_flashspec_num_splits",
                "env_flashspec_block_n", "env_flashspec_num_warps", "num_warps", "length_pattern",
                "passes_lengths_to_attention", "effective_lengths", "effective_min_seq_len", "effective_max_seq_len",
                "paged_layout", "paged_layout_seed", "bandwidth_fields_are_estimates",
                "measured_registers_per_thread", "measured_theoretical_occupancy_pct", "nsight_compute_source_command",
                "nsight_compute_commands", "materializes_dense_kv", "algorithmic_bytes", "achieved_algorithmic_gbps",
                "frac_of_nominal_8tbs"):
        assert key in data, key
    assert data["num_splits"] is None and data["env_flashspec_num_splits"] is None
    assert data["effective_lengths"] == [4] and data["paged_layout"] == "contiguous"
    assert data["passes_lengths_to_attention"] is False
    assert "--clock-control none" in data["nsight_compute_command"]


_CSV = (
    "==PROF== banner line to skip\n"
    '"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size",'
    '"Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"\n'
    '"0","1","python","h","void fsb::decode_kernel<1, 4, 16, 3, 0>(...)","1","7","(160,1,1)","(2048,1,1)","0","10.0",'
    '"Command line profiler metrics","dram__bytes_read.sum","Mbyte","538.70"\n'
    '"0","1","python","h","void fsb::decode_kernel<1, 4, 16, 3, 0>(...)","1","7","(160,1,1)","(2048,1,1)","0","10.0",'
    '"Command line profiler metrics","dram__bytes_write.sum","Mbyte","3.75"\n'
    '"0","1","python","h","void fsb::decode_kernel<1, 4, 16, 3, 0>(...)","1","7","(160,1,1)","(2048,1,1)","0","10.0",'
    '"Command line profiler metrics","gpu__time_duration.sum","usecond","105.76"\n'
    '"0","1","python","h","void fsb::decode_kernel<1, 4, 16, 3, 0>(...)","1","7","(160,1,1)","(2048,1,1)","0","10.0",'
    '"Command line profiler metrics","launch__registers_per_thread","register/thread","127"\n'
)


def test_ncu_backfill_writes_measured_fields():
    from flashspec_b200.harness.ncu_parse import apply_backfill, parse_ncu_csv

    parsed = parse_ncu_csv(_CSV)
    assert len(parsed) == 1
    result = {"bandwidth_fields_are_estimates": True}
    bad = apply_backfill(result, parsed)
    assert bad == []
    assert result["bandwidth_fields_are_estimates"] is False
    assert abs(result["measured_dram_bytes"] - 542.45e6) < 1
    assert abs(result["measured_ncu_kernel_duration_ms"] - 0.10576) < 1e-9
    assert abs(result["measured_achieved_bandwidth_gbps"] - 542.45e6 / 105760.0) < 1e-6
    assert result["measured_registers_per_thread"] == 127
    assert result["measured_ncu_kernel_count"] == 1
    assert "profiler_warning" not in result


def test_ncu_backfill_flags_foreign_kernels():
    from flashspec_b200.harness.ncu_parse import apply_backfill, parse_ncu_csv

    text = _CSV.replace("void fsb::decode_kernel<1, 4, 16, 3, 0>(...)", "vectorized_elementwise_kernel")
    result = {}
    assert apply_backfill(result, parse_ncu_csv(text))
    assert "profiler_warning" in result


def test_profile_matrix_dry_run(tmp_path):
    from flashspec_b200.harness import profile_matrix

    out = tmp_path / "m.csv"
    rows = profile_matrix.main(["--dry-run", "--seq-lens", "2048,4096", "--num-splits", "0,4", "--out", str(out)])
    assert len(rows) == 4
    with out.open() as f:
        got = list(csv.DictReader(f))
    assert [r["seq_len"] for r in got] == ["2048", "2048", "4096", "4096"]
    assert all(r["error"].startswith("dry-run") for r in got)


def test_split_timeline_phases_reads_the_trace_layout():
    """The timeline reader maps the kernel's stamp layout (4 words per CTA, 16 per pair)."""
    import numpy as np

    from flashspec_b200.harness.split_timeline import _phases

    ctas, pairs, t0 = 6, 2, 1_000_000
    buf = np.zeros(4 * ctas + 16 * pairs, dtype=np.int64)
    for c in range(ctas):
        buf[4 * c: 4 * c + 3] = [t0 + 100 * c, t0 + 10_000 + 100 * c, t0 + 12_000]
    for q in range(pairs):
        base = 4 * ctas + 16 * q
        start = t0 + 13_000 + 500 * q
        buf[base] = start
        buf[base + 4] = start + 5_000
        buf[base + 5] = start + 1_000
    out = _phases(buf, ctas, pairs, t0)
    assert out["cta_entry_first_last"] == [0.0, 0.5]
    assert out["stream_done_first_median_last"][0] == 10.0
    assert out["end_last"] == 18.5
    assert out["last_pair_merge_from_its_start"]["lse_loaded"] == 1.0
    assert out["last_pair_merge_from_its_start"]["end"] == 5.0
    assert out["last_pair_merge_from_its_start"]["round1_arrived"] is None
