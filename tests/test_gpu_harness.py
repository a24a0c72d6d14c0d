"""The microbench / profile-matrix harness on the GPU: real runs of the library's
backends produce the reference's JSON schema with roofline fields that agree with the
byte formula, and a sweep writes one manifest row per point with the kernel knob
applied (src/flashspec benchmarks/microbench.py:542-615, scripts/profile_matrix.py:62-224)."""

from __future__ import annotations

import csv
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")


def _env():
    return {k: v for k, v in os.environ.items() if not k.startswith("FLASHSPEC_")}


@pytest.mark.parametrize("backend", ["cuda_paged", "cuda_fused"])
def test_microbench_runs_the_library(backend):
    proc = subprocess.run([sys.executable, "-m", "flashspec_b200.harness.microbench", "--backend", backend,
                           "--batch", "4", "--heads", "8", "--seq-len", "1000", "--paged-layout", "shuffled",
                           "--length-pattern", "descending", "--iters", "5", "--warmup", "2", "--repeats", "3",
                           "--json"], check=True, capture_output=True, text=True, env=_env(), cwd=ROOT, timeout=300)
    data = json.loads(proc.stdout.strip().splitlines()[-1])
    assert data["backend"] == backend and data["latency_ms"] > 0
    assert data["materializes_dense_kv"] == 0.0
    lens = data["effective_lengths"]
    pages = sum((n + 15) // 16 for n in lens)
    assert data["algorithmic_bytes"] >= pages * 8 * 2 * (2048 + 6)
    gbs = data["algorithmic_bytes"] / (data["latency_ms"] * 1e-3) / 1e9
    assert abs(data["achieved_algorithmic_gbps"] - gbs) <= 0.01 * gbs


def test_profile_matrix_sweep_writes_rows(tmp_path):
    out = tmp_path / "sweep.csv"
    subprocess.run([sys.executable, "-m", "flashspec_b200.harness.profile_matrix", "--backend", "cuda_paged",
                    "--batches", "4", "--heads", "8", "--seq-lens", "512,1024", "--num-splits", "0,3",
                    "--iters", "3", "--repeats", "2", "--out", str(out)], check=True, env=_env(), cwd=ROOT,
                   timeout=600, capture_output=True)
    rows = list(csv.DictReader(out.open()))
    assert len(rows) == 4
    for r in rows:
        assert r["returncode"] == "0" and float(r["latency_ms"]) > 0, r
    forced = [r for r in rows if r["num_splits_env"] == "3"]
    assert all(float(r["num_splits"]) == 3 for r in forced)
