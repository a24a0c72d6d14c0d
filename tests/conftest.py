"""Shared pytest fixtures: the ``gpu`` marker, golden-fixture loading, repo paths."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


class Golden(dict):
    """npz contents with ``.quant(prefix)`` rebuilding an oracle OQuant."""

    def quant(self, prefix):
        import flashspec_oracle as O

        return O.OQuant(self[f"{prefix}.values"], self[f"{prefix}.scale"], self[f"{prefix}.zero_point"],
                        int(self[f"{prefix}.block_size"]), tuple(int(x) for x in self[f"{prefix}.original_shape"]))


def load_golden(name: str) -> Golden:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return Golden({k: z[k] for k in z.files})


@pytest.fixture
def golden():
    return load_golden
