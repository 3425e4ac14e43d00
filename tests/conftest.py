"""Shared test setup: import paths, the `gpu` marker, golden fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "int4-gemv-cuda_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(PKG), str(REPO / "oracle"), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def golden_names() -> list[str]:
    """The GEMV / quantize cases (pack_wrap.npz holds only pack vectors)."""
    return sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith("pack_"))


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(params=golden_names())
def golden(request):
    case = load_golden(request.param)
    case["name"] = request.param
    return case


@pytest.fixture
def pack_wrap():
    """int32 q [6, 128] with values inside and outside 0..15, and the reference's pack of it."""
    return load_golden("pack_wrap")
