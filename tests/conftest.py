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


def golden_names(prefix: str | None = None) -> list[str]:
    """prefix None: the GEMV / quantize cases; else the files named prefix* (pack_wrap.npz holds
    only pack vectors, checkpoint_*.npz AWQ / GPTQ tensors)."""
    names = sorted(p.stem for p in GOLDEN.glob("*.npz"))
    if prefix is None:
        return [n for n in names if not n.startswith(("pack_", "checkpoint_"))]
    return [n for n in names if n.startswith(prefix)]


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


@pytest.fixture(params=golden_names("checkpoint_"))
def checkpoint(request):
    """The reference's packed weights and the same weights as AWQ / GPTQ checkpoint tensors."""
    case = load_golden(request.param)
    case["name"] = request.param
    return case
