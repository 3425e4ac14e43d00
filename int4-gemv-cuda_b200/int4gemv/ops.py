"""The compiled operators, loaded from the in-tree build (int4-gemv-cuda_b200/_build).

Drop-in for the reference's int4gemv.ops (int4gemv/ops.py:11-36 of Yu-TingLee/int4-GEMV-cuda):
the same names (sequential, naive, coalesced, vectorized, load_only), the same KERNELS and
KERNEL_INFO tables, plus the B200 fast path `w4a16`, the fused epilogues `w4a16_silu_mul` and
`w4a16_bias_residual`, the unrounded fp32 row sums `w4a16_f32` (K-split partial sums), and the
bit-exact device `quantize` / `pack` / `unpack` / `dequantize`. As
in the reference, INT4GEMV_BUILD_DIR may point at another build directory (its `python/`
subdirectory or the directory itself is searched).

There is no fallback: if the compiled module is missing this import fails and says how to build.
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import torch  # noqa: F401  loads libtorch before int4gemv_ops, which links against it

PKG_ROOT = Path(__file__).resolve().parents[1]
DEFAULT_BUILD_DIR = PKG_ROOT / "_build"


def _find_module() -> Path:
    dirs = []
    env = os.environ.get("INT4GEMV_BUILD_DIR")
    if env:
        d = Path(env)
        if not d.is_absolute():
            d = PKG_ROOT.parent / d
        dirs += [d / "python", d]
    dirs.append(DEFAULT_BUILD_DIR)
    for d in dirs:
        hits = sorted(d.glob("int4gemv_ops*.so")) if d.is_dir() else []
        if hits:
            return hits[0]
    raise ImportError(
        "int4gemv_ops is not built (looked in " + ", ".join(map(str, dirs)) + "). "
        "Run: python int4-gemv-cuda_b200/build.py"
    )


def _load():
    if "int4gemv_ops" in sys.modules:
        return sys.modules["int4gemv_ops"]
    path = _find_module()
    spec = importlib.util.spec_from_file_location("int4gemv_ops", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    sys.modules["int4gemv_ops"] = module
    return module


int4gemv_ops = _load()
LIBRARY_PATH = Path(int4gemv_ops.__file__)

sequential = int4gemv_ops.sequential
naive = int4gemv_ops.naive
coalesced = int4gemv_ops.coalesced
vectorized = int4gemv_ops.vectorized
load_only = int4gemv_ops.load_only
w4a16 = int4gemv_ops.w4a16
w4a16_kernel = int4gemv_ops.w4a16_kernel
w4a16_with = int4gemv_ops.w4a16_with
w4a16_silu_mul = int4gemv_ops.w4a16_silu_mul
w4a16_bias_residual = int4gemv_ops.w4a16_bias_residual
w4a16_f32 = int4gemv_ops.w4a16_f32
w4a16_grouped = int4gemv_ops.w4a16_grouped
unpack = int4gemv_ops.unpack
dequantize = int4gemv_ops.dequantize
quantize = int4gemv_ops.quantize
pack = int4gemv_ops.pack
repack_awq = int4gemv_ops.repack_awq
repack_gptq = int4gemv_ops.repack_gptq
check_inputs = int4gemv_ops.check_inputs

# The GEMV kernels, slowest first. All share the 5-argument signature of csrc/w4a16.h.
KERNELS = {
    "naive": naive,
    "coalesced": coalesced,
    "vectorized": vectorized,
    "w4a16": w4a16,
}

# info(m, **block_config) -> registers, spills and occupancy.
KERNEL_INFO = {
    "naive": int4gemv_ops.naive_info,
    "coalesced": int4gemv_ops.coalesced_info,
    "vectorized": int4gemv_ops.vectorized_info,
    "w4a16": int4gemv_ops.w4a16_info,
}
