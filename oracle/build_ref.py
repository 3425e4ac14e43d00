"""Compile the reference's own C++/CUDA sources into oracle/_ref/ (TEST INFRASTRUCTURE ONLY).

The sources are read where they lie in the reference checkout (csrc/ of Yu-TingLee/int4-GEMV-cuda);
nothing is copied into this repository. The reference's CMake build is not used: the seven files
are compiled directly with torch's extension builder, plus oracle/ref_binding.cpp (our own pybind
module, named int4gemv_ref so it can sit beside the product's int4gemv_ops). The kernels are built
for sm_100a so the reference's GPU kernels can run on the B200 as a second oracle and as the
kernel to beat.

Usage: python oracle/build_ref.py [--reference /path/to/reference]
Without --reference the checkout is taken from $INT4GEMV_REFERENCE, else from BASELINE.json's
"reference_path". The checkout only exists in the build container; the GPU box uses the built .so.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
REPO = HERE.parent


def reference_dir() -> Path | None:
    """The reference checkout: $INT4GEMV_REFERENCE, else BASELINE.json's reference_path."""
    env = os.environ.get("INT4GEMV_REFERENCE")
    if env:
        return Path(env)
    try:
        import json

        path = json.loads((REPO / "BASELINE.json").read_text()).get("reference_path")
    except (OSError, ValueError):
        path = None
    return Path(path) if path else None


SOURCES = ["checks.cpp", "sequential.cpp", "naive.cu", "coalesced.cu", "vectorized.cu",
           "load_only.cu"]


def built_module() -> Path | None:
    hits = sorted(OUT.glob("int4gemv_ref*.so"))
    return hits[0] if hits else None


def build(reference: Path | None = None, verbose: bool = False) -> Path | None:
    reference = reference or reference_dir()
    csrc = reference / "csrc" if reference else None
    if csrc is None or not (csrc / "w4a16.h").exists():
        print(f"build_ref: no reference sources at {csrc}; skipped", file=sys.stderr)
        return built_module()
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    from torch.utils import cpp_extension

    OUT.mkdir(exist_ok=True)
    cpp_extension.load(
        name="int4gemv_ref",
        sources=[str(HERE / "ref_binding.cpp")] + [str(csrc / s) for s in SOURCES],
        extra_include_paths=[str(csrc)],
        extra_cflags=["-O3", "-std=c++20"],
        extra_cuda_cflags=["-O3", "-std=c++20", "-gencode=arch=compute_100a,code=sm_100a"],
        build_directory=str(OUT),
        with_cuda=True,
        verbose=verbose,
    )
    return built_module()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.reference, args.verbose))
