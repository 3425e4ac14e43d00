"""Build the library in-tree (no GPU needed; nvcc cross-compiles for sm_100a).

Two products, both under int4-gemv-cuda_b200/_build/:
  libint4gemv_b200.so   the CUDA kernels and the C ABI of include/int4gemv_b200.h (no torch;
                        cudart linked statically)
  int4gemv_ops<ext>.so  the torch / pybind module with the reference's operator API, a thin
                        layer over the C ABI (loads libint4gemv_b200.so through its rpath)

Usage: python int4-gemv-cuda_b200/build.py [--force] [--verbose]
Rebuilds only what is older than its sources.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
OUT = PKG / "_build"
LIB = OUT / "libint4gemv_b200.so"
EXT_NAME = "int4gemv_ops"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++20", "-Xcompiler", "-fPIC",
                     f"-I{INCLUDE}", f"-I{CSRC}"]
CU_SOURCES = [
    "capi.cu", "simt.cu", "mma_pipeline.cu", "tc_gemv.cu", "stream_mma.cu", "stripe_mma.cu",
    "tc_dequant.cu", "tc_wide.cu",
    "weight_stream.cu",
    "packed.cu", "quantize.cu", "repack.cu",
]
# The CPU path must keep one IEEE rounding per operation: no contraction, no fast-math.
CPU_SOURCES = {"sequential.cpp": ["-O3", "-ffp-contract=off", "-fno-fast-math"]}
TORCH_SOURCES = ["bindings.cpp", "checks.cpp"]
HEADERS = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [INCLUDE / "int4gemv_b200.h"]


def ext_path() -> Path:
    return OUT / (EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths(device_type="cuda")
    inc += [sysconfig.get_paths()["include"], str(CUDA_HOME / "include"), str(INCLUDE), str(CSRC)]
    cflags = [f"-I{p}" for p in inc] + [
        "-O3", "-std=c++20", "-fPIC", "-Wno-unused-parameter",
        f"-DTORCH_EXTENSION_NAME={EXT_NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
    ]
    for attr, macro in (("_PYBIND11_COMPILER_TYPE", "PYBIND11_COMPILER_TYPE"),
                        ("_PYBIND11_STDLIB", "PYBIND11_STDLIB"),
                        ("_PYBIND11_BUILD_ABI", "PYBIND11_BUILD_ABI")):
        val = getattr(torch._C, attr, None)
        if val is not None:
            cflags.append(f'-D{macro}="{val}"')
    libdirs = cpp_extension.library_paths(device_type="cuda")
    ldflags = [f"-L{p}" for p in libdirs] + [f"-Wl,-rpath,{p}" for p in libdirs]
    ldflags += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    return cflags, ldflags


def build(force: bool = False, verbose: bool = False) -> Path:
    OUT.mkdir(exist_ok=True)
    jobs = []  # (target, deps, cmd)
    objs = []
    for src in CU_SOURCES:
        obj = OUT / (src + ".o")
        objs.append(obj)
        jobs.append((obj, [CSRC / src] + HEADERS,
                     [NVCC] + NVCC_FLAGS + ["-c", str(CSRC / src), "-o", str(obj)]))
    for src, flags in CPU_SOURCES.items():
        obj = OUT / (src + ".o")
        objs.append(obj)
        jobs.append((obj, [CSRC / src], ["g++", "-std=c++20", "-fPIC"] + flags +
                     ["-c", str(CSRC / src), "-o", str(obj)]))
    torch_objs = []
    torch_cflags = None
    for src in TORCH_SOURCES:
        obj = OUT / (src + ".torch.o")
        torch_objs.append(obj)
        if force or _stale(obj, [CSRC / src] + HEADERS):
            if torch_cflags is None:
                torch_cflags, torch_ldflags = _torch_flags()
            jobs.append((obj, [CSRC / src] + HEADERS,
                         ["g++"] + torch_cflags + ["-c", str(CSRC / src), "-o", str(obj)]))

    todo = [(t, cmd) for t, deps, cmd in jobs if force or _stale(t, deps)]
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        list(pool.map(lambda tc: _run(tc[1], verbose), todo))

    if force or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs] +
             ["-Xlinker", "-soname=libint4gemv_b200.so", "-lpthread"], verbose)
    ext = ext_path()
    if force or _stale(ext, torch_objs + [LIB]):
        if torch_cflags is None:
            torch_cflags, torch_ldflags = _torch_flags()
        _run(["g++", "-shared", "-o", str(ext)] + [str(o) for o in torch_objs] +
             [f"-L{OUT}", "-lint4gemv_b200", "-Wl,-rpath,$ORIGIN"] + torch_ldflags, verbose)
    return ext


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", "-v", action="store_true")
    args = ap.parse_args()
    print(build(args.force, args.verbose))
