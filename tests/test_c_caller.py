"""The C ABI from plain C: include/int4gemv_b200.h compiles as C99 and as C++17, and a C program
(tests/c/c_abi_example.c) linked against libint4gemv_b200.so computes the CPU path bit for bit
like the reference's own sequential GEMV (the golden vectors)."""

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from int4gemv import capi

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
INCLUDE = REPO / "include"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
@pytest.mark.parametrize("compiler,flags", [("gcc", ["-x", "c", "-std=c99"]),
                                            ("g++", ["-x", "c++", "-std=c++17"])])
def test_header_compiles(compiler, flags, tmp_path):
    src = tmp_path / "h.c"
    src.write_text('#include "int4gemv_b200.h"\nint main(void) { return INT4GEMV_OK; }\n')
    subprocess.run([compiler, *flags, "-Wall", "-Werror", "-pedantic", f"-I{INCLUDE}",
                    "-fsyntax-only", str(src)], check=True)


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_program_runs_cpu_path(golden, tmp_path):
    lib = capi.LIB_PATH
    exe = tmp_path / "c_abi_example"
    subprocess.run(["gcc", "-std=c99", "-O1", f"-I{INCLUDE}", str(HERE / "c" / "c_abi_example.c"),
                    f"-L{lib.parent}", "-lint4gemv_b200", f"-Wl,-rpath,{lib.parent}", "-o",
                    str(exe)], check=True)
    g = int(golden["group_size"])
    x, q, s, z = (np.ascontiguousarray(golden[k]) for k in ("x", "qweight", "scales", "zeros"))
    m, k = x.shape
    n = q.shape[0]
    parts = [f"{m} {n} {k} {g}"]
    for arr in (x.view(np.uint16), q, s.view(np.uint16), z.view(np.uint16)):
        parts.append(" ".join(str(int(v)) for v in arr.ravel()))
    out = subprocess.run([str(exe)], input="\n".join(parts), capture_output=True, text=True,
                         check=True).stdout.split("\n")
    y = np.array([int(v) for v in out[:m * n]], np.uint16).reshape(m, n)
    np.testing.assert_array_equal(y, golden["y_seq"].view(np.uint16))
    assert out[m * n].startswith("version ")
