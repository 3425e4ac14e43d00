"""ctypes front end of the C ABI in include/int4gemv_b200.h (libint4gemv_b200.so).

This is the binding a non-torch caller writes; the tests and the end-to-end leg of bench.py use it
to call the library exactly as such a caller would: plain pointers, sizes and a stream handle.
Errors raise CapiError with the library's message.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]
LIB_PATH = PKG_ROOT / "_build" / "libint4gemv_b200.so"
HEADER_PATH = PKG_ROOT.parent / "include" / "int4gemv_b200.h"

OK, ERR_INVALID, ERR_CUDA, ERR_WORKSPACE = 0, 1, 2, 3

_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_PROTOTYPES = {
    "int4gemv_last_error": (ctypes.c_char_p, []),
    "int4gemv_version": (ctypes.c_int, []),
    "int4gemv_naive": (ctypes.c_int, [_p] * 5 + [_i64] * 4 + [_p]),
    "int4gemv_coalesced": (ctypes.c_int, [_p] * 5 + [_i64] * 4 + [_p]),
    "int4gemv_vectorized": (ctypes.c_int, [_p] * 5 + [_i64] * 6 + [_p]),
    "int4gemv_load_only": (ctypes.c_int, [_p] * 5 + [_i64] * 6 + [_p]),
    "int4gemv_stripe_load_only": (ctypes.c_int, [_p] * 4 + [_i64] * 3 + [_p]),
    "int4gemv_kernel_info": (ctypes.c_int, [ctypes.c_char_p, _i64, _i64, _i64,
                                            ctypes.POINTER(ctypes.c_int64)]),
    "int4gemv_sequential": (ctypes.c_int, [_p] * 5 + [_i64] * 5),
    "int4gemv_w4a16_workspace_size": (ctypes.c_int64, [_i64] * 4),
    "int4gemv_w4a16": (ctypes.c_int, [_p] * 5 + [_i64] * 4 + [_p, _i64, _p]),
    "int4gemv_w4a16_kernel_name": (ctypes.c_char_p, [_p] * 4 + [_i64] * 4),
    "int4gemv_w4a16_kernel": (ctypes.c_int, [ctypes.c_char_p] + [_p] * 5 + [_i64] * 4 + [_p]),
    "int4gemv_w4a16_silu_mul": (ctypes.c_int, [_p] * 5 + [_i64] * 4 + [_p]),
    "int4gemv_w4a16_f32": (ctypes.c_int, [_p] * 5 + [_i64] * 4 + [_p]),
    "int4gemv_unpack": (ctypes.c_int, [_p, _p, _i64, _i64, _p]),
    "int4gemv_dequantize": (ctypes.c_int, [_p] * 4 + [_i64] * 3 + [_p]),
    "int4gemv_w4a16_grouped": (ctypes.c_int, [ctypes.c_int, _p, _p] + [_p] * 4 + [_i64] * 3
                               + [_p]),
    "int4gemv_w4a16_bias_residual": (ctypes.c_int, [_p] * 7 + [_i64] * 4 + [_p]),
    "int4gemv_repack_awq": (ctypes.c_int, [_p] * 6 + [_i64] * 3 + [_p]),
    "int4gemv_repack_gptq": (ctypes.c_int, [_p] * 6 + [ctypes.c_int] + [_i64] * 3 + [_p]),
    "int4gemv_quantize": (ctypes.c_int, [_p] * 4 + [ctypes.c_int] + [_i64] * 3 + [_p]),
    "int4gemv_pack": (ctypes.c_int, [_p, _p, _i64, _i64, _p]),
    "int4gemv_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "int4gemv_set_strict_weights": (ctypes.c_int, [ctypes.c_int]),
    "int4gemv_peers_struct_bytes": (ctypes.c_size_t, []),
    "int4gemv_peer_alloc": (ctypes.c_int, [_i64, ctypes.POINTER(_p), _p]),
    "int4gemv_peer_open": (ctypes.c_int, [_p, ctypes.POINTER(_p)]),
    "int4gemv_peer_close": (ctypes.c_int, [_p]),
    "int4gemv_peer_free": (ctypes.c_int, [_p]),
    "int4gemv_w4a16_exchange": (ctypes.c_int, [_p] * 5 + [_i64] * 4 + [_p, _p]),
    "int4gemv_w4a16_exchange_static": (ctypes.c_int, [_p] * 5 + [_i64] * 4 + [ctypes.c_int, _p]),
}

MAX_PEERS = 8
SHARD_ROWS, SHARD_K = 0, 1
PEER_COUNTER_BYTES = 4096
IPC_HANDLE_BYTES = 64


class Peers(ctypes.Structure):
    """int4gemv_peers_t."""

    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("mode", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("n_total", ctypes.c_int64),
                ("col0", ctypes.c_int64), ("out_bytes", ctypes.c_int64),
                ("out", _p * MAX_PEERS), ("counters", _p)]


class CapiError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lib = None


def lib() -> ctypes.CDLL:
    """Load libint4gemv_b200.so (fails loudly if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OSError(f"{LIB_PATH} is not built; run: python int4-gemv-cuda_b200/build.py")
        lib_ = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _PROTOTYPES.items():
            fn = getattr(lib_, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib_
    return _lib


def header_functions() -> list[str]:
    """Every function the public header declares."""
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"\b(int4gemv_\w+)\s*\(", text)))


def last_error() -> str:
    return lib().int4gemv_last_error().decode()


def check(code: int) -> None:
    if code != OK:
        raise CapiError(code, last_error())


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise CapiError on failure."""
    check(getattr(lib(), name)(*args))


def kernel_info(kernel: str, m: int, threads_per_block: int = 128, rows_per_warp: int = 2) -> dict:
    out = (ctypes.c_int64 * 6)()
    call("int4gemv_kernel_info", kernel.encode(), m, threads_per_block, rows_per_warp, out)
    keys = ("registers", "local_bytes", "threads_per_block", "max_threads_per_block",
            "blocks_per_sm", "warps_per_sm")
    return dict(zip(keys, list(out)))


def device_status() -> int:
    v = ctypes.c_int(0)
    call("int4gemv_device_status", ctypes.byref(v))
    return v.value


def w4a16_kernel_name(x, qweight, scales, zeros, m, n, k, group_size) -> str:
    return lib().int4gemv_w4a16_kernel_name(x, qweight, scales, zeros, m, n, k,
                                            group_size).decode()
