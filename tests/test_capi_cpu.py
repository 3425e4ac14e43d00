"""The C ABI library on the CPU: it loads, exports every declared symbol, runs the CPU path
bit-exactly, and rejects bad arguments with the reference's messages before touching the GPU."""

import ctypes

import numpy as np
import pytest

import oracle
from int4gemv import capi


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def test_library_exports_every_header_symbol():
    lib = capi.lib()
    names = capi.header_functions()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_version():
    assert capi.lib().int4gemv_version() >= 100


def test_sequential_bit_exact(golden):
    g = int(golden["group_size"])
    x, q, s, z = (np.ascontiguousarray(golden[k]) for k in ("x", "qweight", "scales", "zeros"))
    m, k = x.shape
    n = q.shape[0]
    for threads in (1, 3, 0):
        y = np.empty((m, n), np.float16)
        capi.call("int4gemv_sequential", ptr(y), ptr(x), ptr(q), ptr(s), ptr(z), m, n, k, g,
                  threads)
        np.testing.assert_array_equal(y.view(np.uint16), golden["y_seq"].view(np.uint16))


def test_sequential_empty_and_zero_k():
    y = np.full((2, 3), 7, np.float16)
    x = np.zeros((2, 0), np.float16)
    capi.call("int4gemv_sequential", ptr(y), ptr(x), None, None, None, 2, 3, 0, 128, 1)
    assert (y == 0).all()
    capi.call("int4gemv_sequential", None, None, None, None, None, 0, 3, 128, 128, 1)


@pytest.mark.parametrize(
    "fn,extra,args,message",
    [
        ("int4gemv_naive", [], (1, 8, 384, 100), "naive: group_size 100 must be a positive multiple of 8 dividing K = 384"),
        ("int4gemv_coalesced", [], (1, 8, 384, 0), "coalesced: group_size 0 must be a positive multiple of 8 dividing K = 384"),
        ("int4gemv_w4a16", [None, 0], (1, 8, 2**31, 128), "w4a16: M = 1, N = 8, K = 2147483648 must each fit in int"),
        ("int4gemv_vectorized", [24, 2], (1, 8, 384, 128), "vectorized: threads_per_block must be a multiple of 32 in [32, 1024], got 24"),
        ("int4gemv_vectorized", [128, 2], (1, 8, 384, 64 + 64 + 64 + 8), None),
        ("int4gemv_vectorized", [128, 2], (1, 8, 384, 8), "vectorized: group_size must be a multiple of 32, got 8"),
        ("int4gemv_load_only", [128, 2], (2, 8, 384, 128), "load_only: needs M = 1, got 2"),
    ],
)
def test_argument_errors(fn, extra, args, message):
    m, n, k, g = args
    fake = ctypes.c_void_p(4096)  # never dereferenced: the checks fail first
    res = getattr(capi.lib(), fn)(fake, fake, fake, fake, fake, m, n, k, g, *extra, None)
    assert res == capi.ERR_INVALID
    if message:
        assert capi.last_error() == message
    else:
        assert "group_size" in capi.last_error()


def test_misaligned_vectorized():
    res = capi.lib().int4gemv_vectorized(8, 4104, 4096, 4096, 4096, 1, 8, 256, 128, 128, 2, None)
    assert res == capi.ERR_INVALID
    assert capi.last_error() == "vectorized: x and qweight must be 16-byte aligned"


def test_rows_per_warp_error_message():
    # rows_per_warp is checked after the tensor checks and has no name prefix, as in the reference
    res = capi.lib().int4gemv_vectorized(4096, 4096, 4096, 4096, 4096, 1, 8, 256, 128, 128, 3,
                                         None)
    assert res == capi.ERR_INVALID
    assert capi.last_error() == "rows_per_warp must be 1, 2 or 4, got 3"


def test_null_pointer_rejected():
    res = capi.lib().int4gemv_naive(None, None, None, None, None, 1, 8, 256, 128, None)
    assert res == capi.ERR_INVALID and "null pointer" in capi.last_error()


def test_workspace_size_is_nonnegative():
    assert capi.lib().int4gemv_w4a16_workspace_size(1, 8192, 8192, 128) >= 0


def test_peers_struct_layout():
    """The ctypes mirror of int4gemv_peers_t has the C struct's size."""
    import ctypes

    assert ctypes.sizeof(capi.Peers) == capi.lib().int4gemv_peers_struct_bytes()


def test_exchange_rejects_bad_peers():
    """Argument checks of int4gemv_w4a16_exchange run before any CUDA call."""
    import ctypes

    peers = capi.Peers()
    peers.world, peers.rank, peers.mode = 9, 0, capi.SHARD_ROWS
    with pytest.raises(capi.CapiError, match="at most 8 ranks"):
        capi.call("int4gemv_w4a16_exchange", None, 16, 16, 16, 16, 1, 64, 1024, 128,
                  ctypes.addressof(peers), None)
    peers.world, peers.mode = 1, 7
    with pytest.raises(capi.CapiError, match="unknown mode"):
        capi.call("int4gemv_w4a16_exchange", None, 16, 16, 16, 16, 1, 64, 1024, 128,
                  ctypes.addressof(peers), None)
    peers.mode = capi.SHARD_ROWS
    with pytest.raises(capi.CapiError, match="null buffer"):
        capi.call("int4gemv_w4a16_exchange", None, 16, 16, 16, 16, 1, 64, 1024, 128,
                  ctypes.addressof(peers), None)
