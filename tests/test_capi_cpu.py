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


def test_workspace_only_for_the_wide_fast_path():
    """The fast path uses a workspace (x permuted once per call) only where stream_mma's wide path
    runs: 5 <= M <= 8 on its shapes (group 128, K % 1024 == 0) that stripe_mma does not take (K not
    a multiple of 2048, or x and the partials of a CTA's rows too large); from M = 9 on tc_dequant
    is picked and needs none from the caller."""
    size = capi.lib().int4gemv_w4a16_workspace_size
    assert size(1, 8192, 8192, 128) == 0 and size(4, 8192, 8192, 128) == 0
    assert size(8, 8192, 8192, 128) == 0 and size(5, 8192, 8192, 128) == 0  # stripe_mma
    assert size(8, 28672, 8192, 128) > size(5, 8192, 3072, 128) > 0  # stream_mma's wide path
    assert size(8, 28672, 8192, 128) >= 8 * 8192 * 2  # at least x itself, permuted
    assert size(9, 8192, 8192, 128) == 0 and size(32, 8192, 8192, 128) == 0
    assert size(8, 8192, 8192, 64) == 0 and size(8, 8192, 1152, 128) == 0
    assert size(0, 8192, 8192, 128) == 0 and size(16, 8192, 8192, 100) == 0


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


FAKE = 4096  # a 16-byte-aligned address that is never dereferenced: the checks below fail first


@pytest.mark.parametrize("count,ns,message", [
    (0, [1], "w4a16_grouped: count 0 must be in [1, 8] with ys and ns given"),
    (9, [1] * 9, "w4a16_grouped: count 9 must be in [1, 8] with ys and ns given"),
    (2, [4, -1], "w4a16_grouped: ns[1] = -1 < 0"),
])
def test_grouped_argument_errors(count, ns, message):
    ys = (ctypes.c_void_p * max(count, 1))(*([FAKE] * max(count, 1)))
    sizes = (ctypes.c_int64 * max(count, 1))(*(ns or [0]))
    res = capi.lib().int4gemv_w4a16_grouped(count, ys, sizes, FAKE, FAKE, FAKE, FAKE, 1, 1024,
                                            128, None)
    assert res == capi.ERR_INVALID
    assert capi.last_error() == message


def test_grouped_and_bias_empty_calls_launch_nothing():
    ys = (ctypes.c_void_p * 2)(FAKE, FAKE)
    sizes = (ctypes.c_int64 * 2)(0, 0)
    assert capi.lib().int4gemv_w4a16_grouped(2, ys, sizes, FAKE, FAKE, FAKE, FAKE, 1, 1024, 128,
                                             None) == capi.OK
    assert capi.lib().int4gemv_w4a16_bias_residual(FAKE, FAKE, FAKE, FAKE, FAKE, None, None, 0, 64,
                                                   1024, 128, None) == capi.OK
    res = capi.lib().int4gemv_w4a16_bias_residual(FAKE, FAKE, FAKE, FAKE, FAKE, None, None, 1, 64,
                                                  1000, 128, None)
    assert res == capi.ERR_INVALID and "group_size 128" in capi.last_error()


def test_quantize_pack_repack_argument_errors():
    lib = capi.lib()
    cases = [
        (lambda: lib.int4gemv_quantize(FAKE, FAKE, FAKE, FAKE, 7, 4, 256, 128, None),
         "quantize: unknown weight dtype 7"),
        (lambda: lib.int4gemv_quantize(FAKE, FAKE, FAKE, FAKE, 0, 4, 256, 100, None),
         "quantize: group_size 100 must be a positive multiple of 8 dividing K = 256"),
        (lambda: lib.int4gemv_quantize(FAKE, FAKE, FAKE, FAKE + 4, 0, 4, 256, 128, None),
         "quantize: w must be 16-byte aligned"),
        (lambda: lib.int4gemv_pack(FAKE, FAKE, 4, 12, None),
         "pack: N = 4, K = 12: K must be a non-negative multiple of 8"),
        (lambda: lib.int4gemv_pack(FAKE, FAKE + 8, 4, 16, None), "pack: q must be 16-byte aligned"),
        (lambda: lib.int4gemv_repack_awq(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 60, 256, 128, None),
         "repack_awq: N = 60 must be a multiple of 8 (packed zero points)"),
        (lambda: lib.int4gemv_repack_gptq(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 2, 64, 256, 128,
                                          None),
         "repack_gptq: zero_offset 2 must be 0 or 1"),
    ]
    for call, message in cases:
        assert call() == capi.ERR_INVALID
        assert capi.last_error() == message
    assert lib.int4gemv_quantize(FAKE, FAKE, FAKE, FAKE, 1, 0, 256, 128, None) == capi.OK


def test_exchange_size_checks():
    peers = capi.Peers()
    peers.world, peers.rank, peers.mode = 2, 1, capi.SHARD_ROWS
    peers.out[0], peers.out[1], peers.counters = FAKE, FAKE, FAKE
    peers.n_total, peers.col0, peers.out_bytes = 100, 64, 1 << 20
    res = capi.lib().int4gemv_w4a16_exchange(FAKE, FAKE, FAKE, FAKE, FAKE, 1, 64, 1024, 128,
                                             ctypes.addressof(peers), None)
    assert res == capi.ERR_INVALID and "equal shards" in capi.last_error()
    peers.n_total = 128
    peers.out_bytes = 1024  # two halves of 1 x 128 tagged 8-byte words need 2048
    res = capi.lib().int4gemv_w4a16_exchange(FAKE, FAKE, FAKE, FAKE, FAKE, 1, 64, 1024, 128,
                                             ctypes.addressof(peers), None)
    assert res == capi.ERR_INVALID
    assert capi.last_error() == ("w4a16_exchange: out buffers of 1024 bytes, 2048 needed "
                                 "(two halves)")
    res = capi.lib().int4gemv_w4a16_exchange_static(FAKE, FAKE, FAKE, FAKE, FAKE, 32, 16384, 1024,
                                                    128, capi.SHARD_K, None)
    assert res == capi.ERR_INVALID and "the static buffer holds 4194304" in capi.last_error()
    res = capi.lib().int4gemv_w4a16_exchange_static(FAKE, FAKE, FAKE, FAKE, FAKE, 1, 64, 1024,
                                                    128, 5, None)
    assert res == capi.ERR_INVALID
    assert capi.last_error() == "w4a16_exchange_static: unknown mode 5"


def test_exchange_static_checks_come_before_setup():
    """Every argument error of the no-allocation entry point is reported before its first-call
    setup (which would need a GPU here): null pointers, bad group sizes, shapes the fast path does
    not take, and sizes whose M x N would overflow if multiplied first."""
    lib = capi.lib()
    cases = [
        ((None, None, None, None, None, 1, 4096, 4096, 128, capi.SHARD_ROWS),
         "w4a16_exchange_static: null pointer for a non-empty tensor"),
        ((FAKE, FAKE, FAKE, FAKE, FAKE, 1, 4096, 4096, 100, capi.SHARD_ROWS),
         "w4a16_exchange_static: group_size 100 must be a positive multiple of 8 dividing "
         "K = 4096"),
        ((FAKE, FAKE, FAKE, FAKE, FAKE, 0, 4096, 4096, 128, capi.SHARD_K),
         "w4a16_exchange_static: M, N and K must be positive"),
        ((FAKE, FAKE, FAKE, FAKE, FAKE, 2**31 - 1, 2**31 - 1, 4096, 128, capi.SHARD_K),
         None),
        ((FAKE, FAKE, FAKE, FAKE, FAKE, 1, 4096, 1000, 8, capi.SHARD_ROWS), None),
    ]
    for args, message in cases:
        assert lib.int4gemv_w4a16_exchange_static(*args, None) == capi.ERR_INVALID
        if message is not None:
            assert capi.last_error() == message
    # the overflow case is the size limit, the last one a shape the fast path does not take
    lib.int4gemv_w4a16_exchange_static(FAKE, FAKE, FAKE, FAKE, FAKE, 2**31 - 1, 2**31 - 1, 4096,
                                       128, capi.SHARD_K, None)
    assert "the static buffer holds 4194304 bytes (M x N <= 262144)" in capi.last_error()


def test_set_strict_weights_values():
    lib = capi.lib()
    assert lib.int4gemv_set_strict_weights(2) == capi.ERR_INVALID
    assert capi.last_error() == "set_strict_weights: strict must be 0 or 1, got 2"
    assert lib.int4gemv_set_strict_weights(1) == capi.OK
    assert lib.int4gemv_set_strict_weights(0) == capi.OK

