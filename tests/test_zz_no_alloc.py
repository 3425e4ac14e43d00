"""int4gemv_w4a16_exchange_static (no allocation: static device scratch) against the existing
entry point int4gemv_w4a16_exchange with caller-allocated buffers (world 1), two calls in a row per
mode, bit for bit; and its size limit. Collected last, and passes alone as well."""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from int4gemv import capi

pytestmark = pytest.mark.gpu


def _alloc(nbytes):
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_char * capi.IPC_HANDLE_BYTES)()
    capi.check(capi.lib().int4gemv_peer_alloc(nbytes, ctypes.byref(ptr), ctypes.addressof(handle)))
    return ptr.value


@pytest.mark.parametrize("mode", [capi.SHARD_ROWS, capi.SHARD_K])
def test_static_matches_existing_entry_two_calls(mode):
    m, n, k = 2, 4096, 4096
    _, q, s, z = oracle.synthetic(1, n, k, 128, seed=21)
    tq, ts, tz = (torch.from_numpy(a).cuda() for a in (q, s, z))
    out_bytes = 2 * m * n * 8  # two halves of one 8-byte tagged word per output
    out, counters = _alloc(out_bytes), _alloc(capi.PEER_COUNTER_BYTES)
    peers = capi.Peers()
    peers.world, peers.rank, peers.mode, peers.n_total, peers.col0 = 1, 0, mode, n, 0
    peers.out_bytes, peers.out[0], peers.counters = out_bytes, out, counters
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for call in range(2):
            x = np.random.default_rng(call).standard_normal((m, k)).astype(np.float16)
            tx = torch.from_numpy(x).cuda()
            y_static = torch.empty(m, n, dtype=torch.float16, device="cuda")
            y_alloc = torch.empty(m, n, dtype=torch.float16, device="cuda")
            capi.call("int4gemv_w4a16_exchange_static", y_static.data_ptr(), tx.data_ptr(),
                      tq.data_ptr(), ts.data_ptr(), tz.data_ptr(), m, n, k, 128, mode, stream)
            capi.call("int4gemv_w4a16_exchange", y_alloc.data_ptr(), tx.data_ptr(), tq.data_ptr(),
                      ts.data_ptr(), tz.data_ptr(), m, n, k, 128, ctypes.addressof(peers), stream)
            torch.cuda.synchronize()
            assert torch.equal(y_static.view(torch.int16), y_alloc.view(torch.int16)), call
            ok, msg = oracle.check_close(y_static.float().cpu().numpy(),
                                         oracle.reference(x, q, s, z, 128))
            assert ok, msg
        assert capi.device_status() == 0
    finally:
        capi.check(capi.lib().int4gemv_peer_free(out))
        capi.check(capi.lib().int4gemv_peer_free(counters))


def test_static_rejects_oversize():
    x = torch.zeros(32, 1024, dtype=torch.float16, device="cuda")
    with pytest.raises(capi.CapiError, match="static buffer holds"):
        capi.call("int4gemv_w4a16_exchange_static", x.data_ptr(), x.data_ptr(), x.data_ptr(),
                  x.data_ptr(), x.data_ptr(), 32, 16384, 1024, 128, capi.SHARD_K, None)


def test_static_alternating_shapes_share_one_buffer():
    """Calls of different shapes and modes in a row on the one static buffer, with a rejected
    oversize call in between: each result is bit-identical to the same kernel (stripe_mma, which
    the exchange runs on for M <= 8 and K % 2048 == 0) run through the named-kernel entry point,
    and the device status stays clean."""
    k = 4096
    _, q, s, z = oracle.synthetic(1, 8192, k, 128, seed=23)
    tq, ts, tz = (torch.from_numpy(a).cuda() for a in (q, s, z))
    stream = torch.cuda.current_stream().cuda_stream
    sequence = [(capi.SHARD_ROWS, 1, 8192), (capi.SHARD_K, 4, 4096), (None, 32, 16384),
                (capi.SHARD_ROWS, 2, 4096), (capi.SHARD_K, 1, 8192)]
    for i, (mode, m, n) in enumerate(sequence):
        x = np.random.default_rng(100 + i).standard_normal((m, k)).astype(np.float16)
        tx = torch.from_numpy(x).cuda()
        y_static = torch.empty(m, n, dtype=torch.float16, device="cuda")
        if mode is None:  # larger than the static buffer: rejected, nothing launched
            with pytest.raises(capi.CapiError, match="static buffer holds"):
                capi.call("int4gemv_w4a16_exchange_static", y_static.data_ptr(), tx.data_ptr(),
                          tq.data_ptr(), ts.data_ptr(), tz.data_ptr(), m, n, k, 128,
                          capi.SHARD_K, stream)
            continue
        y_plain = torch.empty(m, n, dtype=torch.float16, device="cuda")
        capi.call("int4gemv_w4a16_exchange_static", y_static.data_ptr(), tx.data_ptr(),
                  tq.data_ptr(), ts.data_ptr(), tz.data_ptr(), m, n, k, 128, mode, stream)
        capi.call("int4gemv_w4a16_kernel", b"stripe_mma", y_plain.data_ptr(), tx.data_ptr(),
                  tq.data_ptr(), ts.data_ptr(), tz.data_ptr(), m, n, k, 128, stream)
        torch.cuda.synchronize()
        assert torch.equal(y_static.view(torch.int16), y_plain.view(torch.int16)), (mode, m, n)
    assert capi.device_status() == 0

