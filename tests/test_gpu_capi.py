"""The C ABI on a B200, called exactly as a non-torch caller would: raw device pointers, sizes
and a stream handle (torch only allocates the buffers)."""

import numpy as np
import pytest
import torch

import oracle
from int4gemv import capi

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptrs(*ts):
    return [t.data_ptr() for t in ts]


@pytest.mark.parametrize("m,n,k", [(1, 8192, 8192), (4, 4096, 14336), (16, 1000, 1024)])
def test_w4a16_through_c_abi(m, n, k):
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=k)
    tx, tq, ts, tz = dev(x), dev(q), dev(s), dev(z)
    y = torch.empty(m, n, dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ws_bytes = capi.lib().int4gemv_w4a16_workspace_size(m, n, k, 128)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    capi.call("int4gemv_w4a16", *ptrs(y, tx, tq, ts, tz), m, n, k, 128, ws.data_ptr(), ws_bytes,
              stream)
    torch.cuda.synchronize()
    ok, msg = oracle.check_close(y.float().cpu().numpy(), oracle.reference(x, q, s, z))
    assert ok, msg
    want = "tc_dequant" if m >= 9 else "stripe_mma" if k % 2048 == 0 else "stream_mma"
    assert capi.w4a16_kernel_name(*ptrs(tx, tq, ts, tz), m, n, k, 128) == want


def test_every_gemv_entry_point():
    m, n, k = 3, 300, 1024
    x, q, s, z = oracle.synthetic(m, n, k, 128, seed=1)
    tx, tq, ts, tz = dev(x), dev(q), dev(s), dev(z)
    ref = oracle.reference(x, q, s, z)
    stream = torch.cuda.current_stream().cuda_stream
    for fn, extra in (("int4gemv_naive", []), ("int4gemv_coalesced", []),
                      ("int4gemv_vectorized", [128, 2])):
        y = torch.empty(m, n, dtype=torch.float16, device="cuda")
        capi.call(fn, *ptrs(y, tx, tq, ts, tz), m, n, k, 128, *extra, stream)
        torch.cuda.synchronize()
        ok, msg = oracle.check_close(y.float().cpu().numpy(), ref)
        assert ok, (fn, msg)


def test_unpack_dequantize_through_c_abi():
    _, q, s, z = oracle.synthetic(1, 77, 512, 64, seed=4)
    tq, ts, tz = dev(q), dev(s), dev(z)
    out_q = torch.empty(77, 512, dtype=torch.int32, device="cuda")
    out_w = torch.empty(77, 512, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    capi.call("int4gemv_unpack", out_q.data_ptr(), tq.data_ptr(), 77, 512, stream)
    capi.call("int4gemv_dequantize", out_w.data_ptr(), tq.data_ptr(), ts.data_ptr(), tz.data_ptr(),
              77, 512, 64, stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out_q.cpu().numpy(), oracle.unpack(q))
    np.testing.assert_array_equal(out_w.cpu().numpy().view(np.uint32),
                                  oracle.dequantize(q, s, z, 64).view(np.uint32))


def test_kernel_info_and_status():
    for kern in ("naive", "coalesced", "vectorized", "w4a16"):
        info = capi.kernel_info(kern, 1)
        assert info["registers"] > 0 and info["max_threads_per_block"] >= info["threads_per_block"]
    with pytest.raises(capi.CapiError, match="unknown kernel"):
        capi.kernel_info("bogus", 1)
    assert capi.device_status() == 0


def stripe_fold_oracle(q, s, z):
    """out[r] = XOR of the row's packed words and, per group, of (scale bits | zero bits << 16)."""
    out = np.bitwise_xor.reduce(q.view(np.uint32), axis=1)
    sz = s.view(np.uint16).astype(np.uint32) | (z.view(np.uint16).astype(np.uint32) << 16)
    return out ^ np.bitwise_xor.reduce(sz, axis=1)


@pytest.mark.parametrize("n,k", [(8192, 8192), (37, 2048), (148 * 4 + 3, 4096), (1000, 28672),
                                 (16, 6144)])
def test_stripe_load_only(n, k):
    """The loads-only ceiling of the M <= 2 stream folds exactly the bytes the GEMV reads."""
    _, q, s, z = oracle.synthetic(1, n, k, 128, seed=n + k)
    tq, ts, tz = dev(q), dev(s), dev(z)
    out = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the second call reads weights the first one left in L2
        capi.call("int4gemv_stripe_load_only", *ptrs(out, tq, ts, tz), n, k, 128, stream)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32),
                                      stripe_fold_oracle(q, s, z))
    assert capi.device_status() == 0


def test_stripe_load_only_rejects():
    _, q, s, z = oracle.synthetic(1, 64, 3072, 128)
    tq, ts, tz = dev(q), dev(s), dev(z)
    out = torch.empty(64, dtype=torch.int32, device="cuda")
    with pytest.raises(capi.CapiError, match="K must be a multiple of 2048"):
        capi.call("int4gemv_stripe_load_only", *ptrs(out, tq, ts, tz), 64, 3072, 128, None)
