"""Device quantize / pack (ops.quantize, ops.pack, the C ABI's int4gemv_quantize / int4gemv_pack)
compared bit for bit with the reference's golden vectors and with the C oracle, which restates
int4gemv/quant.py:14-37.

One documented divergence from the reference: when a group's minimum is a zero present with both
signs, torch's vectorised min reduction picks the sign by SIMD lane order (host dependent); the
kernel and the oracle take the first zero in k order. Only the sign bit of a zero zero-point can
differ, and z = +0 and z = -0 dequantise identically. Such groups are compared with the oracle.
"""

import numpy as np
import pytest
import torch

import oracle
from int4gemv import capi, ops, quant

pytestmark = pytest.mark.gpu


def bits16(t):
    a = t.cpu().numpy() if isinstance(t, torch.Tensor) else t
    return np.ascontiguousarray(a).view(np.uint16)


def assert_same(got, want, what=""):
    q, s, z = got
    wq, ws, wz = want
    np.testing.assert_array_equal(q.cpu().numpy(), wq, err_msg=f"qweight {what}")
    np.testing.assert_array_equal(bits16(s), bits16(ws), err_msg=f"scales {what}")
    np.testing.assert_array_equal(bits16(z), bits16(wz), err_msg=f"zeros {what}")


def test_golden(golden):
    if "w" not in golden:
        pytest.skip("case stores no float weights")
    g = int(golden["group_size"])
    got = ops.quantize(torch.from_numpy(golden["w"]).cuda(), g)
    assert got[0].dtype == torch.int32 and got[1].dtype == torch.float16
    assert_same(got, (golden["qweight"], golden["scales"], golden["zeros"]), golden["name"])


def edge_rows(k, rng):
    """Rows that reach every branch: all zero, signed zeros in mixed order, constant, all
    positive / negative, .5 ties of w / s, subnormal, huge, and random."""
    pos = np.abs(rng.standard_normal(k)).astype(np.float32) + 0.1
    rows = [np.zeros(k), -np.zeros(k), np.full(k, 0.37), np.full(k, -2.5), pos, -pos,
            np.round(rng.uniform(-15, 15, k)) / 30.0,
            rng.standard_normal(k) * 1e-39, rng.standard_normal(k) * 3e4,
            rng.standard_normal(k) * 0.02]
    for a, b in ((0, 3), (3, 0), (1, k - 1), (k - 1, 1)):
        r = pos.copy()
        r[a], r[b] = -0.0, 0.0
        rows.append(r)
    return np.stack(rows).astype(np.float32)


@pytest.mark.parametrize("g", [8, 16, 24, 32, 40, 64, 128, 256, 384, 512, 1024])
def test_group_sizes_against_oracle(g):
    rng = np.random.default_rng(g)
    k = g * max(1, 2048 // g)
    w = np.concatenate([edge_rows(k, rng), (rng.standard_normal((53, k)) * 0.02)]).astype(
        np.float32)
    assert_same(ops.quantize(torch.from_numpy(w).cuda(), g), oracle.quantize(w, g), f"g={g}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_narrow_input_types(dtype):
    """The kernel reads fp16 / bf16 directly; the reference widens to fp32 first (exact)."""
    gen = torch.Generator().manual_seed(7)
    w = (torch.randn(300, 4096, generator=gen) * 0.02).to(dtype)
    w[0, :128] = 0
    w[1, 5:9] = torch.tensor([1e-7, -3e-6, 60000.0, -0.0]).to(dtype)
    got = ops.quantize(w.cuda(), 128)
    assert_same(got, oracle.quantize(w.float().numpy(), 128), str(dtype))
    assert_same(got, tuple(t.numpy() for t in quant.quantize(w, 128)), f"host {dtype}")


def test_full_size_rows_against_oracle():
    """28672 x 8192 (the sharded up projection): sampled rows bit-exact with the oracle, and the
    whole matrix row-independent (a slice quantises to the same rows)."""
    gen = torch.Generator(device="cuda").manual_seed(0)
    w = torch.randn(28672, 8192, generator=gen, device="cuda", dtype=torch.float16) * 0.02
    q, s, z = ops.quantize(w, 128)
    torch.cuda.synchronize()
    rows = np.random.default_rng(1).choice(28672, 40, replace=False)
    rows.sort()
    idx = torch.from_numpy(rows).cuda()
    want = oracle.quantize(w[idx].float().cpu().numpy(), 128)
    assert_same((q[idx], s[idx], z[idx]), want, "sampled rows")
    part = ops.quantize(w[20000:20480].contiguous(), 128)
    for a, b in zip(part, (q[20000:20480], s[20000:20480], z[20000:20480])):
        assert torch.equal(a.view(torch.int16) if a.dtype == torch.float16 else a,
                           b.view(torch.int16) if b.dtype == torch.float16 else b)
    # dequantised weights stay within one step of the input: half a step of rounding, plus at most
    # half a step at the top of the range, where the rounded zero point can push q past 15
    deq = ops.dequantize(q[:512], s[:512], z[:512], 128)
    step = s[:512].float().repeat_interleave(128, dim=1)
    assert bool(((deq - w[:512].float()).abs() <= step * (1 + 1e-3)).all())


def test_quant_quantize_uses_device_kernel():
    """quant.quantize on a CUDA tensor runs the device kernel and matches the host path."""
    w = torch.randn(64, 1024, generator=torch.Generator().manual_seed(3)) * 0.02
    got = quant.quantize(w.cuda(), 128)
    assert all(t.is_cuda for t in got)
    assert_same(got, tuple(t.numpy() for t in quant.quantize(w, 128)), "host vs device")
    w64 = w.double()
    assert_same(quant.quantize(w64.cuda(), 128), tuple(t.numpy() for t in quant.quantize(w64, 128)),
                "float64 input")


def test_pack_golden(pack_wrap):
    got = ops.pack(torch.from_numpy(pack_wrap["q"]).cuda())
    np.testing.assert_array_equal(got.cpu().numpy(), pack_wrap["qweight"])


def test_pack_unpack_round_trip_full_size():
    gen = torch.Generator(device="cuda").manual_seed(5)
    qw = torch.randint(-2**31, 2**31 - 1, (28672, 1024), generator=gen, device="cuda",
                       dtype=torch.int32)
    assert torch.equal(ops.pack(ops.unpack(qw)), qw)


def test_empty_and_errors():
    q, s, z = ops.quantize(torch.empty(0, 256, device="cuda"), 128)
    assert q.shape == (0, 32) and s.shape == (0, 2)
    assert ops.pack(torch.empty(3, 0, dtype=torch.int32, device="cuda")).shape == (3, 0)
    with pytest.raises(RuntimeError, match="group_size"):
        ops.quantize(torch.zeros(4, 256, device="cuda"), 100)
    with pytest.raises(RuntimeError, match="float32, float16 or bfloat16"):
        ops.quantize(torch.zeros(4, 256, dtype=torch.int32, device="cuda"), 128)
    with pytest.raises(RuntimeError, match="contiguous"):
        ops.quantize(torch.zeros(256, 4, device="cuda").t(), 128)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        ops.pack(torch.zeros(4, 12, dtype=torch.int32, device="cuda"))


def test_through_c_abi():
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((37, 768)) * 0.02).astype(np.float32)
    tw = torch.from_numpy(w).cuda()
    q = torch.empty(37, 96, dtype=torch.int32, device="cuda")
    s = torch.empty(37, 6, dtype=torch.float16, device="cuda")
    z = torch.empty(37, 6, dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    capi.call("int4gemv_quantize", q.data_ptr(), s.data_ptr(), z.data_ptr(), tw.data_ptr(), 0, 37,
              768, 128, stream)
    torch.cuda.synchronize()
    assert_same((q, s, z), oracle.quantize(w, 128), "C ABI")
    q2 = torch.empty_like(q)
    unpacked = ops.unpack(q)
    capi.call("int4gemv_pack", q2.data_ptr(), unpacked.data_ptr(), 37, 768, stream)
    torch.cuda.synchronize()
    assert torch.equal(q2, q)
    with pytest.raises(RuntimeError, match="dtype"):
        capi.call("int4gemv_quantize", q.data_ptr(), s.data_ptr(), z.data_ptr(), tw.data_ptr(), 7,
                  37, 768, 128, stream)
