"""AWQ / GPTQ checkpoint repacking on the device (ops.repack_awq / ops.repack_gptq and the C ABI),
bit for bit against the vLLM-packed golden tensors, the oracle's restatement on ragged shapes, and
at full size (28672 x 8192) against a torch-side construction of the checkpoint layouts."""

import numpy as np
import pytest
import torch

import oracle
from int4gemv import capi, checkpoint, ops

pytestmark = pytest.mark.gpu


def cuda(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def bits16(t):
    a = t.cpu().numpy() if isinstance(t, torch.Tensor) else t
    return np.ascontiguousarray(a).view(np.uint16)


def assert_layout(got, q, s, z):
    np.testing.assert_array_equal(got[0].cpu().numpy(), q)
    np.testing.assert_array_equal(bits16(got[1]), bits16(s))
    np.testing.assert_array_equal(got[2].float().cpu().numpy(), np.asarray(z, np.float32))


def test_awq_golden(checkpoint_case):
    c = checkpoint_case
    got = checkpoint.from_awq(*cuda(c["awq_qweight"], c["awq_qzeros"], c["awq_scales"]),
                              int(c["group_size"]))
    assert_layout(got, c["qweight"], c["scales"], c["zeros"])


@pytest.mark.parametrize("fmt", ["gptq", "gptq_v2"])
def test_gptq_golden(checkpoint_case, fmt):
    c = checkpoint_case
    g = int(c["group_size"])
    qz = c["gptq_qzeros"] if fmt == "gptq" else c["gptq_v2_qzeros"]
    g_idx = torch.arange(c["gptq_qweight"].shape[0] * 8, dtype=torch.int32, device="cuda") // g
    got = checkpoint.from_gptq(*cuda(c["gptq_qweight"], qz, c["gptq_scales"]), g, g_idx=g_idx,
                               checkpoint_format=fmt)
    want = oracle.gptq_to_packed(c["gptq_qweight"], qz, c["gptq_scales"], g, fmt)
    assert_layout(got, *want)
    np.testing.assert_array_equal(got[0].cpu().numpy(), c["qweight"])


@pytest.fixture(params=__import__("conftest").golden_names("checkpoint_"))
def checkpoint_case(request):
    from conftest import load_golden

    return load_golden(request.param)


# ragged against the tiles: N not a multiple of 256 (AWQ) or 32 (GPTQ), K not a multiple of 64
SHAPES = [(8, 8, 8), (200, 1000, 8), (264, 1088, 64), (1032, 4096, 128), (4104, 2944, 128)]


@pytest.mark.parametrize("n,k,g", SHAPES, ids=[f"n{n}_k{k}_g{g}" for n, k, g in SHAPES])
def test_ragged_shapes_against_oracle(n, k, g):
    _, q, s, z = oracle.synthetic(1, n, k, g, seed=n + k)
    aq, az, as_ = oracle.packed_to_awq(q, s, z)
    got = ops.repack_awq(*cuda(aq, az, as_), g)
    assert_layout(got, *oracle.awq_to_packed(aq, az, as_, g))
    np.testing.assert_array_equal(got[0].cpu().numpy(), q)
    for fmt, off in (("gptq", 1), ("gptq_v2", 0)):
        gq, gz, gs = oracle.packed_to_gptq(q, s, z, fmt)
        got = ops.repack_gptq(*cuda(gq, gz, gs), g, off)
        assert_layout(got, *oracle.gptq_to_packed(gq, gz, gs, g, fmt))


def test_full_size_round_trip_and_gemv():
    """28672 x 8192: build both checkpoint layouts from a packed matrix with torch ops on the
    device, repack, and get the matrix back exactly; the GEMV on the repacked weights then matches
    the oracle."""
    n, k, g = 28672, 8192, 128
    gen = torch.Generator(device="cuda").manual_seed(3)
    w = torch.randn(n, k, generator=gen, device="cuda", dtype=torch.float16) * 0.02
    q, s, z = ops.quantize(w, g)
    del w
    vals = ops.unpack(q).t().contiguous()                   # [K, N] values 0..15
    shifts = torch.arange(0, 32, 4, device="cuda", dtype=torch.int64)
    order = torch.tensor([0, 2, 4, 6, 1, 3, 5, 7], device="cuda")

    def pack8(v):  # [..., 8] -> int32 words, element i in nibble i
        word = (v.to(torch.int64) << shifts).sum(-1) & 0xFFFFFFFF
        return torch.where(word >= 2**31, word - 2**32, word).to(torch.int32)

    zi = z.float().round().to(torch.int32).t().contiguous()  # [K/g, N]
    awq_q = pack8(vals.view(k, n // 8, 8)[..., order])
    awq_z = pack8(zi.view(k // g, n // 8, 8)[..., order])
    got = ops.repack_awq(awq_q, awq_z, s.t().contiguous(), g)
    del awq_q
    assert torch.equal(got[0], q) and torch.equal(got[1].view(torch.int16), s.view(torch.int16))
    assert torch.equal(got[2].float(), z.float())
    gptq_q = q.t().contiguous()                              # [K/8, N]: already k-packed
    gptq_z = pack8(((zi - 1) & 0xF).view(k // g, n // 8, 8))
    got = checkpoint.from_gptq(gptq_q, gptq_z, s.t().contiguous(), g)
    assert torch.equal(got[0], q)
    assert torch.equal(got[2].float(), torch.where(z.float() == 0, 16.0, z.float()))
    del vals, gptq_q
    x = torch.randn(1, k, generator=gen, device="cuda", dtype=torch.float16)
    rows = slice(0, 2048)
    y = ops.w4a16(x, got[0][rows].contiguous(), got[1][rows].contiguous(),
                  got[2][rows].contiguous(), g)
    ref = oracle.reference(x.cpu().numpy(), got[0][rows].cpu().numpy(),
                           got[1][rows].cpu().numpy(), got[2][rows].cpu().numpy(), g)
    ok, msg = oracle.check_close(y.float().cpu().numpy(), ref)
    assert ok, msg


def test_checks_and_c_abi():
    _, q, s, z = oracle.synthetic(1, 64, 256, 128, seed=1)
    aq, az, as_ = cuda(*oracle.packed_to_awq(q, s, z))
    with pytest.raises(RuntimeError, match="qzeros must be"):
        ops.repack_awq(aq, az[:1], as_, 128)
    with pytest.raises(RuntimeError, match="group_size"):
        ops.repack_awq(aq, az, as_, 100)
    gq, gz, gs = cuda(*oracle.packed_to_gptq(q, s, z))
    with pytest.raises(RuntimeError, match="zero_offset"):
        ops.repack_gptq(gq, gz, gs, 128, 2)
    outs = [torch.empty(64, 32, dtype=torch.int32, device="cuda"),
            torch.empty(64, 2, dtype=torch.float16, device="cuda"),
            torch.empty(64, 2, dtype=torch.float16, device="cuda")]
    stream = torch.cuda.current_stream().cuda_stream
    capi.call("int4gemv_repack_gptq", *(t.data_ptr() for t in outs), gq.data_ptr(), gz.data_ptr(),
              gs.data_ptr(), 1, 64, 256, 128, stream)
    torch.cuda.synchronize()
    assert_layout(outs, *oracle.gptq_to_packed(*(t.cpu().numpy() for t in (gq, gz, gs)), 128))
    with pytest.raises(RuntimeError, match="multiple of 8"):
        capi.call("int4gemv_repack_awq", *(t.data_ptr() for t in outs), aq.data_ptr(),
                  az.data_ptr(), as_.data_ptr(), 60, 256, 128, stream)
