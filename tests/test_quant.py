"""The package's quant.py (torch) is bit-exact with the reference's, pinned by golden vectors."""

import numpy as np
import pytest
import torch

import oracle
from int4gemv import quant
from int4gemv.reference import assert_matches_reference, w4a16_reference


def bits16(t):
    return np.ascontiguousarray(t.numpy() if isinstance(t, torch.Tensor) else t).view(np.uint16)


def test_quantize_matches_golden(golden):
    if "w" not in golden:
        pytest.skip("case stores no float weights")
    g = int(golden["group_size"])
    q, s, z = quant.quantize(torch.from_numpy(golden["w"]), g)
    assert q.dtype == torch.int32 and s.dtype == torch.float16 and z.dtype == torch.float16
    np.testing.assert_array_equal(q.numpy(), golden["qweight"])
    np.testing.assert_array_equal(bits16(s), bits16(golden["scales"]))
    np.testing.assert_array_equal(bits16(z), bits16(golden["zeros"]))


def test_dequantize_matches_golden(golden):
    if "deq" not in golden:
        pytest.skip("case stores no dequantized weights")
    g = int(golden["group_size"])
    w = quant.dequantize(*(torch.from_numpy(golden[k]) for k in ("qweight", "scales", "zeros")), g)
    np.testing.assert_array_equal(w.numpy().view(np.uint32), golden["deq"].view(np.uint32))


def test_unpack_pack(golden):
    qw = torch.from_numpy(golden["qweight"])
    q = quant.unpack(qw)
    np.testing.assert_array_equal(q.numpy(), oracle.unpack(golden["qweight"]))
    assert torch.equal(quant.pack(q), qw)


def test_pack_wraps_like_reference(pack_wrap):
    assert torch.equal(quant.pack(torch.from_numpy(pack_wrap["q"])),
                       torch.from_numpy(pack_wrap["qweight"]))


def test_pack_sign_bit_words():
    q = torch.full((2, 16), 15, dtype=torch.int32)
    packed = quant.pack(q)
    assert packed.dtype == torch.int32 and int(packed[0, 0]) == -1
    assert torch.equal(quant.unpack(packed), q)


def test_bits_per_weight():
    assert quant.bits_per_weight() == 4.25
    assert quant.bits_per_weight(32) == 5.0


def test_reference_api(golden):
    g = int(golden["group_size"])
    args = [torch.from_numpy(golden[k]) for k in ("x", "qweight", "scales", "zeros")]
    ref = w4a16_reference(*args, g)
    np.testing.assert_allclose(ref.numpy(), golden["y_ref"], rtol=1e-5, atol=1e-6)
    assert_matches_reference(torch.from_numpy(golden["y_seq"]), ref)
    with pytest.raises(AssertionError):
        assert_matches_reference(torch.from_numpy(golden["y_seq"]) * 1.1 + 0.1, ref)


def test_interleave_rows():
    g = torch.arange(12, dtype=torch.int32).reshape(3, 4)
    u = -g
    r = quant.interleave_rows(g, u)
    assert r.shape == (6, 4)
    assert torch.equal(r[0::2], g) and torch.equal(r[1::2], u)
    with pytest.raises(ValueError):
        quant.interleave_rows(g, u[:2])


def test_stack_rows():
    a = torch.arange(6, dtype=torch.int32).reshape(2, 3)
    b = torch.arange(6, 15, dtype=torch.int32).reshape(3, 3)
    st = quant.stack_rows(a, b)
    assert st.shape == (5, 3) and st.is_contiguous()
    assert torch.equal(st[:2], a) and torch.equal(st[2:], b)
