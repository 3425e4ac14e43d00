"""The CPU oracle (oracle/w4a16_oracle.c) pinned to golden vectors the reference produced.

tests/golden/make_golden.py recorded, from the reference itself: quantize / dequantize
(int4gemv/quant.py), the fp32 reference (int4gemv/reference.py) and the compiled CPU path
(csrc/sequential.cpp). The oracle must be bit-exact with all but the fp32 matmul, whose
summation order is BLAS-specific; against that it must agree to ~1e-6 relative.
"""

import numpy as np
import pytest

import oracle


def bits16(a):
    return np.ascontiguousarray(a).view(np.uint16)


def test_quantize_bit_exact(golden):
    if "w" not in golden:
        pytest.skip("case stores no float weights")
    g = int(golden["group_size"])
    q, s, z = oracle.quantize(golden["w"], g)
    np.testing.assert_array_equal(q, golden["qweight"])
    np.testing.assert_array_equal(bits16(s), bits16(golden["scales"]))
    # bitwise, including the -0.0 zero points quantize produces for all-positive groups
    np.testing.assert_array_equal(bits16(z), bits16(golden["zeros"]))


def test_unpack_pack_round_trip(golden):
    q = oracle.unpack(golden["qweight"])
    assert q.min() >= 0 and q.max() <= 15
    np.testing.assert_array_equal(oracle.pack(q), golden["qweight"])


def test_pack_wraps_like_reference(pack_wrap):
    np.testing.assert_array_equal(oracle.pack(pack_wrap["q"]), pack_wrap["qweight"])


def test_dequantize_bit_exact(golden):
    if "deq" not in golden:
        pytest.skip("case stores no dequantized weights")
    g = int(golden["group_size"])
    w = oracle.dequantize(golden["qweight"], golden["scales"], golden["zeros"], g)
    np.testing.assert_array_equal(w.view(np.uint32), golden["deq"].view(np.uint32))


def test_sequential_bit_exact(golden):
    g = int(golden["group_size"])
    y = oracle.sequential(golden["x"], golden["qweight"], golden["scales"], golden["zeros"], g)
    np.testing.assert_array_equal(bits16(y), bits16(golden["y_seq"]))


def test_reference_matches_torch_fp32(golden):
    g = int(golden["group_size"])
    y = oracle.reference(golden["x"], golden["qweight"], golden["scales"], golden["zeros"], g)
    ref = golden["y_ref"]
    scale = max(oracle.rms(ref), 1e-30)
    assert np.max(np.abs(y - ref)) <= 1e-5 * scale + 1e-5 * np.max(np.abs(ref))


def test_reference_sequential_within_tolerance(golden):
    """The reference's own CPU path meets the tolerance rule against the fp32 reference."""
    ok, msg = oracle.check_close(golden["y_seq"], golden["y_ref"])
    assert ok, msg


def test_check_close_catches_a_planted_error():
    x, q, s, z = oracle.synthetic(2, 64, 256, 128, seed=3)
    ref = oracle.reference(x, q, s, z)
    y = ref.astype(np.float16)
    assert oracle.check_close(y, ref)[0]
    bad = y.copy()
    bad[1, 7] = np.float16(float(bad[1, 7]) * 1.05 + 0.05)
    assert not oracle.check_close(bad, ref)[0]


def test_config0_cpu_case():
    """BASELINE config 0 (N = K = 4096, M = 1) runs on the CPU oracle: sequential vs reference."""
    x, q, s, z = oracle.synthetic(1, 4096, 4096, 128, seed=0)
    y = oracle.sequential(x, q, s, z)
    ref = oracle.reference(x, q, s, z)
    ok, msg = oracle.check_close(y, ref)
    assert ok, msg
