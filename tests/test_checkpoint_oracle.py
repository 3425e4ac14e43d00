"""The oracle's restatement of the AWQ / GPTQ checkpoint formats, pinned to tensors that an
independent packer (vLLM's awq_pack / gptq_pack / pack_cols) made from weights the reference
quantised (tests/golden/make_checkpoint_golden.py), and the host-side checks of int4gemv.checkpoint.
"""

import numpy as np
import pytest
import torch

import oracle


def bits16(a):
    return np.ascontiguousarray(a).view(np.uint16)


def test_awq_to_packed(checkpoint):
    c = checkpoint
    q, s, z = oracle.awq_to_packed(c["awq_qweight"], c["awq_qzeros"], c["awq_scales"],
                                   int(c["group_size"]))
    np.testing.assert_array_equal(q, c["qweight"])
    np.testing.assert_array_equal(bits16(s), bits16(c["scales"]))
    np.testing.assert_array_equal(z, c["zeros"])  # values: a checkpoint stores no sign of zero


@pytest.mark.parametrize("fmt", ["gptq", "gptq_v2"])
def test_gptq_to_packed(checkpoint, fmt):
    c = checkpoint
    qz = c["gptq_qzeros"] if fmt == "gptq" else c["gptq_v2_qzeros"]
    q, s, z = oracle.gptq_to_packed(c["gptq_qweight"], qz, c["gptq_scales"], int(c["group_size"]),
                                    fmt)
    np.testing.assert_array_equal(q, c["qweight"])
    np.testing.assert_array_equal(bits16(s), bits16(c["scales"]))
    want = c["zeros"].astype(np.float32)
    if fmt == "gptq":  # "gptq" stores z - 1 in four bits: z = 0 comes back as 16
        want = np.where(want == 0, 16, want)
    np.testing.assert_array_equal(z.astype(np.float32), want)
    assert fmt != "gptq" or (z == 16).any()


def test_inverse_packers_match_vllm(checkpoint):
    c = checkpoint
    aq, az, as_ = oracle.packed_to_awq(c["qweight"], c["scales"], c["zeros"])
    np.testing.assert_array_equal(aq, c["awq_qweight"])
    np.testing.assert_array_equal(az, c["awq_qzeros"])
    np.testing.assert_array_equal(bits16(as_), bits16(c["awq_scales"]))
    for fmt, key in (("gptq", "gptq_qzeros"), ("gptq_v2", "gptq_v2_qzeros")):
        gq, gz, _ = oracle.packed_to_gptq(c["qweight"], c["scales"], c["zeros"], fmt)
        np.testing.assert_array_equal(gq, c["gptq_qweight"])
        np.testing.assert_array_equal(gz, c[key])


def test_from_gptq_rejects_act_order_and_unknown_format():
    from int4gemv import checkpoint

    qw = torch.zeros(64, 16, dtype=torch.int32)
    qz = torch.zeros(4, 2, dtype=torch.int32)
    s = torch.ones(4, 16, dtype=torch.float16)
    g_idx = torch.arange(512, dtype=torch.int32).flip(0) // 128
    with pytest.raises(ValueError, match="act-order"):
        checkpoint.from_gptq(qw, qz, s, 128, g_idx=g_idx)
    with pytest.raises(ValueError, match="checkpoint_format"):
        checkpoint.from_gptq(qw, qz, s, 128, checkpoint_format="exl2")
