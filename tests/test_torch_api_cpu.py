"""The torch API (int4gemv.ops) on the CPU: names, defaults, the CPU path, and the reference's
input checks with the same messages. Where the reference itself is built (oracle/_ref), its own
check_inputs is run on the same bad inputs and the messages compared verbatim."""

import importlib.util
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from int4gemv import ops

REF_SO = sorted((Path(__file__).resolve().parents[1] / "oracle" / "_ref").glob("int4gemv_ref*.so"))


def ref_module():
    if not REF_SO:
        return None
    spec = importlib.util.spec_from_file_location("int4gemv_ref", REF_SO[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def tensors(case):
    return [torch.from_numpy(np.ascontiguousarray(case[k])) for k in ("x", "qweight", "scales", "zeros")]


def test_api_surface():
    for name in ("sequential", "naive", "coalesced", "vectorized", "load_only"):
        assert callable(getattr(ops, name))
    assert list(ops.KERNELS)[:3] == ["naive", "coalesced", "vectorized"]
    assert set(ops.KERNEL_INFO) >= {"naive", "coalesced", "vectorized"}
    for fn in (ops.vectorized, ops.load_only, ops.int4gemv_ops.vectorized_info):
        assert re.search(r"threads_per_block: [\w.]+ = 128", fn.__doc__), fn.__doc__
        assert re.search(r"rows_per_warp: [\w.]+ = 2", fn.__doc__), fn.__doc__


def test_sequential_bit_exact(golden):
    y = ops.sequential(*tensors(golden), int(golden["group_size"]))
    assert y.dtype == torch.float16 and y.shape == golden["y_seq"].shape
    np.testing.assert_array_equal(y.numpy().view(np.uint16), golden["y_seq"].view(np.uint16))


def test_sequential_empty():
    x = torch.zeros(0, 256, dtype=torch.float16)
    q = torch.zeros(4, 32, dtype=torch.int32)
    s = torch.ones(4, 2, dtype=torch.float16)
    assert ops.sequential(x, q, s, s, 128).shape == (0, 4)
    x = torch.zeros(2, 0, dtype=torch.float16)
    y = ops.sequential(x, torch.zeros(4, 0, dtype=torch.int32), torch.zeros(4, 0, dtype=torch.float16),
                       torch.zeros(4, 0, dtype=torch.float16), 128)
    assert y.shape == (2, 4) and (y == 0).all()


def bad_inputs():
    """(label, args, expected message or None). Expected messages are the reference's format
    (csrc/checks.cpp:22-35) for the cases where the reference build here cannot be asked: its
    compiled check_inputs crashes (SIGSEGV) while formatting integer sizes under torch 2.11."""
    x = torch.zeros(2, 256, dtype=torch.float16)
    q = torch.zeros(8, 32, dtype=torch.int32)
    s = torch.zeros(8, 2, dtype=torch.float16)
    return [
        ("dtype", (x.float(), q, s, s, 128), None),
        ("rank", (x[None], q, s, s, 128), None),
        ("group", (x, q, s, s, 100),
         "group_size 100 must be a positive multiple of 8 dividing K = 256"),
        ("group0", (x, q, s, s, 0), "group_size 0 must be a positive multiple of 8 dividing K = 256"),
        ("pack", (x, q[:, :16], s, s, 128), "qweight of shape [8, 16] does not pack K = 256"),
        ("scales", (x, q, s[:, :1], s[:, :1], 128), "scales [8, 1] and zeros [8, 1] must be [8, 2]"),
        ("zeros", (x, q, s, s[:4], 128), "scales [8, 2] and zeros [4, 2] must be [8, 2]"),
        ("contig", (x, torch.zeros(32, 8, dtype=torch.int32).T, s, s, 128), None),
    ]


@pytest.mark.parametrize("label,args,expected", bad_inputs(), ids=[b[0] for b in bad_inputs()])
def test_check_messages_match_reference(label, args, expected):
    with pytest.raises(RuntimeError) as mine:
        ops.sequential(*args)
    text = str(mine.value).splitlines()[0]
    assert text.startswith("sequential: ")
    if expected is not None:
        assert text == "sequential: " + expected
        return
    ref = ref_module()
    if ref is None:
        pytest.skip("reference not built here (oracle/_ref)")
    with pytest.raises(RuntimeError) as theirs:
        ref.check_inputs(*args, cuda=False)
    assert text.replace("sequential: ", "check: ", 1) == str(theirs.value).splitlines()[0]


def test_cuda_op_rejects_cpu_tensors():
    x = torch.zeros(1, 256, dtype=torch.float16)
    q = torch.zeros(8, 32, dtype=torch.int32)
    s = torch.zeros(8, 2, dtype=torch.float16)
    for name in ("naive", "coalesced", "vectorized", "w4a16", "load_only"):
        with pytest.raises(RuntimeError) as e:
            getattr(ops, name)(x, q, s, s, 128)
        assert str(e.value).splitlines()[0] == (
            f"{name}: expected all inputs on one cuda device, got cpu and cpu")


def test_new_ops_reject_cpu_tensors():
    """The B200 additions refuse CPU tensors with a clear message (no CPU fallback)."""
    x = torch.zeros(1, 1024, dtype=torch.float16)
    q = torch.zeros(8, 128, dtype=torch.int32)
    s = torch.zeros(8, 8, dtype=torch.float16)
    for call in (lambda: ops.w4a16_silu_mul(x, q, s, s, 128),
                 lambda: ops.w4a16_bias_residual(x, q, s, s, 128),
                 lambda: ops.w4a16_grouped(x, q, s, s, 128, [8])):
        with pytest.raises(RuntimeError, match="cuda"):
            call()
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quantize(torch.zeros(8, 1024), 128)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.pack(torch.zeros(8, 1024, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.repack_gptq(torch.zeros(128, 8, dtype=torch.int32), torch.zeros(8, 1, dtype=torch.int32),
                        torch.zeros(8, 8, dtype=torch.float16), 128)
