"""numpy front end of the CPU oracle in w4a16_oracle.c. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only
to check or to time the reference algorithm on the host. The shipped library never calls it.

Each function names the reference code it restates (paths inside Yu-TingLee/int4-GEMV-cuda):
  quantize / pack / unpack / dequantize   int4gemv/quant.py:14-53
  sequential                              csrc/sequential.cpp:11-54 (bit-exact)
  reference                               int4gemv/reference.py:8-10 (double accumulation)
  assert_matches_reference                int4gemv/reference.py:13-22 (the tolerance rule)

Checkpoint formats (not in the reference, whose quant.py:5 only names them): AWQ and GPTQ 4-bit
tensors and their conversion to the reference's layout, restated from the published packers
(AutoAWQ's GEMM layout, order 0 2 4 6 1 3 5 7; AutoGPTQ's QuantLinear.pack, which stores zeros
minus one; as implemented by vLLM 0.22 quantization/utils/quant_utils.py awq_pack / gptq_pack /
pack_cols, which tests/golden/make_checkpoint_golden.py runs to pin these functions).

Arrays are numpy: x float16 [M, K], qweight int32 [N, K/8], scales / zeros float16 [N, K/g].
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libw4a16_oracle.so"
GROUP_SIZE = 128

_lib = None


def build() -> Path:
    """Compile w4a16_oracle.c with the committed Makefile (gcc, a second or two)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        i64, p = ctypes.c_int64, ctypes.c_void_p
        _lib.oracle_unpack.argtypes = [p, p, i64, i64]
        _lib.oracle_pack.argtypes = [p, p, i64, i64]
        _lib.oracle_dequantize.argtypes = [p, p, p, p, i64, i64, i64]
        _lib.oracle_quantize.argtypes = [p, p, p, p, p, i64, i64, i64]
        _lib.oracle_sequential.argtypes = [p, p, p, p, p, i64, i64, i64, i64, p, p, p]
        _lib.oracle_reference.argtypes = [p, p, p, p, p, i64, i64, i64, i64, p]
        for f in (_lib.oracle_unpack, _lib.oracle_pack, _lib.oracle_dequantize,
                  _lib.oracle_quantize, _lib.oracle_sequential, _lib.oracle_reference):
            f.restype = None
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def unpack(qweight: np.ndarray) -> np.ndarray:
    """quant.py:40-44. int32 [N, K/8] -> int32 [N, K] of 4-bit values."""
    qweight = _c(qweight, np.int32)
    n, words = qweight.shape
    q = np.empty((n, words * 8), np.int32)
    lib().oracle_unpack(_ptr(qweight), _ptr(q), n, words * 8)
    return q


def pack(q: np.ndarray) -> np.ndarray:
    """quant.py:32-37. int [N, K] of 4-bit values -> int32 [N, K/8]."""
    q = _c(q, np.int32)
    n, k = q.shape
    out = np.empty((n, k // 8), np.int32)
    lib().oracle_pack(_ptr(q), _ptr(out), n, k)
    return out


def dequantize(qweight, scales, zeros, group_size: int = GROUP_SIZE) -> np.ndarray:
    """quant.py:47-53. float32 [N, K], bit-exact with the reference."""
    qweight, scales, zeros = _c(qweight, np.int32), _c(scales, np.float16), _c(zeros, np.float16)
    n = qweight.shape[0]
    k = qweight.shape[1] * 8
    w = np.empty((n, k), np.float32)
    lib().oracle_dequantize(_ptr(qweight), _ptr(scales), _ptr(zeros), _ptr(w), n, k, group_size)
    return w


def quantize(w: np.ndarray, group_size: int = GROUP_SIZE):
    """quant.py:14-29. float [N, K] -> (qweight int32, scales float16, zeros float16), bit-exact."""
    w = _c(w, np.float32)
    n, k = w.shape
    assert k % group_size == 0 and group_size % 8 == 0, (k, group_size)
    qweight = np.empty((n, k // 8), np.int32)
    scales = np.empty((n, k // group_size), np.float16)
    zeros = np.empty((n, k // group_size), np.float16)
    scratch = np.empty((n, k), np.int32)
    lib().oracle_quantize(_ptr(w), _ptr(qweight), _ptr(scales), _ptr(zeros), _ptr(scratch), n, k,
                          group_size)
    return qweight, scales, zeros


def sequential(x, qweight, scales, zeros, group_size: int = GROUP_SIZE) -> np.ndarray:
    """csrc/sequential.cpp:11-54, bit-exact. Returns float16 [M, N]."""
    x = _c(x, np.float16)
    qweight, scales, zeros = _c(qweight, np.int32), _c(scales, np.float16), _c(zeros, np.float16)
    m, k = x.shape
    n = qweight.shape[0]
    y = np.empty((m, n), np.float16)
    if m == 0 or n == 0:
        return y
    xs = np.empty((m, k), np.float32)
    ws = np.empty(group_size, np.float32)
    acc = np.empty(max(m, 1), np.float32)
    lib().oracle_sequential(_ptr(x), _ptr(qweight), _ptr(scales), _ptr(zeros), _ptr(y), m, n, k,
                            group_size, _ptr(xs), _ptr(ws), _ptr(acc))
    return y


def reference(x, qweight, scales, zeros, group_size: int = GROUP_SIZE) -> np.ndarray:
    """reference.py:8-10 with double accumulation. Returns float32 [M, N]."""
    x = _c(x, np.float16)
    qweight, scales, zeros = _c(qweight, np.int32), _c(scales, np.float16), _c(zeros, np.float16)
    m, k = x.shape
    n = qweight.shape[0]
    y = np.empty((m, n), np.float32)
    if m == 0 or n == 0:
        return y
    ws = np.empty(k, np.float32)
    lib().oracle_reference(_ptr(x), _ptr(qweight), _ptr(scales), _ptr(zeros), _ptr(y), m, n, k,
                           group_size, _ptr(ws))
    return y


def rms(ref: np.ndarray) -> float:
    ref = np.asarray(ref, np.float64)
    return float(np.sqrt(np.sum(ref * ref) / max(ref.size, 1)))


def check_close(y, ref, rtol: float = 1e-2, atol: float = 1e-2) -> tuple[bool, str]:
    """The parity rule for a fp16 GEMV output against the fp32 oracle.

    reference.py:13-22 allows |y - ref| <= atol_ref + rtol * |ref| with atol_ref = 1e-2 * rms(ref)
    and rtol = 1e-2. The tier's own bar is rtol = 1e-2, atol = 1e-2 absolute. Both must hold, so
    the absolute term used is min(1e-2 * rms, atol).
    """
    y = np.asarray(y, np.float32)
    ref = np.asarray(ref, np.float32)
    if y.shape != ref.shape:
        return False, f"shape {y.shape} != {ref.shape}"
    if y.size == 0:
        return True, "empty"
    a = min(1e-2 * rms(ref), atol)
    err = np.abs(y.astype(np.float64) - ref)
    bound = a + rtol * np.abs(ref.astype(np.float64))
    bad = ~(err <= bound)
    if bad.any():
        i = np.unravel_index(int(np.argmax(np.where(bad, err - bound, -np.inf))), y.shape)
        return False, (f"{int(bad.sum())} of {y.size} outside atol={a:.3g} rtol={rtol}: at {i} "
                       f"got {y[i]} want {ref[i]}")
    return True, f"max |err| {float(err.max()):.3g}, atol {a:.3g}"


def assert_matches_reference(y, ref, rtol: float = 1e-2, atol: float = 1e-2) -> None:
    ok, msg = check_close(y, ref, rtol, atol)
    assert ok, msg


def synthetic(m: int, n: int, k: int, group_size: int = GROUP_SIZE, seed: int = 0,
              w_std: float = 0.02):
    """Seeded inputs with the distributions the benchmark configs name: weights N(0, w_std) RTN
    group-quantised, activations N(0, 1) rounded to fp16. numpy generator, so no torch needed."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(w_std)).astype(np.float32)
    x = rng.standard_normal((m, k), dtype=np.float32).astype(np.float16)
    qweight, scales, zeros = quantize(w, group_size)
    return x, qweight, scales, zeros


# ---------------------------------------------------------------- AWQ / GPTQ checkpoint formats
AWQ_ORDER = np.array([0, 2, 4, 6, 1, 3, 5, 7])  # nibble i of an AWQ word holds column AWQ_ORDER[i]
GPTQ_ZERO_OFFSET = {"gptq": 1, "gptq_v2": 0}


def _nibbles(words: np.ndarray) -> np.ndarray:
    """int32 [..., W] -> int32 [..., W, 8], element i = nibble i (bits 4i .. 4i + 3)."""
    u = words.astype(np.uint32)[..., None] >> (np.arange(8, dtype=np.uint32) * 4)
    return (u & 0xF).astype(np.int32)


def _pack_nibbles(nib: np.ndarray) -> np.ndarray:
    """int [..., W, 8] of 0..15 -> int32 [..., W], element i in nibble i."""
    words = (nib.astype(np.uint32) << (np.arange(8, dtype=np.uint32) * 4)).sum(-1, dtype=np.uint64)
    return (words & 0xFFFFFFFF).astype(np.uint32).view(np.int32)


def awq_unpack(words: np.ndarray) -> np.ndarray:
    """AWQ-packed [R, C/8] -> values [R, C] by column (column AWQ_ORDER[i] <- nibble i)."""
    nib = _nibbles(words)
    cols = np.empty_like(nib)
    cols[..., AWQ_ORDER] = nib
    return cols.reshape(words.shape[0], -1)


def awq_pack(values: np.ndarray) -> np.ndarray:
    """values [R, C] (0..15) -> AWQ-packed [R, C/8]."""
    r, c = values.shape
    return _pack_nibbles(values.reshape(r, c // 8, 8)[..., AWQ_ORDER])


def awq_to_packed(qweight, qzeros, scales, group_size: int = GROUP_SIZE):
    """AWQ (qweight [K, N/8], qzeros [K/g, N/8], scales [K/g, N]) -> (qweight [N, K/8] int32,
    scales [N, K/g] float16, zeros [N, K/g] float16) of the reference's layout."""
    q = awq_unpack(np.asarray(qweight))  # [K, N]
    z = awq_unpack(np.asarray(qzeros))   # [K/g, N]
    return (pack(np.ascontiguousarray(q.T)), np.ascontiguousarray(np.asarray(scales).T),
            np.ascontiguousarray(z.T).astype(np.float16))


def packed_to_awq(qweight, scales, zeros):
    """The inverse of awq_to_packed for integer zeros 0..15."""
    q = unpack(qweight)  # [N, K]
    return (awq_pack(np.ascontiguousarray(q.T)),
            awq_pack(np.ascontiguousarray(zeros.T).astype(np.int32)),
            np.ascontiguousarray(np.asarray(scales).T))


def gptq_to_packed(qweight, qzeros, scales, group_size: int = GROUP_SIZE,
                   checkpoint_format: str = "gptq"):
    """GPTQ (qweight [K/8, N] packed along K, qzeros [K/g, N/8] packed along N in order and stored
    minus GPTQ_ZERO_OFFSET[format], scales [K/g, N]) -> the reference's layout."""
    qweight = np.asarray(qweight)
    nib = _nibbles(qweight)                                   # [K/8, N, 8]: q[8r + i, n]
    q = nib.transpose(0, 2, 1).reshape(-1, qweight.shape[1])  # [K, N]
    z = _nibbles(np.asarray(qzeros)).reshape(qzeros.shape[0], -1) + GPTQ_ZERO_OFFSET[
        checkpoint_format]
    return (pack(np.ascontiguousarray(q.T)), np.ascontiguousarray(np.asarray(scales).T),
            np.ascontiguousarray(z.T).astype(np.float16))


def packed_to_gptq(qweight, scales, zeros, checkpoint_format: str = "gptq"):
    """The inverse of gptq_to_packed for integer zeros (0..15 for "gptq_v2", 1..16 for "gptq")."""
    q = unpack(qweight).T                                      # [K, N]
    k, n = q.shape
    qw = _pack_nibbles(q.reshape(k // 8, 8, n).transpose(0, 2, 1))
    zs = np.ascontiguousarray(zeros.T).astype(np.int32) - GPTQ_ZERO_OFFSET[checkpoint_format]
    qz = _pack_nibbles((zs & 0xF).reshape(zs.shape[0], -1, 8))
    return qw, qz, np.ascontiguousarray(np.asarray(scales).T)
