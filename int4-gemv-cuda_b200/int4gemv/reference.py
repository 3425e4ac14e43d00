"""The fp32 reference and the tolerance rule every kernel must meet.

Same API and rule as the reference's int4gemv/reference.py:8-22: the reference result is
x.float() @ dequantize(W).T in fp32, and an fp16 kernel output passes if
|y - ref| <= 1e-2 * rms(ref) + 1e-2 * |ref| elementwise.
"""

from __future__ import annotations

import torch

from int4gemv.quant import dequantize


def w4a16_reference(x, qweight, scales, zeros, group_size: int) -> torch.Tensor:
    """x [M, K] @ dequant(W).T in fp32, shape [M, N]."""
    return x.float() @ dequantize(qweight, scales, zeros, group_size).T


def assert_matches_reference(y: torch.Tensor, ref: torch.Tensor) -> None:
    """Check a kernel's fp16 output against the fp32 reference (1% relative, 1% of RMS absolute).

    RMS rather than std: std is NaN for a single output and 0 when all outputs are equal.
    """
    assert y.dtype == torch.float16 and y.shape == ref.shape, (y.dtype, y.shape, ref.shape)
    rms = torch.linalg.vector_norm(ref.float()).item() / max(ref.numel(), 1) ** 0.5
    torch.testing.assert_close(y.float().cpu(), ref.float().cpu(), rtol=1e-2, atol=1e-2 * rms)
