"""AWQ and GPTQ 4-bit checkpoints -> this library's packed layout, on the device.

The reference quantises unquantised fp16 / bf16 weights itself (int4gemv/quant.py:5 names AWQ and
GPTQ only as the origin of group size 128); this module lets a user load an already quantised
checkpoint instead. Both formats dequantise as (q - z) * s per group, like quant.py, so repacking
is exact bit movement (ops.repack_awq / ops.repack_gptq, the CUDA kernels of csrc/repack.cu):

- AWQ (AutoAWQ, GEMM layout): qweight [K, N/8] int32 and qzeros [K/g, N/8] int32 pack eight
  output columns per word in the order 0 2 4 6 1 3 5 7; scales [K/g, N] fp16.
- GPTQ (AutoGPTQ / GPTQModel): qweight [K/8, N] int32 packs eight consecutive k per word;
  qzeros [K/g, N/8] int32 packs eight columns per word in order; scales [K/g, N] fp16. The
  original "gptq" checkpoint format stores z - 1 in qzeros (so a stored 15 means z = 16, which the
  fp16 zeros of this layout hold exactly); "gptq_v2" stores z.

Act-order GPTQ checkpoints (a g_idx that is not k // group_size) group non-contiguous k and would
need x permuted on every call; they are rejected.
"""

from __future__ import annotations

import torch

from . import ops

GPTQ_ZERO_OFFSET = {"gptq": 1, "gptq_v2": 0}


def from_awq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
             group_size: int = 128):
    """AWQ tensors (CUDA) -> (qweight [N, K/8] int32, scales [N, K/g] fp16, zeros [N, K/g] fp16)."""
    return ops.repack_awq(qweight.contiguous(), qzeros.contiguous(),
                          scales.to(torch.float16).contiguous(), group_size)


def from_gptq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
              group_size: int = 128, g_idx: torch.Tensor | None = None,
              checkpoint_format: str = "gptq"):
    """GPTQ tensors (CUDA) -> (qweight [N, K/8] int32, scales [N, K/g] fp16, zeros [N, K/g] fp16).

    checkpoint_format "gptq" (zeros stored minus one) or "gptq_v2" (zeros stored as they are).
    """
    if checkpoint_format not in GPTQ_ZERO_OFFSET:
        raise ValueError(f"checkpoint_format must be one of {sorted(GPTQ_ZERO_OFFSET)}, "
                         f"got {checkpoint_format!r}")
    k = qweight.shape[0] * 8
    if g_idx is not None:
        expect = torch.arange(k, device=g_idx.device, dtype=g_idx.dtype) // group_size
        if g_idx.shape != (k,) or not torch.equal(g_idx, expect):
            raise ValueError("g_idx is not k // group_size (act-order checkpoint): groups are not "
                             "contiguous along K, which this layout requires")
    return ops.repack_gptq(qweight.contiguous(), qzeros.contiguous(),
                           scales.to(torch.float16).contiguous(), group_size,
                           GPTQ_ZERO_OFFSET[checkpoint_format])
