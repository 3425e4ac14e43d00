"""Round-to-nearest 4-bit group quantisation in the packed format the kernels read.

Same contract as the reference's int4gemv/quant.py:5-53, bit for bit (pinned by the tests against
golden vectors the reference produced): per group of `group_size` weights along K, the range
[min, max] widened to include 0 is spread over the levels 0..15; the scale is rounded to fp16
before q is computed; q and the zero point are rounded half to even; eight 4-bit q are packed per
int32 with weight k in bits 4 (k % 8) .. 4 (k % 8) + 3 of word k // 8.
"""

from __future__ import annotations

import torch

GROUP_SIZE = 128  # weights per scale and zero, as in AWQ and GPTQ checkpoints
_NIBBLE_SHIFTS = tuple(range(0, 32, 4))


def bits_per_weight(group_size: int = GROUP_SIZE) -> float:
    """4 bits per weight plus one fp16 scale and one fp16 zero per group."""
    return 4.0 + 32.0 / group_size


def quantize(w: torch.Tensor, group_size: int = GROUP_SIZE):
    """w [N, K] -> (qweight [N, K/8] int32, scales [N, K/g] fp16, zeros [N, K/g] fp16).

    A CUDA tensor is quantised on its device by the compiled kernel (ops.quantize), which reads
    fp32, fp16 and bf16 as they are; other dtypes are widened to fp32 first, as the reference does.
    """
    n, k = w.shape
    assert k % group_size == 0 and group_size % 8 == 0, (k, group_size)
    if w.is_cuda:
        from . import ops

        if w.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            w = w.float()
        return ops.quantize(w.contiguous(), group_size)
    groups = w.float().reshape(n, k // group_size, group_size)
    lo, hi = torch.aminmax(groups, dim=-1, keepdim=True)
    lo = torch.clamp(lo, max=0.0)
    hi = torch.clamp(hi, min=0.0)
    # q is computed with the fp16-rounded scale, the one the kernels read back.
    scale = torch.clamp((hi - lo) / 15, min=1e-6).to(torch.float16).to(torch.float32)
    zero = torch.clamp(torch.round(-lo / scale), 0, 15)
    q = torch.clamp(torch.round(groups / scale + zero), 0, 15).to(torch.int32).reshape(n, k)
    return pack(q), scale.squeeze(-1).to(torch.float16), zero.squeeze(-1).to(torch.float16)


def pack(q: torch.Tensor) -> torch.Tensor:
    """q [N, K] of values 0..15 -> [N, K/8] int32, lowest nibble = lowest k.

    word = sum_j q[8w + j] << 4j modulo 2^32, like the reference's int64 sum and int32 cast: values
    outside 0..15 are not masked and carry into the neighbouring nibbles."""
    n, k = q.shape
    parts = q.to(torch.int64).reshape(n, k // 8, 8)
    word = torch.zeros(n, k // 8, dtype=torch.int64, device=q.device)
    for j, shift in enumerate(_NIBBLE_SHIFTS):
        word += parts[..., j] << shift
    # keep the low 32 bits, then reinterpret them as int32 (torch has no uint32 arithmetic)
    word = word & 0xFFFFFFFF
    word = torch.where(word >= 2**31, word - 2**32, word)
    return word.to(torch.int32)


def unpack(qweight: torch.Tensor) -> torch.Tensor:
    """qweight [N, K/8] int32 -> 4-bit values [N, K] int32."""
    n, words = qweight.shape
    shifts = torch.tensor(_NIBBLE_SHIFTS, dtype=torch.int32, device=qweight.device)
    return ((qweight.unsqueeze(-1) >> shifts) & 0xF).reshape(n, words * 8)


def dequantize(qweight, scales, zeros, group_size: int) -> torch.Tensor:
    """The fp32 weights [N, K] the packed format stands for: (q - z) * s."""
    q = unpack(qweight).to(torch.float32)
    n, k = q.shape
    q = q.reshape(n, k // group_size, group_size)
    w = (q - zeros.to(torch.float32).unsqueeze(-1)) * scales.to(torch.float32).unsqueeze(-1)
    return w.reshape(n, k)


def interleave_rows(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Row i of gate -> row 2i, row i of up -> row 2i + 1 (any of qweight, scales, zeros): the
    layout ops.w4a16_silu_mul reads, so one weight stream feeds both projections."""
    if gate.shape != up.shape:
        raise ValueError(f"gate and up shapes differ: {tuple(gate.shape)} vs {tuple(up.shape)}")
    return torch.stack((gate, up), dim=1).reshape(2 * gate.shape[0], *gate.shape[1:]).contiguous()


def stack_rows(*tensors: torch.Tensor) -> torch.Tensor:
    """The matrices' rows one after another (any of qweight, scales, zeros): the stacked layout
    ops.w4a16_grouped reads, built once at load time."""
    return torch.cat(tensors, dim=0).contiguous()
