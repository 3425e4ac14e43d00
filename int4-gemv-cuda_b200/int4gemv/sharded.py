"""The W4A16 GEMV sharded over the ranks of a torch.distributed process group (one GPU per rank).

Two layouts, each with one exchange step per call:

- N-split ("up" projections, e.g. 28672 x 8192): rank r holds rows [n0, n1) of qweight, scales and
  zeros, x is replicated, the local GEMV gives y[:, n0:n1], and an all-gather assembles y on every
  rank.
- K-split ("down" projections, e.g. 8192 x 28672): rank r holds columns [k0, k1) of the weights
  (k0, k1 multiples of the group size, so every rank owns whole groups and whole packed words) and
  the same slice of x; the local GEMV gives the partial y as fp32 row sums (`ops.w4a16_f32`, never
  rounded to fp16), which an fp32 all-reduce adds across ranks before the one rounding to fp16.

The local GEMVs are `ops.w4a16` (rows split) and `ops.w4a16_f32` (K split), the CUDA fast path,
unless the caller passes other callables with the same signatures: there is no CPU fallback in the
product path.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

LocalGemv = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, int], torch.Tensor]


def split_range(total: int, parts: int, index: int, align: int = 1) -> tuple[int, int]:
    """[begin, end) of part `index` when `total` (a multiple of `align`) is cut into `parts` pieces
    of whole `align` units, as equal as possible; earlier parts take the remainder."""
    if total % align:
        raise ValueError(f"total {total} is not a multiple of {align}")
    units = total // align
    base, extra = divmod(units, parts)
    begin = index * base + min(index, extra)
    end = begin + base + (1 if index < extra else 0)
    return begin * align, end * align


def shard_rows(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, rank: int,
               world: int):
    """Rows [n0, n1) of the packed weights for N-split rank `rank`."""
    n0, n1 = split_range(qweight.shape[0], world, rank)
    return (qweight[n0:n1].contiguous(), scales[n0:n1].contiguous(), zeros[n0:n1].contiguous(),
            (n0, n1))


def shard_cols(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, group_size: int,
               rank: int, world: int):
    """Columns [k0, k1) (whole groups) of the packed weights for K-split rank `rank`."""
    k = qweight.shape[1] * 8
    k0, k1 = split_range(k, world, rank, group_size)
    return (qweight[:, k0 // 8:k1 // 8].contiguous(),
            scales[:, k0 // group_size:k1 // group_size].contiguous(),
            zeros[:, k0 // group_size:k1 // group_size].contiguous(), (k0, k1))


def _default_gemv() -> LocalGemv:
    from . import ops

    return ops.w4a16


def _default_partial() -> LocalGemv:
    from . import ops

    return ops.w4a16_f32


class ShardedW4A16:
    """One weight matrix sharded over a process group; calling it with the full x returns the full
    y on every rank.

    mode "n": N-split + all-gather. mode "k": K-split + fp32 all-reduce. The constructor takes the
    full packed tensors (as every rank would load them) and keeps only this rank's shard.
    local_gemv (rows split) returns fp16 y; local_partial (K split) returns the fp32 row sums.
    """

    def __init__(self, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                 group_size: int, mode: str, process_group=None,
                 local_gemv: LocalGemv | None = None, local_partial: LocalGemv | None = None):
        if mode not in ("n", "k"):
            raise ValueError(f"mode must be 'n' or 'k', got {mode!r}")
        self.mode = mode
        self.group_size = int(group_size)
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.n = qweight.shape[0]
        self.k = qweight.shape[1] * 8
        self.gemv = local_gemv or _default_gemv()
        self.partial = local_partial or _default_partial()
        if mode == "n":
            self.q, self.s, self.z, self.span = shard_rows(qweight, scales, zeros, self.rank,
                                                           self.world)
            self.max_rows = split_range(self.n, self.world, 0)[1]
        else:
            if self.k % self.group_size:
                raise ValueError("K must be a multiple of group_size")
            self.q, self.s, self.z, self.span = shard_cols(qweight, scales, zeros,
                                                           self.group_size, self.rank, self.world)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != self.k:
            raise ValueError(f"x must be [M, {self.k}], got {tuple(x.shape)}")
        m = x.shape[0]
        if self.mode == "n":
            y_local = self.gemv(x, self.q, self.s, self.z, self.group_size)
            # Shards differ by at most one row: gather into equal padded slots, then trim.
            slot = torch.zeros(m, self.max_rows, dtype=y_local.dtype, device=y_local.device)
            slot[:, :y_local.shape[1]] = y_local
            gathered = torch.empty(self.world * m, self.max_rows, dtype=slot.dtype,
                                   device=slot.device)
            dist.all_gather_into_tensor(gathered, slot, group=self.pg)
            gathered = gathered.view(self.world, m, self.max_rows)
            parts = []
            for r in range(self.world):
                n0, n1 = split_range(self.n, self.world, r)
                parts.append(gathered[r, :, :n1 - n0])
            return torch.cat(parts, dim=1)
        k0, k1 = self.span
        if k1 > k0:
            partial = self.partial(x[:, k0:k1].contiguous(), self.q, self.s, self.z,
                                   self.group_size)
            if partial.dtype != torch.float32:
                raise TypeError(f"local_partial must return float32, got {partial.dtype}")
        else:
            partial = torch.zeros(m, self.n, dtype=torch.float32, device=x.device)
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.pg)
        return partial.half()
