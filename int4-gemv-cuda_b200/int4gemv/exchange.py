"""A W4A16 layer sharded over the GPUs of one node with the exchange fused into the GEMV kernel.

Same two layouts as int4gemv.sharded (rows split with an all-gather of y; K split with a sum of
the partial y), but instead of a NCCL collective after the GEMV, the GEMV's own epilogue writes
its outputs straight into the other ranks' buffers over NVLink (peer stores into CUDA-IPC-mapped
memory), each output tagged with the call number in the same 8-byte store, and each CTA reads the
words its counterparts on the other ranks wrote as their tags arrive (bounded waits; no fence and
no separate flag; int4gemv_w4a16_exchange in the C ABI). One kernel per call, no collective launch, and the exchange
of a CTA's rows overlaps the other CTAs' weight streaming.

Buffers: each rank allocates one exchange buffer with two halves, used by alternate calls (a rank
can run at most one call ahead of the slowest one), and a call counter in device memory, so a call
needs no host-side state and can be captured in a CUDA graph and replayed. The handles travel over the process group once, at
construction. Each call returns a new y tensor.

Constraints: the fast path's shapes (group 128, the rank's K a multiple of 1024, M <= 32); rows
split needs N % world == 0 (equal shards, so a rank knows where every other rank's columns go); K
split cuts K in whole 1024-weight stages, as evenly as they go (28672 over 8 ranks: 4 ranks of
4096, 4 of 3072); at most 8 ranks; every rank makes the same calls in the same order.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import capi
from .sharded import split_range

_STAGE_K = 1024


class PeerBuffer:
    """`nbytes` of zeroed device memory on every rank of `group`, mapped into every rank."""

    def __init__(self, nbytes: int, group=None):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        lib = capi.lib()
        local = ctypes.c_void_p()
        handle = (ctypes.c_char * capi.IPC_HANDLE_BYTES)()
        capi.check(lib.int4gemv_peer_alloc(nbytes, ctypes.byref(local), ctypes.addressof(handle)))
        self.local = local.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.local)
                continue
            mapped = ctypes.c_void_p()
            buf = (ctypes.c_char * capi.IPC_HANDLE_BYTES).from_buffer_copy(h)
            capi.check(lib.int4gemv_peer_open(ctypes.addressof(buf), ctypes.byref(mapped)))
            self.ptrs.append(mapped.value)

    def close(self) -> None:
        if not self.ptrs:
            return
        lib = capi.lib()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                capi.check(lib.int4gemv_peer_close(p))
        capi.check(lib.int4gemv_peer_free(self.local))
        self.ptrs = []


class FusedShardedW4A16:
    """One weight matrix sharded over a process group; calling it with the full x returns the full
    y on every rank, the exchange done inside the GEMV kernel.

    mode "n": rows split (up projections, N % world == 0). mode "k": K split (down projections).
    The constructor takes the full packed tensors (as every rank would load them), keeps this
    rank's shard and sets up the peer buffers for inputs of up to `max_m` rows. Call close()
    (on every rank) to release them.
    """

    def __init__(self, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                 group_size: int, mode: str, process_group=None, max_m: int = 32):
        if mode not in ("n", "k"):
            raise ValueError(f"mode must be 'n' or 'k', got {mode!r}")
        self.mode, self.group_size, self.pg, self.max_m = mode, int(group_size), process_group, max_m
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        if self.world > capi.MAX_PEERS:
            raise ValueError(f"at most {capi.MAX_PEERS} ranks, got {self.world}")
        self.n = qweight.shape[0]
        self.k = qweight.shape[1] * 8
        if mode == "n":
            if self.n % self.world:
                raise ValueError(f"N = {self.n} must be a multiple of the world size {self.world}")
            n0, n1 = split_range(self.n, self.world, self.rank)
            self.q, self.s, self.z = (t[n0:n1].contiguous() for t in (qweight, scales, zeros))
            self.span = (n0, n1)
            half_bytes = max_m * self.n * 8  # one 8-byte tagged word per output
        else:
            if self.k % _STAGE_K or self.k < _STAGE_K * self.world:
                raise ValueError(f"K = {self.k} must be a multiple of {_STAGE_K} and at least "
                                 f"{_STAGE_K} x world ({self.world})")
            k0, k1 = split_range(self.k, self.world, self.rank, _STAGE_K)
            g = self.group_size
            self.q = qweight[:, k0 // 8:k1 // 8].contiguous()
            self.s = scales[:, k0 // g:k1 // g].contiguous()
            self.z = zeros[:, k0 // g:k1 // g].contiguous()
            self.span = (k0, k1)
            half_bytes = self.world * max_m * self.n * 8
        self.out_bytes = 2 * half_bytes
        self.out = PeerBuffer(self.out_bytes, process_group)
        self.counters = ctypes.c_void_p()
        handle = (ctypes.c_char * capi.IPC_HANDLE_BYTES)()
        capi.check(capi.lib().int4gemv_peer_alloc(capi.PEER_COUNTER_BYTES,
                                                  ctypes.byref(self.counters),
                                                  ctypes.addressof(handle)))
        self.peers = capi.Peers()
        self.peers.world, self.peers.rank = self.world, self.rank
        self.peers.out_bytes = self.out_bytes
        for r in range(self.world):
            self.peers.out[r] = self.out.ptrs[r]
        self.peers.counters = self.counters.value
        if mode == "n":
            self.peers.mode, self.peers.n_total = capi.SHARD_ROWS, self.n
            self.peers.col0 = self.span[0]
        else:
            self.peers.mode = capi.SHARD_K

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.pg)  # no rank still writes into another's buffers
        self.out.close()
        capi.check(capi.lib().int4gemv_peer_free(self.counters.value))

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != self.k or x.dtype != torch.float16 or not x.is_cuda:
            raise ValueError(f"x must be a float16 CUDA tensor [M, {self.k}], got "
                             f"{x.dtype} {tuple(x.shape)}")
        m = x.shape[0]
        if not 1 <= m <= self.max_m:
            raise ValueError(f"M = {m} must be in [1, {self.max_m}]")
        stream = torch.cuda.current_stream().cuda_stream
        if self.mode == "n":
            xs, n_local, k_local = x.contiguous(), self.q.shape[0], self.k
        else:
            k0, k1 = self.span
            xs, n_local, k_local = x[:, k0:k1].contiguous(), self.n, k1 - k0
        y = torch.empty(m, self.n, dtype=torch.float16, device=x.device)
        capi.call("int4gemv_w4a16_exchange", y.data_ptr(), xs.data_ptr(), self.q.data_ptr(),
                  self.s.data_ptr(), self.z.data_ptr(), m, n_local, k_local, self.group_size,
                  ctypes.addressof(self.peers), stream)
        return y
