"""Host-side logic of the multi-GPU stack (int4gemv.sharded) on CPU: world size 2 and 3 over gloo.

The local GEMV is the oracle (CPU), injected through the `local_gemv` parameter, so these tests check
the sharding of the packed tensors, the exchange steps and the reassembly; the CUDA kernels are
checked on the GPU by the parity tests.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from int4gemv.sharded import ShardedW4A16, split_range

# (mode, m, n, k, group): N-split with N not divisible by the world size, K-split with K not an
# even number of groups per rank.
CASES = [("n", 1, 300, 1024, 128), ("n", 3, 97, 512, 128), ("k", 1, 64, 1408, 128),
         ("k", 2, 40, 768, 64)]


def oracle_gemv(x, q, s, z, g):
    y = oracle.reference(x.numpy(), q.numpy(), s.numpy(), z.numpy(), g)
    return torch.from_numpy(y.astype(np.float16))


def oracle_partial(x, q, s, z, g):
    y = oracle.reference(x.numpy(), q.numpy(), s.numpy(), z.numpy(), g)
    return torch.from_numpy(y.astype(np.float32))


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _worker(rank, world, port, cases, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = []
        for mode, m, n, k, g in cases:
            x, q, s, z = oracle.synthetic(m, n, k, g, seed=n + k)
            t = [torch.from_numpy(a) for a in (x, q, s, z)]
            layer = ShardedW4A16(t[1], t[2], t[3], g, mode, local_gemv=oracle_gemv,
                                 local_partial=oracle_partial)
            out.append(layer(t[0]).float().numpy())
        results[rank] = out
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_matches_single_device(world):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, CASES, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    for (mode, m, n, k, g), i in zip(CASES, range(len(CASES))):
        x, q, s, z = oracle.synthetic(m, n, k, g, seed=n + k)
        ref = oracle.reference(x, q, s, z, g)
        for r in range(world):
            y = results[r][i]
            assert y.shape == (m, n)
            ok, msg = oracle.check_close(y, ref, 1e-2, 1e-2)
            assert ok, f"{mode}-split world {world} rank {r}: {msg}"
        # every rank holds the same y
        for r in range(1, world):
            np.testing.assert_array_equal(results[r][i], results[0][i])


def test_split_range():
    assert [split_range(10, 3, i) for i in range(3)] == [(0, 4), (4, 7), (7, 10)]
    assert [split_range(1408, 2, i, 128) for i in range(2)] == [(0, 768), (768, 1408)]
    assert split_range(256, 4, 3, 128) == (256, 256)  # more ranks than groups: empty shard
    with pytest.raises(ValueError):
        split_range(100, 2, 0, 64)


def _fused_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from int4gemv.exchange import FusedShardedW4A16

        q = torch.zeros(6, 384, dtype=torch.int32)
        s = torch.zeros(6, 24, dtype=torch.float16)
        msgs = []
        for mode in ("n", "k", "x"):
            try:
                FusedShardedW4A16(q, s, s, 128, mode)
            except ValueError as e:
                msgs.append(str(e))
        results[rank] = msgs
    finally:
        dist.destroy_process_group()


def test_fused_layer_shape_checks():
    """int4gemv.exchange checks the sharding constraints on every rank before allocating: rows
    split needs N % world == 0, K split at least one whole 1024-weight stage per rank."""
    world = 4
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        n_msg, k_msg, mode_msg = results[r]
        assert "multiple of the world size" in n_msg
        assert "multiple of 1024 and at least 1024 x world" in k_msg
        assert "mode must be" in mode_msg


def _ksplit_rounding_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, n, k, g = 2, 64, 1024, 128
        x, q, s, z = oracle.synthetic(m, n, k, g, seed=77)
        t = [torch.from_numpy(a) for a in (x, q, s, z)]
        layer = ShardedW4A16(t[1], t[2], t[3], g, "k", local_gemv=oracle_gemv,
                             local_partial=oracle_partial)
        results[rank] = layer(t[0]).numpy()
    finally:
        dist.destroy_process_group()


def test_k_split_rounds_once():
    """The K-split layer adds the ranks' fp32 partial sums and rounds to fp16 once: its output is
    bit-identical to fp16(p0 + p1), and differs from the twice-rounded fp16(fp16(p0) + fp16(p1))
    on this case (so the test would catch a partial rounded to fp16 before the all-reduce)."""
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_ksplit_rounding_worker, args=(r, world, port, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    m, n, k, g = 2, 64, 1024, 128
    x, q, s, z = oracle.synthetic(m, n, k, g, seed=77)
    partials = []
    for r in range(world):
        k0, k1 = split_range(k, world, r, g)
        partials.append(oracle.reference(x[:, k0:k1], q[:, k0 // 8:k1 // 8],
                                         s[:, k0 // g:k1 // g], z[:, k0 // g:k1 // g],
                                         g).astype(np.float32))
    once = (partials[0] + partials[1]).astype(np.float16)
    twice = (partials[0].astype(np.float16).astype(np.float32)
             + partials[1].astype(np.float16).astype(np.float32)).astype(np.float16)
    for r in range(world):
        np.testing.assert_array_equal(results[r].view(np.uint16), once.view(np.uint16))
    assert not np.array_equal(once.view(np.uint16), twice.view(np.uint16))
