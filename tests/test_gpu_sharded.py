"""The sharded GEMV (int4gemv.sharded) on 2 GPUs over NCCL: N-split + all-gather and K-split + fp32
all-reduce, each rank running the CUDA fast path, checked against the oracle on the full matrix.
Skipped when fewer than 2 GPUs are visible."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

CASES = [("n", 1, 6000, 4096), ("n", 8, 4096, 2048), ("k", 1, 2048, 7168), ("k", 4, 1024, 8192)]


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _worker(rank, world, port, results):
    import torch.distributed as dist

    from int4gemv.sharded import ShardedW4A16

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        out = []
        for mode, m, n, k in CASES:
            x, q, s, z = oracle.synthetic(m, n, k, 128, seed=n + k + m)
            dev = [torch.from_numpy(a).cuda() for a in (x, q, s, z)]
            layer = ShardedW4A16(dev[1], dev[2], dev[3], 128, mode)
            y = layer(dev[0])
            torch.cuda.synchronize()
            out.append(y.float().cpu().numpy())
        results[rank] = out
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_sharded_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    for i, (mode, m, n, k) in enumerate(CASES):
        x, q, s, z = oracle.synthetic(m, n, k, 128, seed=n + k + m)
        ref = oracle.reference(x, q, s, z, 128)
        for r in range(world):
            ok, msg = oracle.check_close(results[r][i], ref, 1e-2, 1e-2)
            assert ok, f"{mode}-split rank {r} {m}x{n}x{k}: {msg}"
        np.testing.assert_array_equal(results[0][i], results[1][i])
