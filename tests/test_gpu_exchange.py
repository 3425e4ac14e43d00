"""The sharded layer with the exchange fused into the GEMV (int4gemv.exchange, the C ABI's
int4gemv_w4a16_exchange): rows split (peer stores of y into every rank) and K split (peer stores of
fp32 partials, summed in rank order), checked against the oracle on the full matrix over several
consecutive calls (alternating buffers, increasing call numbers), eager and replayed from a
captured CUDA graph. World size 1 runs on one GPU; the 2-GPU test is skipped when fewer GPUs are
visible."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

# (mode, M, N, K): rows split needs N % world == 0, K split K % 1024 == 0 and K >= 1024 x world
# (uneven stage counts per rank allowed: 3072 over 2 ranks is 2 + 1 stages)
CASES = [("n", 1, 28672, 8192), ("n", 8, 4096, 2048), ("k", 1, 8192, 28672), ("k", 5, 1024, 8192),
         ("n", 32, 2048, 1024), ("k", 2, 4100, 4096), ("k", 3, 512, 3072)]
CALLS = 3  # consecutive calls per case, each with its own x


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _inputs(case_index, mode, m, n, k):
    _, q, s, z = oracle.synthetic(1, n, k, 128, seed=100 + case_index)
    xs = [np.random.default_rng(1000 * case_index + c).standard_normal((m, k)).astype(np.float16)
          for c in range(CALLS)]
    return xs, q, s, z


def _run_cases(rank, world):
    from int4gemv import capi
    from int4gemv.exchange import FusedShardedW4A16

    out = []
    for i, (mode, m, n, k) in enumerate(CASES):
        xs, q, s, z = _inputs(i, mode, m, n, k)
        dev = [torch.from_numpy(a).cuda() for a in (q, s, z)]
        layer = FusedShardedW4A16(*dev, 128, mode)
        ys = []
        for x in xs:
            y = layer(torch.from_numpy(x).cuda())
            ys.append(y.float().cpu().numpy())
        # the same calls replayed from a captured CUDA graph (call numbers kept on the device)
        static_x = torch.zeros(m, k, dtype=torch.float16, device="cuda")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_y = layer(static_x)
        for x in xs:
            static_x.copy_(torch.from_numpy(x).cuda())
            graph.replay()
            ys.append(static_y.float().cpu().numpy())
        torch.cuda.synchronize()
        del graph
        layer.close()
        out.append(ys)
    assert capi.device_status() == 0
    return out


def _check(results_per_rank):
    for i, (mode, m, n, k) in enumerate(CASES):
        xs, q, s, z = _inputs(i, mode, m, n, k)
        for c, x in enumerate(xs + xs):  # eager calls, then graph replays
            ref = oracle.reference(x, q, s, z, 128)
            for r, res in enumerate(results_per_rank):
                ok, msg = oracle.check_close(res[i][c], ref, 1e-2, 1e-2)
                assert ok, f"{mode}-split {m}x{n}x{k} call {c} rank {r}: {msg}"
            for res in results_per_rank[1:]:
                np.testing.assert_array_equal(res[i][c], results_per_rank[0][i][c])


def test_exchange_world_one():
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        _check([_run_cases(0, 1)])
    finally:
        dist.destroy_process_group()


def _worker(rank, world, port, results):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        results[rank] = _run_cases(rank, world)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_exchange_two_gpus():
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
        p.join(timeout=600)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    _check([results[r] for r in range(world)])
