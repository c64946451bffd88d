"""M-row sharding host logic on CPU with world_size-2 gloo ranks (no GPU).

Each rank computes its rows of C with the CPU oracle (standing in for the per-GPU kernel), the
slices are all-gathered and must equal the unsharded product; max_over_ranks must return the
slowest rank's value. The same functions drive bench.py under torchrun on B200s.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from zoxide_b200.shard import row_shard, shard_sizes


def test_row_shard_partition():
    for M in (1, 7, 1024, 8192, 65536):
        for world in (1, 2, 3, 4, 8):
            spans = [row_shard(M, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(shard_sizes(M, world)) - min(shard_sizes(M, world)) <= 1
    with pytest.raises(ValueError):
        row_shard(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, N, K, q):
    import torch
    import torch.distributed as dist

    import oracle
    from zoxide_b200.shard import gather_rows, max_over_ranks, row_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = oracle.Rng(0x13579BDF)
        A = r.s8((M, K))
        B = r.s8((N, K))
        m0, m1 = row_shard(M, world, rank)
        c_local = oracle.gemm_s8(np.ascontiguousarray(A[m0:m1]), B, m1 - m0, N, K, oracle.NT)
        full = gather_rows(torch.from_numpy(c_local), M).numpy()
        slowest = max_over_ranks(10.0 + rank)
        if rank == 0:
            ok = np.array_equal(full, oracle.gemm_s8(A, B, M, N, K, oracle.NT))
            q.put((ok, slowest))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [256, 255])
def test_sharded_gemm_gloo_world2(zxo, M):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, M, 64, 128, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ok, slowest = q.get(timeout=10)
    assert ok
    assert slowest == 11.0
