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

from zoxide_b200.shard import interleaved_blocks, row_shard, shard_sizes


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


def test_interleaved_blocks_partition():
    for M, world, chunks in [(8192, 8, 4), (1024, 2, 2), (96, 3, 2), (16, 1, 4)]:
        spans = sorted(s for r in range(world) for s in interleaved_blocks(M, world, chunks, r))
        assert spans[0][0] == 0 and spans[-1][1] == M
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        # chunk j of every rank is contiguous, in rank order
        for j in range(chunks):
            starts = [interleaved_blocks(M, world, chunks, r)[j][0] for r in range(world)]
            assert starts == sorted(starts) and starts[0] == j * M // chunks
    with pytest.raises(ValueError):
        interleaved_blocks(100, 3, 2, 0)


def _worker_overlap(rank, world, port, M, N, K, chunks, q):
    import torch
    import torch.distributed as dist

    import oracle
    from zoxide_b200.shard import gemm_allgather_overlapped, interleaved_blocks

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = oracle.Rng(0x0FDB9753)
        A = r.s8((M, K))
        B = r.s8((N, K))
        mine = np.concatenate([A[g0:g1] for g0, g1 in interleaved_blocks(M, world, chunks, rank)])
        c_full = torch.full((M, N), -7, dtype=torch.int32)

        def gemm(a_rows, c_rows):  # the per-GPU kernel's job, done by the CPU oracle here
            c_rows.copy_(torch.from_numpy(oracle.gemm_s8(a_rows.numpy(), B, a_rows.shape[0], N, K, oracle.NT)))

        gemm_allgather_overlapped(gemm, torch.from_numpy(mine), c_full, chunks)
        q.put((rank, np.array_equal(c_full.numpy(), oracle.gemm_s8(A, B, M, N, K, oracle.NT))))
    finally:
        dist.destroy_process_group()


def test_overlapped_allgather_gloo_world2(zxo):
    """Chunk-interleaved shards + per-chunk in-place all-gather give every rank the full C."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_overlap, args=(r, 2, port, 128, 64, 96, 4, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: True, 1: True}


def _worker_host_sharded(rank, world, port, M, N, K, q):
    import torch
    import torch.distributed as dist

    import oracle
    from zoxide_b200.shard import b_slice, gemm_host_sharded, row_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = oracle.Rng(0x13579BDF)
        A = r.s8((M, K))
        B = r.s8((N, K))
        m0, m1 = row_shard(M, world, rank)
        b0, b1 = b_slice(N, world, rank)
        B_host = torch.zeros((N, K), dtype=torch.int8)
        B_host[b0:b1] = torch.from_numpy(B[b0:b1])  # this rank only has its slice of B on the host
        A_host = torch.from_numpy(np.ascontiguousarray(A[m0:m1]))
        C_host = torch.full((m1 - m0, N), -1, dtype=torch.int32)
        A_dev, B_dev = torch.empty_like(A_host), torch.full((N, K), 99, dtype=torch.int8)
        C_dev = torch.empty_like(C_host)

        def gemm(a_rows, b_full, c_rows):  # the per-GPU kernel's job, done by the CPU oracle here
            c_rows.copy_(torch.from_numpy(oracle.gemm_s8(a_rows.numpy(), b_full.numpy(), a_rows.shape[0], N, K,
                                                         oracle.NT)))

        gemm_host_sharded(gemm, A_host, B_host, C_host, A_dev, B_dev, C_dev, chunks=3)
        want = oracle.gemm_s8(np.ascontiguousarray(A[m0:m1]), B, m1 - m0, N, K, oracle.NT)
        q.put((rank, np.array_equal(C_host.numpy(), want) and np.array_equal(B_dev.numpy(), B)))
    finally:
        dist.destroy_process_group()


def test_host_sharded_b_split_gloo_world2(zxo):
    """Each rank copies half of B from the host; the all-gather assembles B and C is exact."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_host_sharded, args=(r, 2, port, 100, 64, 96, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: True, 1: True}


def test_b_slice_partition():
    from zoxide_b200.shard import b_slice

    assert [b_slice(8192, 8, r) for r in (0, 7)] == [(0, 1024), (7168, 8192)]
    with pytest.raises(ValueError):
        b_slice(100, 3, 0)
