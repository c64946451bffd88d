"""The GEMM with its all-gather fused in (zx_gemm_s8_replicated): each C tile is stored to C and
to every peer buffer from the same staged tile.

On one GPU the "peers" are other buffers of the same device, which runs the same store path;
with two GPUs, two processes map each other's full C through CUDA IPC (shard.PeerBuffers) and
every rank must end with the whole product. The reference has no multi-GPU path
(src/cuda_driver.zig:284-288); the oracle is its exact CPU check (src/host.zig:302-317)."""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,npeers", [(256, 512, 512, 1), (300, 520, 256, 3), (1024, 1536, 1024, 7),
                                          (2048, 2048, 512, 2)])
def test_replicas_equal_oracle(zx, zxo, M, N, K, npeers):
    r = zxo.Rng.from_seed(M * 7 + N)
    A, B = r.s8((M, K)), r.s8((N, K))
    want = zxo.gemm_s8(A, B, M, N, K, zxo.NT)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
    peers = [torch.full((M, N), -1, dtype=torch.int32, device="cuda") for _ in range(npeers)]
    zx.gemm_s8_replicated(Ad, Bd, C, [p.data_ptr() for p in peers])
    torch.cuda.synchronize()
    assert "gemm_tc2w_kernel" in zx.last_kernel(), zx.last_kernel()
    assert zx.device_status() == 0
    assert np.array_equal(C.cpu().numpy(), want)
    for p in peers:
        assert np.array_equal(p.cpu().numpy(), want)


def test_replicas_into_row_slices(zx, zxo):
    """Shard-style pointers: the rows [m0, m0 + Mr) of a larger full C on each 'peer'."""
    M, N, K, m0, Mr = 1024, 1024, 512, 256, 512
    r = zxo.Rng.from_seed(11)
    A, B = r.s8((Mr, K)), r.s8((N, K))
    want = zxo.gemm_s8(A, B, Mr, N, K, zxo.NT)
    full = [torch.full((M, N), -1, dtype=torch.int32, device="cuda") for _ in range(3)]
    zx.gemm_s8_replicated(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), full[0][m0:m0 + Mr],
                          [f[m0:m0 + Mr].data_ptr() for f in full[1:]])
    torch.cuda.synchronize()
    for f in full:
        h = f.cpu().numpy()
        assert np.array_equal(h[m0:m0 + Mr], want)
        assert (h[:m0] == -1).all() and (h[m0 + Mr:] == -1).all()  # nothing outside its rows


def test_peer_buffer_checks(zx):
    """A peer buffer shorter than M x N int32 (its own cudaMalloc, so the allocation ends where
    the buffer does) and a host address are rejected before the launch."""
    from cuda.bindings import runtime as rt

    lib = zx.lib()
    M, N, K = 256, 512, 256
    A = torch.zeros((M, K), dtype=torch.int8, device="cuda")
    B = torch.zeros((N, K), dtype=torch.int8, device="cuda")
    C = torch.empty((M, N), dtype=torch.int32, device="cuda")
    err, short = rt.cudaMalloc(M * N * 4 - 4096)
    assert err == rt.cudaError_t.cudaSuccess
    try:
        arr = (ctypes.c_uint64 * 1)(int(short))
        rc = lib.zx_gemm_s8_replicated(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, arr, 1, None)
        torch.cuda.synchronize()
        if rc == 0:
            pytest.skip("the driver reports a rounded-up allocation size; the stores stayed inside it")
        assert rc == zx.abi.ZX_ERR_SHAPE and "holds" in zx.abi.last_error()
    finally:
        rt.cudaFree(short)
    host = np.zeros(M * N, dtype=np.int32)
    arr = (ctypes.c_uint64 * 1)(host.ctypes.data)
    rc = lib.zx_gemm_s8_replicated(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, arr, 1, None)
    assert rc != 0, "a host address must be rejected"
    assert zx.device_status() == 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ipc_worker(rank, world, port, M, N, K, q):
    import torch.distributed as dist

    import oracle
    import zoxide_b200 as zx
    from zoxide_b200.shard import PeerBuffers, gemm_allgather_fused, row_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = oracle.Rng.from_seed(0x2468)
        A, B = r.s8((M, K)), r.s8((N, K))
        m0, m1 = row_shard(M, world, rank)
        c_full = torch.full((M, N), -1, dtype=torch.int32, device="cuda")
        pb = PeerBuffers(c_full)
        try:
            gemm_allgather_fused(torch.from_numpy(np.ascontiguousarray(A[m0:m1])).cuda(),
                                 torch.from_numpy(B).cuda(), c_full, m0, pb)
            torch.cuda.synchronize()
            dist.barrier()  # every rank's kernel (and so its stores into this c_full) completed
            ok = np.array_equal(c_full.cpu().numpy(), oracle.gemm_s8(A, B, M, N, K, oracle.NT))
            status = zx.device_status()
        finally:
            torch.cuda.synchronize()
            dist.barrier()
            pb.close()
            dist.barrier()
        q.put((rank, ok, status))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [2048, 1000])
def test_two_gpus_every_rank_gets_all_rows(zx, M):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    N, K, world = 1024, 512, 2
    port = _port()
    procs = [ctx.Process(target=_ipc_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(q.get(timeout=5) for _ in range(world))
    assert got == [(0, True, 0), (1, True, 0)], got
