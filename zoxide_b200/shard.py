"""M-row sharding of one GEMM across the GPUs of a node (one process per GPU).

Each rank owns a contiguous block of A's rows and the same rows of C, and holds all of B (and
the column scales). The data path has no collective: every rank runs the single-GPU kernel on
its shard. Two collectives exist only around it: `max_over_ranks` for the job's wall time (the
slowest rank), and an optional all-gather of C slices that is timed on its own.
The reference is single-device (src/cuda_driver.zig:284-288 opens device 0); this module is
the multi-GPU layer the B200 build adds.
"""
from __future__ import annotations


def row_shard(M: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [m0, m1) of rank `rank`: contiguous, sizes differ by at most one row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return rank * M // world, (rank + 1) * M // world


def shard_sizes(M: int, world: int) -> list[int]:
    return [row_shard(M, world, r)[1] - row_shard(M, world, r)[0] for r in range(world)]


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank float over the default process group (the value itself if none)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(c_local, M: int):
    """All-gather every rank's rows of C into the full M x N matrix (equal or ragged shards)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size()
    sizes = shard_sizes(M, world)
    mx = max(sizes)
    n = c_local.shape[1]
    pad = torch.zeros((mx, n), dtype=c_local.dtype, device=c_local.device)
    pad[: c_local.shape[0]] = c_local
    out = torch.empty((world * mx, n), dtype=c_local.dtype, device=c_local.device)
    dist.all_gather_into_tensor(out, pad)
    parts = [out[r * mx: r * mx + sizes[r]] for r in range(world)]
    return torch.cat(parts, dim=0)


# ------------------------- all-gather of C overlapped with the GEMM -------------------------
# For the overlapped gather the M rows are dealt out chunk by chunk: with `world` ranks and
# `chunks` chunks, row block b = j * world + r (cr = M / (world * chunks) rows each) belongs to rank
# r, so chunk j of every rank sits in rows [j * world * cr, (j + 1) * world * cr) of the full C in
# rank order. Each rank computes its chunk j straight into its slot of the full C, and the
# in-place all-gather of chunk j (one NCCL call on its own stream) runs while the GEMM of chunk
# j + 1 is computing. Every rank still holds all of B; no data-path collective other than the
# gather itself.

def interleaved_blocks(M: int, world: int, chunks: int, rank: int) -> list[tuple[int, int]]:
    """Global row spans [start, stop) that `rank` owns, chunk by chunk (M % (world * chunks) == 0)."""
    if world < 1 or chunks < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank}, world {world}, chunks {chunks}")
    if M % (world * chunks):
        raise ValueError(f"M={M} is not a multiple of world x chunks = {world * chunks}")
    cr = M // (world * chunks)
    return [((j * world + rank) * cr, (j * world + rank + 1) * cr) for j in range(chunks)]


def gemm_allgather_overlapped(gemm, a_local, c_full, chunks: int):
    """Run gemm(a_rows, c_rows) for each of this rank's `chunks` row blocks into its slots of
    `c_full` (M x N, every rank's copy) and all-gather each block as soon as it is computed.

    `a_local` holds this rank's rows in chunk order (chunks x cr rows). The gathers are issued
    asynchronously after each block's GEMM (NCCL orders them after it on its own stream), so the
    transfer of block j overlaps the GEMM of block j + 1. Returns when all gathers are enqueued;
    the caller's stream waits on them before it returns, so work queued next sees all of c_full."""
    import torch.distributed as dist

    world, rank = dist.get_world_size(), dist.get_rank()
    M = c_full.shape[0]
    spans = interleaved_blocks(M, world, chunks, rank)
    cr = spans[0][1] - spans[0][0]
    works = []
    for j, (g0, g1) in enumerate(spans):
        gemm(a_local[j * cr:(j + 1) * cr], c_full[g0:g1])
        chunk = c_full[j * world * cr:(j + 1) * world * cr]
        works.append(dist.all_gather_into_tensor(chunk, c_full[g0:g1], async_op=True))
    for w in works:
        w.wait()


# ------------------- all-gather fused into the GEMM (stores to peer memory) -------------------
# Every rank holds the full M x N C. Its kernel (zx_gemm_s8_replicated) writes each tile of its
# own rows into its copy and, over NVLink, into the same rows of every other rank's copy, so the
# gather traffic overlaps the tensor-core work and no collective runs on the data path. The
# other ranks' copies are mapped into this process with CUDA IPC (cudaIpcOpenMemHandle with
# peer access, plain device pointers: no multicast object is created).

class PeerBuffers:
    """Maps every other rank's copy of a tensor into this process (collective over the default
    process group: every rank constructs it with its own copy, same shape and dtype).

    `peer_ptr(rank, byte_offset)` is a device address this rank's kernels can store to;
    `close()` unmaps the peers (every rank, after the last kernel that writes to them)."""

    def __init__(self, local):
        import ctypes

        import torch.distributed as dist

        from . import abi

        lib = abi.lib()
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        self.nbytes = local.numel() * local.element_size()
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        abi.check(lib.zx_ipc_export(local.data_ptr(), h, ctypes.byref(off)))
        mine = (bytes(h.raw), int(off.value), self.nbytes)
        allv = [None] * self.world
        dist.all_gather_object(allv, mine)
        self._bases, self._ptrs = {}, {}
        try:
            for r, (handle, offset, nbytes) in enumerate(allv):
                if r == self.rank:
                    continue
                if nbytes != self.nbytes:
                    raise ValueError(f"rank {r} shares {nbytes} bytes, this rank {self.nbytes}")
                base = ctypes.c_uint64(0)
                abi.check(lib.zx_ipc_import(handle, ctypes.byref(base)))
                self._bases[r] = base.value
                self._ptrs[r] = base.value + offset
        except Exception:
            self.close()
            raise

    def peer_ptr(self, rank: int, byte_offset: int = 0) -> int:
        if not 0 <= byte_offset < self.nbytes:
            raise ValueError(f"offset {byte_offset} outside the {self.nbytes}-byte buffer")
        return self._ptrs[rank] + byte_offset

    def peers(self) -> list[int]:
        return sorted(self._ptrs)

    def close(self) -> None:
        from . import abi

        lib = abi.lib()
        for r in list(self._bases):
            abi.check(lib.zx_ipc_close(self._bases.pop(r)))
            self._ptrs.pop(r, None)


def gemm_allgather_fused(a_local, b, c_full, m0: int, peer_bufs: PeerBuffers, stream=None):
    """C rows [m0, m0 + rows) = a_local * b^T into this rank's c_full and every peer's copy.

    The caller orders reads of c_full after every rank's kernel has completed (e.g. stream
    synchronisation on each rank followed by a barrier)."""
    from . import gemm_s8_replicated

    rows, n = a_local.shape[0], c_full.shape[1]
    off = m0 * n * c_full.element_size()
    peers = [peer_bufs.peer_ptr(r, off) for r in peer_bufs.peers()]
    return gemm_s8_replicated(a_local, b, c_full[m0:m0 + rows], peers, stream=stream)


# ------------------------ host buffers on several GPUs: B split across ranks ------------------------
# From host memory each rank needs its rows of A, all of B and a place for its rows of C. Copying
# all of B from the host on every rank moves B once per GPU over the shared host side; instead each
# rank copies 1/world of B's rows, and one in-place NCCL all-gather assembles the full B on every
# GPU over NVLink. The GEMM then runs by row chunks, each chunk of C copied back while the next
# one computes, so the host traffic of the job is A + B + C once.

def b_slice(nrows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of B that `rank` copies from the host (nrows % world == 0: an in-place
    all-gather needs equal slices)."""
    if nrows % world:
        raise ValueError(f"B has {nrows} rows, not a multiple of the world size {world}")
    per = nrows // world
    return rank * per, (rank + 1) * per


def gemm_host_sharded(gemm, A_host, B_host, C_host, A_dev, B_dev, C_dev, stream=None, chunks: int = 4):
    """This rank's rows of C from host buffers: C_host = gemm(A_host, B) with B split over ranks.

    A_host: this rank's rows of A; B_host: all of B (N x K rows, NT; only this rank's slice
    b_slice(N, world, rank) is read); C_host: this rank's rows of C. A_dev / B_dev / C_dev are
    device buffers of the same shapes. `gemm(a_rows, b_full, c_rows)` enqueues the GEMM of a row
    block on the current stream. Host tensors should be pinned for the copies to overlap.

    On CUDA tensors the copies run on two side streams: H2D of this rank's B slice then A in
    `chunks` row blocks, the all-gather of B (NCCL orders it after the slice), the GEMM of block j
    once its rows of A are in, and D2H of block j's C while block j + 1 computes. `stream` (the
    current stream by default) waits for the last copy back. With CPU tensors (gloo) the same
    steps run in order."""
    import torch
    import torch.distributed as dist

    world, rank = dist.get_world_size(), dist.get_rank()
    r0, r1 = b_slice(B_dev.shape[0], world, rank)
    M = A_dev.shape[0]
    bounds = [M * j // chunks for j in range(chunks + 1)]
    if not A_dev.is_cuda:
        B_dev[r0:r1].copy_(B_host[r0:r1])
        A_dev.copy_(A_host)
        dist.all_gather_into_tensor(B_dev, B_dev[r0:r1])
        for j in range(chunks):
            a0, a1 = bounds[j], bounds[j + 1]
            gemm(A_dev[a0:a1], B_dev, C_dev[a0:a1])
            C_host[a0:a1].copy_(C_dev[a0:a1])
        return C_host
    s = stream if stream is not None else torch.cuda.current_stream(A_dev.device)
    h2d, d2h = _side_streams(A_dev.device)
    start = torch.cuda.Event()
    start.record(s)
    h2d.wait_event(start)
    d2h.wait_event(start)
    with torch.cuda.stream(h2d):
        B_dev[r0:r1].copy_(B_host[r0:r1], non_blocking=True)
        b_in = torch.cuda.Event()
        b_in.record(h2d)
        a_in = []
        for j in range(chunks):
            a0, a1 = bounds[j], bounds[j + 1]
            A_dev[a0:a1].copy_(A_host[a0:a1], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
            a_in.append(ev)
    with torch.cuda.stream(s):
        s.wait_event(b_in)
        dist.all_gather_into_tensor(B_dev, B_dev[r0:r1])
        for j in range(chunks):
            a0, a1 = bounds[j], bounds[j + 1]
            s.wait_event(a_in[j])
            gemm(A_dev[a0:a1], B_dev, C_dev[a0:a1])
            done = torch.cuda.Event()
            done.record(s)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                C_host[a0:a1].copy_(C_dev[a0:a1], non_blocking=True)
        back = torch.cuda.Event()
        back.record(d2h)
        s.wait_event(back)
    return C_host


_SIDE = {}


def _side_streams(device):
    import torch

    key = torch.device(device).index
    if key not in _SIDE:
        _SIDE[key] = (torch.cuda.Stream(device), torch.cuda.Stream(device))
    return _SIDE[key]
