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
