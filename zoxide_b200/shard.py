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
