"""Batch sharding of ACFUN0 inference across the GPUs of one node.

Images are independent (the executor has batch-1 semantics: model.cpp:274-349), so a batch
of n images splits into contiguous per-rank shards with no collective inside the graph.  The
only exchange is the final gather of the [n, out] outputs (NCCL all-gather over NVLink on GPU
ranks, any torch.distributed backend on CPU ranks).
"""
from __future__ import annotations


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of the images rank `rank` of `world` processes: contiguous, sizes differ
    by at most one, every image exactly once."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def gather_outputs(dist, local_out, n: int, world: int):
    """All-gather per-rank outputs [shard, out] into the full [n, out] tensor on every rank,
    in image order.  Shards of unequal size are padded to the largest for the collective."""
    import torch
    sizes = [shard_bounds(n, world, r) for r in range(world)]
    mx = max(e - b for b, e in sizes)
    out_dim = local_out.shape[1]
    pad = torch.zeros((mx, out_dim), dtype=local_out.dtype, device=local_out.device)
    pad[: local_out.shape[0]] = local_out
    full = torch.empty((world * mx, out_dim), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(full, pad)
    parts = [full[r * mx: r * mx + (e - b)] for r, (b, e) in enumerate(sizes)]
    return torch.cat(parts, 0)
