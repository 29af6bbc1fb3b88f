"""Batch sharding across GPUs for the denoise loop (one process per GPU, torch.distributed).

Observations are independent, so a global batch is split into contiguous shards, each rank runs
its own engine on its shard (own prefix KV / context and noise, full weight replica), and the
action chunks are gathered once at the end. There is no collective inside the loop; the gather
is the only data exchange (all_gather of the per-rank action chunks, padded to equal shard size).
"""
from __future__ import annotations

import torch


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of observations for `rank`: sizes differ by at most one, lower ranks
    take the extra observations."""
    if batch < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad shard request batch={batch} world={world} rank={rank}")
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_actions(local: torch.Tensor, batch: int, group=None) -> torch.Tensor:
    """All-gathers the per-rank action chunks [b_r][T][AD] into the global [batch][T][AD] (in
    rank order, which is batch order by shard_range). Works with the nccl and gloo backends."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    width = (batch + world - 1) // world
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    out = [parts[r][: shard_range(batch, world, r)[1] - shard_range(batch, world, r)[0]] for r in range(world)]
    return torch.cat(out, 0)
