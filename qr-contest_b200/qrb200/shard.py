"""Batch sharding across ranks (one process per GPU).

Every matrix is factored independently and the pipeline is forkless (no data-dependent
routing), so a static contiguous split is balanced: rank r of W gets
``[r * ceil(b/W), min(b, (r+1) * ceil(b/W)))``.  There is no collective on the data path; a
caller that needs every result on one rank gathers them afterwards.
"""
from __future__ import annotations


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    if world < 1 or not 0 <= rank < world or batch < 0:
        raise ValueError(f"bad shard request batch={batch} world={world} rank={rank}")
    per = -(-batch // world)
    lo = min(batch, rank * per)
    return lo, min(batch, lo + per)


def gather_results(H, tau, batch: int, group=None):
    """All-gather each rank's (H, tau) slice into full (batch, n, n) / (batch, n) tensors.

    Slices may be ragged (the last ranks can hold fewer matrices): every rank pads to
    ceil(batch / world) before ``all_gather_into_tensor`` and the padding is dropped.
    """
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    per = -(-batch // world)
    n = H.shape[-1]
    Hp = torch.zeros(per, n, n, dtype=H.dtype, device=H.device)
    tp = torch.zeros(per, n, dtype=tau.dtype, device=tau.device)
    Hp[: H.shape[0]] = H
    tp[: tau.shape[0]] = tau
    Hall = torch.empty(world * per, n, n, dtype=H.dtype, device=H.device)
    tall = torch.empty(world * per, n, dtype=tau.dtype, device=tau.device)
    dist.all_gather_into_tensor(Hall, Hp, group=group)
    dist.all_gather_into_tensor(tall, tp, group=group)
    return Hall[:batch], tall[:batch]
