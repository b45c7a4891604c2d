"""One model replica per GPU: request sharding and the host-side helpers of a multi-process run.

Concurrent TTS streams are independent (each owns its per-slot GDN / conv / KV state), so a box serves them with
one replica per GPU and no collective on the data path. These helpers split a request list across ranks, and
combine per-rank timings (max over ranks) and results on the host. They work with any torch.distributed backend
(NCCL on the GPU box, gloo in the CPU tests).
"""

from __future__ import annotations

import torch


def shard(n_requests: int, world: int, rank: int) -> range:
    """Contiguous, balanced share of ``n_requests`` for ``rank`` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n_requests, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def max_over_ranks(value: float, group=None, device=None) -> float:
    """The largest ``value`` over all ranks (the step time of a synchronous multi-replica run)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_rows(local: torch.Tensor, n_requests: int, group=None) -> torch.Tensor:
    """Concatenate every rank's [len(shard), ...] result rows back into request order (host-side, for the
    dispatcher; not used inside a timed region)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return local
    world = dist.get_world_size(group)
    sizes = [len(shard(n_requests, world, r)) for r in range(world)]
    width = max(sizes)
    padded = torch.zeros((width, *local.shape[1:]), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p[:n] for p, n in zip(parts, sizes)])
