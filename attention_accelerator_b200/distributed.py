"""Multi-GPU plumbing for the decode path: one process per GPU over torch.distributed.

Two schemes:

* **Sequence sharding (no collective).**  A batch of decode requests is split
  across ranks by :func:`balance_sequences` (greedy longest-first assignment
  by visible-key count); every rank decodes its own sequences.
* **Long-context split.**  One sequence's keys are cut into contiguous shards,
  :func:`shard_range`; each rank computes FP32 partial rows for its shard
  (``plan_batch(..., pos_begin, pos_end, partial=True)`` + ``decode_batch``),
  :func:`gather_partials` all-gathers them (NCCL over NVLink on GPUs), and
  ``combine_partials`` merges them with a log-sum-exp combine.

The reference has a single device and no collective; this is the scaling
scheme of the new build.
"""
from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


def shard_range(n_keys: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous key range ``[lo, hi)`` of ``rank`` among ``world`` shards (sizes differ by <= 1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(n_keys, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def balance_sequences(visible_keys, world: int) -> list[list[int]]:
    """Assign sequence indices to ``world`` ranks, longest first to the least-loaded rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for idx in sorted(range(len(visible_keys)), key=lambda i: (-int(visible_keys[i]), i)):
        load, r = heapq.heappop(heap)
        out[r].append(idx)
        heapq.heappush(heap, (load + int(visible_keys[idx]), r))
    return [sorted(x) for x in out]


def gather_partials(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather one rank's partial rows ``[B, 32, 132]`` into ``[world, B, 32, 132]``."""
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    if local.is_cuda:
        dist.all_gather_into_tensor(out.view(world, -1), local.contiguous().view(-1), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), local.contiguous(), group=group)
    return out
