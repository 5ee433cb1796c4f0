"""Work split of the reused-KV path across the GPUs of one node.

* Data parallel (requests are independent): ``assign_requests`` gives each
  rank a bytes-balanced set of requests; ranks never exchange data.
* Tensor parallel over KV heads (the 70B shape): rank r holds heads
  ``tp_head_range(r, world, H)``; rotation and scatter are head-local. The
  per-token deviation score is a sum over heads, so each rank computes its
  partial [layers, tokens] fp32 matrix (rerotate_scatter_pages ``scores``)
  and ``allreduce_scores`` sums it across ranks (one NCCL all-reduce for all
  layers); every rank then runs the same selection on identical scores.

The reference records its TP/PP ranks (integration/vllm/utils.py:160-170)
and suffixes store keys per rank (management/client.py:81-85); its tensor
collectives belong to vLLM.
"""
from __future__ import annotations

import heapq
from typing import Optional, Sequence

import torch

__all__ = ["assign_requests", "tp_head_range", "allreduce_scores"]


def assign_requests(request_bytes: Sequence[int], world: int) -> list[list[int]]:
    """Largest-first greedy assignment of requests to ``world`` ranks by
    bytes; returns each rank's request indices in ascending order."""
    if world <= 0:
        raise ValueError("world must be positive")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    order = sorted(range(len(request_bytes)), key=lambda i: (-int(request_bytes[i]), i))
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(request_bytes[i]), r))
    return [sorted(x) for x in out]


def tp_head_range(rank: int, world: int, num_heads: int) -> tuple[int, int]:
    """Contiguous KV-head shard [h0, h1) of a rank (vLLM's KV head split)."""
    if num_heads % world:
        raise ValueError(f"{num_heads} KV heads do not split over {world} ranks")
    per = num_heads // world
    return rank * per, (rank + 1) * per


def allreduce_scores(partial: torch.Tensor, group=None) -> torch.Tensor:
    """Sums per-rank partial scores in place (one all-reduce of the whole
    [layers, tokens] matrix). Every rank receives the same values."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
