"""Partitioning of the decode-attention work across the GPUs of one node.

One process per GPU. Two partitions, no data-path collective inside attention:

  by sequence  each rank owns whole sequences (their arena rows live only on that
               rank); sequences are bin-packed by KV bytes, which are proportional
               to their lengths (longest-first onto the least-loaded rank).
  by kv head   each rank owns a contiguous block of kv heads and the query heads of
               their GQA groups (Hq/N query heads, Hkv/N kv heads).

The only exchange is the ctx all-gather of the kv-head partition, needed when the
output projection that follows is not sharded: ctx [B, Hq/N, D] from each rank
becomes [B, Hq, D] on every rank (NCCL over NVLink; gloo in the CPU tests).
"""
from __future__ import annotations

from typing import List, Sequence

import torch


def partition_sequences(lengths: Sequence[int], world_size: int) -> List[List[int]]:
    """Sequence indices per rank; greedy longest-first bin packing by length (KV bytes).

    Deterministic: ties go to the lowest rank, equal lengths keep index order.
    """
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0] * world_size
    parts: List[List[int]] = [[] for _ in range(world_size)]
    for i in order:
        r = min(range(world_size), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += int(lengths[i])
    for p in parts:
        p.sort()
    return parts


def partition_by_cost(costs: Sequence[float], world_size: int) -> List[List[int]]:
    """Like partition_sequences but for arbitrary non-negative costs (e.g. L*(L+1)/2 for prefill)."""
    order = sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i))
    load = [0.0] * world_size
    parts: List[List[int]] = [[] for _ in range(world_size)]
    for i in order:
        r = min(range(world_size), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += float(costs[i])
    for p in parts:
        p.sort()
    return parts


def partition_kv_heads(kv_heads: int, q_heads: int, world_size: int, rank: int):
    """(kv_lo, kv_hi, q_lo, q_hi) owned by `rank`; kv_heads must be divisible by world_size."""
    if kv_heads % world_size != 0:
        raise ValueError(f"{kv_heads} kv heads do not split over {world_size} ranks")
    if q_heads % kv_heads != 0:
        raise ValueError("q_heads must be a multiple of kv_heads")
    per = kv_heads // world_size
    g = q_heads // kv_heads
    kv_lo = rank * per
    return kv_lo, kv_lo + per, kv_lo * g, (kv_lo + per) * g


def gather_ctx(local_ctx: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather of head-sharded ctx [B, Hq/N, D] into [B, Hq, D] on every rank.

    The collective runs on a contiguous [N, B, Hq/N, D] buffer (rank-major), then the
    heads are put back in order; with `out` given nothing is allocated but the
    staging buffer (pass it as out=... of shape [N, B, Hq/N, D] to avoid that too).
    """
    import torch.distributed as dist

    n = dist.get_world_size(group)
    B, hl, D = local_ctx.shape
    stage = torch.empty((n, B, hl, D), dtype=local_ctx.dtype, device=local_ctx.device)
    dist.all_gather_into_tensor(stage.view(n * B * hl * D), local_ctx.contiguous().view(B * hl * D), group=group)
    res = stage.permute(1, 0, 2, 3).reshape(B, n * hl, D)
    if out is not None:
        out.copy_(res)
        return out
    return res
