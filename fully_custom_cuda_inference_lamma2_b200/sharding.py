"""Partitioning of the decode-attention work across the GPUs of one node.

One process per GPU. Two partitions, no data-path collective inside attention:

  by sequence  each rank owns whole sequences (their arena rows live only on that
               rank); sequences are bin-packed by KV bytes, which are proportional
               to their lengths (longest-first onto the least-loaded rank).
  by kv head   each rank owns a contiguous block of kv heads and the query heads of
               their GQA groups (Hq/N query heads, Hkv/N kv heads).

The only exchange is the ctx all-gather of the kv-head partition, needed when the
output projection that follows is not sharded: ctx [B, Hq/N, D] from each rank
becomes [B, Hq, D] on every rank. Two ways: `CtxExchange`, where the decode launch
itself stores its slice into every rank's buffer over NVLink (peer stores to CUDA IPC
mappings) and raises a flag, and `gather_ctx`, an NCCL all-gather after the launch
(gloo in the CPU tests).
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


def gather_ctx(local_ctx: torch.Tensor, group=None, out: torch.Tensor | None = None,
               stage: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather of head-sharded ctx [B, Hq/N, D] into [B, Hq, D] on every rank.

    The collective writes a rank-major [N, B, Hq/N, D] buffer, whose heads are then put
    back in order ([B, Hq, D]). `stage` (shape [N, B, Hq/N, D]) is that buffer; without it
    one is allocated per call. With `out` the ordered result is written there (a copy),
    otherwise it is returned as a new tensor."""
    import torch.distributed as dist

    n = dist.get_world_size(group)
    B, hl, D = local_ctx.shape
    if stage is None:
        stage = torch.empty((n, B, hl, D), dtype=local_ctx.dtype, device=local_ctx.device)
    dist.all_gather_into_tensor(stage.view(n * B * hl * D), local_ctx.contiguous().view(B * hl * D), group=group)
    res = stage.permute(1, 0, 2, 3)
    if out is not None:
        out.view(B, n, hl, D).copy_(res)
        return out
    return res.reshape(B, n * hl, D)


def exchange_layout(B: int, Hq: int, D: int, world: int, buffers: int = 2):
    """Byte offsets inside one rank's exchange allocation: `buffers` full-ctx buffers
    [B, Hq, D] fp16 (alternate layers), then the flag array (world uint32), the epoch and
    the error word, each 256-byte aligned. Every rank uses the same layout, so a peer's
    slot is its base address plus the same offset."""
    up = lambda x: (x + 255) // 256 * 256
    ctx = B * Hq * D * 2
    flags = up(ctx * buffers)
    epoch = flags + up(4 * world)
    err = epoch + 256
    return dict(ctx_bytes=ctx, buffers=buffers, flags=flags, epoch=epoch, err=err, total=err + 256)


def slice_offset(B: int, Hq: int, D: int, q_lo: int, buffer: int) -> int:
    """Byte offset of rank-slice [:, q_lo:, :] of full-ctx buffer `buffer` ([B, Hq, D] fp16):
    where the slice's first element sits in every rank's allocation."""
    return buffer * B * Hq * D * 2 + q_lo * D * 2


class CtxExchange:
    """The kv-head partition's ctx exchange fused into the decode launch.

    Every rank allocates one IPC buffer (exchange_layout) and maps every other rank's.
    `decode(...)` runs this rank's decode step with `out` = its slice of its own full-ctx
    buffer for the layer, and the kernel stores the same slice into every peer's buffer
    (one plain store per peer over NVLink) before its last CTA raises this rank's slot
    of every flag array to the next epoch. `wait()` holds the current stream until every
    rank's slot has reached this rank's epoch (bounded: FCCI_DEV_ERR_TIMEOUT in `err`
    when it runs out). Layers alternate between two buffers, so a rank that passed layer
    l's wait can store layer l+1's slice while another still reads layer l.
    Every rank must make the same calls in the same order."""

    def __init__(self, B: int, Hq: int, D: int, group=None, buffers: int = 2, limit_ns: int = 2_000_000_000):
        import torch.distributed as dist

        from . import attn_varlen

        self.av = attn_varlen
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise ValueError("the ctx exchange needs 2 to 8 ranks on one node")
        self.B, self.Hq, self.D = B, Hq, D
        self.limit_ns = int(limit_ns)
        self.layout = L = exchange_layout(B, Hq, D, self.world, buffers)
        self.mem, handle = attn_varlen.ipc_alloc(L["total"])
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.peers = [r for r in range(self.world) if r != self.rank]
        self.peer_base = {r: attn_varlen.ipc_open(handles[r]) for r in self.peers}
        dist.barrier(group=group)
        ctx = L["ctx_bytes"]
        self.full = [self.mem[i * ctx:(i + 1) * ctx].view(torch.float16).view(B, Hq, D) for i in range(buffers)]
        self.flags = self.mem[L["flags"]:L["flags"] + 4 * self.world]
        self.epoch = self.mem[L["epoch"]:L["epoch"] + 4]
        self.err = self.mem[L["err"]:L["err"] + 4]

    def buffer(self, layer: int) -> torch.Tensor:
        """The full ctx [B, Hq, D] of `layer` on this rank (valid after wait())."""
        return self.full[layer % len(self.full)]

    def decode(self, q, k_cache, v_cache, q_lo: int, layer: int, **kw) -> torch.Tensor:
        """attn_varlen.decode of this rank's shard (query heads q_lo .. q_lo + q.shape[1]),
        with its ctx slice exchanged; returns the layer's full-ctx buffer."""
        buf = layer % len(self.full)
        hl = q.shape[1]
        out = self.full[buf][:, q_lo:q_lo + hl]
        off = slice_offset(self.B, self.Hq, self.D, q_lo, buf)
        assert out.data_ptr() - self.mem.data_ptr() == off
        self.av.decode(q, k_cache, v_cache, out, peer_out=[self.peer_base[r] + off for r in self.peers],
                       peer_flags=[self.peer_base[r] + self.layout["flags"] for r in self.peers],
                       exch_flags=self.flags.data_ptr(), exch_epoch=self.epoch.data_ptr(), exch_rank=self.rank, **kw)
        return self.full[buf]

    def wait(self) -> None:
        self.av.exchange_wait(self.flags, self.world, self.epoch, self.err, self.limit_ns)

    def error(self) -> int:
        """The device error word (synchronises)."""
        return int(self.err.view(torch.int32).item())

    def close(self) -> None:
        """Unmap the peers' buffers once every rank is done with them; the own buffer is
        freed when the last reference to it goes."""
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for r, ptr in self.peer_base.items():
            self.av.ipc_close(ptr)
        self.peer_base = {}
        dist.barrier(group=self.group)
