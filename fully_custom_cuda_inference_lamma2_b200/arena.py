"""Persistent GQA KV arena and the per-step decode-attention call.

The reference keeps one arena per session, k/v = [L, 1, H, max_len, D] fp16
with a device int32 seq_len (case4_graph_generator_server_ipc.py:1224-1262).
KVArena generalises it to B sequences and two HBM layouts:

  batched  k/v [L, B, Hkv, capacity, D]   sequence b owns rows [0, capacity)
  packed   k/v [L, Hkv, total, D]         sequence b owns rows
                                          [cu_seqlens[b], cu_seqlens[b+1])

Both are head-major, so the keys of one (sequence, kv head) are contiguous and
a 16-key box of the TMA pipeline is one 4 KB stretch of HBM (K and V together).
`seq_lens` (device int32 [B]) holds each sequence's cached length T_b; a
decode step reads it on the device, appends at T_b and, when asked, bumps it.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

from . import attn_varlen


class KVArena:
    """Device-resident KV arena of `layers` layers for B sequences."""

    def __init__(self, layers: int, batch: int, kv_heads: int, head_dim: int, *,
                 capacity: Optional[int] = None, seq_capacities: Optional[Sequence[int]] = None,
                 q_heads: Optional[int] = None, device=None, dtype=torch.float16, fill: str = "empty"):
        if dtype != torch.float16:
            raise ValueError("the decode kernels take fp16 K/V")
        if (capacity is None) == (seq_capacities is None):
            raise ValueError("give exactly one of capacity (batched) or seq_capacities (packed)")
        self.layers, self.batch, self.kv_heads, self.head_dim = layers, batch, kv_heads, head_dim
        self.q_heads = q_heads if q_heads is not None else kv_heads
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        alloc = torch.zeros if fill == "zeros" else torch.empty
        if capacity is not None:
            self.packed = False
            self.capacity = int(capacity)
            shape = (layers, batch, kv_heads, self.capacity, head_dim)
            self.cu_seqlens = None
        else:
            self.packed = True
            caps = [int(c) for c in seq_capacities]
            if len(caps) != batch:
                raise ValueError("one capacity per sequence")
            offs = [0]
            for c in caps:
                offs.append(offs[-1] + c)
            self.capacity = offs[-1]
            shape = (layers, kv_heads, self.capacity, head_dim)
            self.cu_seqlens = torch.tensor(offs, dtype=torch.int32, device=self.device)
        self.k = alloc(shape, dtype=dtype, device=self.device)
        self.v = alloc(shape, dtype=dtype, device=self.device)
        self.seq_lens = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self.workspace = attn_varlen.make_workspace(batch, self.q_heads, kv_heads, head_dim, self.device)

    def layer(self, l: int):
        """(k, v) views of layer l in the layout decode() takes."""
        return self.k[l], self.v[l]

    def kv_bytes(self) -> int:
        """Bytes of K and V currently attended to by one layer (host read of seq_lens)."""
        lens = self.seq_lens.to("cpu", torch.int64)
        return int(lens.sum()) * self.kv_heads * self.head_dim * 2 * 2


def decode_attention(arena: KVArena, layer: int, q: torch.Tensor, out: torch.Tensor, *,
                     k_new: Optional[torch.Tensor] = None, v_new: Optional[torch.Tensor] = None,
                     advance: bool = False, scale: Optional[float] = None, rope_theta: float = 10000.0,
                     rotary_dim: int = -1, q_rot_out: Optional[torch.Tensor] = None,
                     prefetch_kv: bool = False) -> torch.Tensor:
    """One decode-attention step of `layer`: RoPE + append at T_b (when k_new is given) and
    split-KV attention, on the current stream, without allocation or host sync.

    prefetch_kv: read the lengths and the first cached K/V tiles before waiting for the
    previous kernel on the stream (FCCI_DECODE_PREFETCH_KV). Only when no kernel that may
    still be running writes seq_lens or this layer's cached rows, e.g. right after the
    projection that produced q/k_new/v_new, or after another layer's decode step that
    does not advance."""
    k, v = arena.layer(layer)
    attn_varlen.decode(q, k, v, out, k_new=k_new, v_new=v_new, seq_lens=arena.seq_lens,
                       cu_seqlens=arena.cu_seqlens, scale=-1.0 if scale is None else float(scale),
                       rope_theta=rope_theta, rotary_dim=rotary_dim, advance=advance,
                       workspace=arena.workspace, q_rot_out=q_rot_out, split=True, prefetch_kv=prefetch_kv)
    return out


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
