"""CPU oracle of the Llama-2-shaped greedy decode — TEST INFRASTRUCTURE ONLY.

Only tests/ use it, as the checker. It restates in
torch fp32 the model the reference decodes (an HF LlamaForCausalLM: RMSNorm,
q/k/v/o projections, rotate-half RoPE at the token's position, causal softmax
attention, SiLU-gated MLP, tied embeddings, greedy argmax;
case4_graph_generator_server_ipc.py:1241-1262 for the prompt,
scripts/direct_custom_decode_500.py:229-250 for the per-token step, RoPE as
scripts/direct_custom_decode_500.py:90-108).

`logits_for(tokens)` runs the whole sequence causally and returns the logits at
every position, so a decoder's per-step logits can be compared under teacher forcing.
"""
from __future__ import annotations

import math

import torch

from . import decode_oracle as O


def rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def logits_for(weights, tokens) -> torch.Tensor:
    """fp32 logits [n, vocab] at every position of `tokens` (list or int64 tensor)."""
    s = weights.shape
    f = lambda t: t.detach().float().cpu()
    emb = f(weights.embed)
    tok = torch.as_tensor(tokens, dtype=torch.int64).cpu()
    n = tok.numel()
    Hq, Hkv, D, I = s.heads, s.kv_heads, s.head_dim, s.intermediate
    G = Hq // Hkv
    x = emb[tok]
    pos = torch.arange(n)
    half = D // 2
    inv = O.inv_freq(D, s.rope_theta)
    ang = pos.float().view(-1, 1) * inv.view(1, -1)
    cos, sin = torch.cos(ang).unsqueeze(1), torch.sin(ang).unsqueeze(1)

    def rope(t):  # [n, H, D]
        a, b = t[..., :half], t[..., half:]
        return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)

    mask = torch.triu(torch.ones(n, n, dtype=torch.bool), 1)
    for l in range(s.layers):
        h = rms(x, f(weights.rms_in[l]), s.eps)
        qkv = h @ f(weights.w_qkv[l]).t()
        q = rope(qkv[:, : Hq * D].view(n, Hq, D))
        k = rope(qkv[:, Hq * D: (Hq + Hkv) * D].view(n, Hkv, D))
        v = qkv[:, (Hq + Hkv) * D:].view(n, Hkv, D)
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
        sc = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(D)
        sc = sc.masked_fill(mask, float("-inf"))
        ctx = torch.einsum("hqk,khd->qhd", torch.softmax(sc, -1), v).reshape(n, Hq * D)
        x = x + ctx @ f(weights.w_o[l]).t()
        h = rms(x, f(weights.rms_post[l]), s.eps)
        gu = h @ f(weights.w_gu[l]).t()
        x = x + (torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]) @ f(weights.w_down[l]).t()
    return rms(x, f(weights.rms_final), s.eps) @ emb.t()
