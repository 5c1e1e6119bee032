"""CPU oracle of the decode-attention path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only as the checker or as the timed CPU baseline; the product
(fully_custom_cuda_inference_lamma2_b200) never imports it.

It restates, in torch fp32 eager on the CPU, the reference algorithm of each
step (paths inside divakar-yadav/Fully_Custom_Cuda_Inference_Lamma2):

  rope_rotate_half    scripts/direct_custom_decode_500.py:90-108 (rotate-half on the
                      first rotary_dim dims, inv_freq = theta**(-i/half), fp32 math,
                      result rounded to the input dtype)
  append_row          scripts/direct_custom_decode_500.py:237-240
  attention           case4_graph_generator_server_ipc.py:1000-1006 (einsum -> softmax
                      -> einsum), the math of custom_kernels/attn_varlen_kernel.cu:9-86;
                      GQA query head h reads kv head h // G as the
                      repeat_interleave of direct_custom_decode_500.py:245-247
  decode_step         the per-layer attention step of direct_custom_decode_500.py:229-250
  attn_varlen_forward custom_kernels/attn_varlen.cpp:16-45 (attention over the first
                      seq_len keys)
  placeholder_step    custom_kernels/capture_decode_step_kernel.cu:58-92
  prefill_step        case4_graph_generator_server_ipc.py:1241-1262 (kv_init: the model
                      forward over the prompt - RoPE at positions T_b + i, causal
                      attention - and the copy of the rotated keys / values into the
                      arena rows T_b .. T_b + n_b - 1)

Pinned against the reference's own code run here (tests/golden/make_golden.py:
RoPE of the decode driver and of the server) and against the reference CUDA
kernel built from its sources and run on a B200 (tests/golden/make_golden_gpu.py).
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def inv_freq(rotary_dim: int, theta: float, device=None) -> torch.Tensor:
    """fp32 inverse frequencies theta ** (-i / half), i < half (driver :95-97)."""
    half = rotary_dim // 2
    idx = torch.arange(half, dtype=torch.float32, device=device)
    return theta ** (-idx / float(half))


def rope_rotate_half(x: torch.Tensor, pos: int, rotary_dim: int, theta: float = 10000.0) -> torch.Tensor:
    """Rotate-half RoPE of x [n, D] at integer position pos; returns a new tensor of x's dtype.

    Evaluated on x's device, as the driver evaluates it on its own (CUDA) tensors, so a
    CUDA input reproduces the reference's device arithmetic (its powf/cosf/sinf)."""
    out = x.clone()
    if rotary_dim <= 0:
        return out
    half = rotary_dim // 2
    angle = pos * inv_freq(rotary_dim, theta, x.device).view(1, -1)
    cos, sin = torch.cos(angle), torch.sin(angle)
    x1 = x[:, :half].float()
    x2 = x[:, half:rotary_dim].float()
    out[:, :half] = (x1 * cos - x2 * sin).to(x.dtype)
    out[:, half:rotary_dim] = (x2 * cos + x1 * sin).to(x.dtype)
    return out


def rope_server_inplace(x: torch.Tensor, pos: int, theta: float = 10000.0) -> torch.Tensor:
    """The server's table RoPE (case4_graph_generator_server_ipc.py:869-898) on fp32 heads.

    inv_freq = 1 / theta**(2i/D); it writes the first half in place before computing
    the second half from the same view, so the second half reads the ROTATED first
    half: x2' = x1' * sin + x2 * cos. Restated here only to pin the fixture; the
    decode path follows the driver's rotation (rope_rotate_half), which is correct.
    """
    D = x.shape[1]
    h = D // 2
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    ang = torch.arange(pos, pos + 1, dtype=torch.float32).view(-1, 1) * inv.view(1, -1)
    c, s = torch.cos(ang[0]), torch.sin(ang[0])
    out = x.float().clone()
    first = out[:, :h] * c - out[:, h:] * s
    out[:, :h] = first
    out[:, h:] = out[:, :h] * s + out[:, h:] * c
    return out


def attention(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, scale: float) -> torch.Tensor:
    """ctx[h] = softmax(q[h] . K[h//G]^T * scale) V[h//G] in fp32.

    q [Hq, D]; K, V [Hkv, L, D]; returns fp32 [Hq, D]. L == 0 gives zeros.
    """
    Hq, D = q.shape
    Hkv, L, _ = K.shape
    G = Hq // Hkv
    if L == 0:
        return torch.zeros(Hq, D, dtype=torch.float32)
    qg = q.float().view(Hkv, G, D)
    scores = torch.einsum("kgd,ktd->kgt", qg, K.float()) * scale
    probs = torch.softmax(scores, dim=-1)
    return torch.einsum("kgt,ktd->kgd", probs, V.float()).reshape(Hq, D)


def attn_varlen_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_len: int, scale: float) -> torch.Tensor:
    """The reference forward(q[H,D], k[H,T,D], v[H,T,D], seq_len, scale) on its first seq_len keys."""
    return attention(q, k[:, :seq_len], v[:, :seq_len], scale)


def _rows(cache: torch.Tensor, b: int, t0: int, t1: int, cu: Optional[torch.Tensor]) -> torch.Tensor:
    """Keys t0..t1 of sequence b as [Hkv, t1-t0, D] (batched [B,Hkv,cap,D] or packed [Hkv,total,D])."""
    if cu is None:
        return cache[b, :, t0:t1]
    base = int(cu[b])
    return cache[:, base + t0: base + t1]


def append_row(k_cache, v_cache, b: int, T: int, k_row, v_row, cu=None) -> None:
    """arena[.., T, :] = k_row / v_row for sequence b (driver :237-240)."""
    if cu is None:
        k_cache[b, :, T] = k_row
        v_cache[b, :, T] = v_row
    else:
        base = int(cu[b])
        k_cache[:, base + T] = k_row
        v_cache[:, base + T] = v_row


def decode_step(q, k_cache, v_cache, seq_lens, *, k_new=None, v_new=None, cu_seqlens=None, scale=None,
                theta: float = 10000.0, rotary_dim: Optional[int] = None, capacity: Optional[int] = None,
                inplace: bool = False):
    """One decode step over B sequences, on copies of the caches.

    q [B,Hq,D] fp16; k_new/v_new [B,Hkv,D] fp16 or None; caches batched [B,Hkv,cap,D] or
    packed [Hkv,total,D] with cu_seqlens [B+1]; seq_lens [B] cached lengths T_b.
    With k_new: RoPE(q, k_new) at position T_b, append at T_b, attend to T_b+1 keys;
    without: attend to the first T_b keys with q as given (rotary_dim defaults to 0).
    A sequence whose T_b (+1) does not fit its capacity gets ctx = 0 and no append.
    Returns dict(ctx fp32 [B,Hq,D], q_rot fp16, k_cache, v_cache, seq_lens, ok [B] bool).
    With inplace=True the given caches receive the appended rows instead of copies.
    """
    B, Hq, D = q.shape
    if not inplace:
        k_cache = k_cache.clone()
        v_cache = v_cache.clone()
    scale = (1.0 / math.sqrt(D)) if scale is None else scale
    append = k_new is not None
    rot = (D if append else 0) if rotary_dim is None else rotary_dim
    ctx = torch.zeros(B, Hq, D, dtype=torch.float32)
    q_rot = q.clone()
    new_lens = seq_lens.clone()
    ok = torch.zeros(B, dtype=torch.bool)
    for b in range(B):
        T = int(seq_lens[b])
        if cu_seqlens is None:
            cap = k_cache.shape[2] if capacity is None else capacity
        else:
            cap = int(cu_seqlens[b + 1]) - int(cu_seqlens[b])
        L = T + (1 if append else 0)
        if T < 0 or L > cap:
            continue
        ok[b] = True
        qr = rope_rotate_half(q[b], T, rot, theta)
        q_rot[b] = qr
        if append:
            kr = rope_rotate_half(k_new[b], T, rot, theta)
            append_row(k_cache, v_cache, b, T, kr, v_new[b], cu_seqlens)
            new_lens[b] = T + 1
        K = _rows(k_cache, b, 0, L, cu_seqlens)
        V = _rows(v_cache, b, 0, L, cu_seqlens)
        ctx[b] = attention(qr, K, V, scale)
    return dict(ctx=ctx, q_rot=q_rot, k_cache=k_cache, v_cache=v_cache, seq_lens=new_lens, ok=ok)


def rope_positions(x: torch.Tensor, pos: torch.Tensor, rotary_dim: int, theta: float = 10000.0) -> torch.Tensor:
    """Rotate-half RoPE of x [n, H, D] where row i sits at position pos[i].

    Row by row the same fp32 arithmetic as rope_rotate_half (angle = pos * inv_freq,
    cos/sin, x1*cos - x2*sin and x2*cos + x1*sin, rounded to x's dtype), evaluated on
    x's device."""
    out = x.clone()
    if rotary_dim <= 0 or x.shape[0] == 0:
        return out
    half = rotary_dim // 2
    angle = pos.to(device=x.device, dtype=torch.float32).view(-1, 1) * inv_freq(rotary_dim, theta, x.device).view(1, -1)
    cos, sin = torch.cos(angle).unsqueeze(1), torch.sin(angle).unsqueeze(1)
    x1 = x[:, :, :half].float()
    x2 = x[:, :, half:rotary_dim].float()
    out[:, :, :half] = (x1 * cos - x2 * sin).to(x.dtype)
    out[:, :, half:rotary_dim] = (x2 * cos + x1 * sin).to(x.dtype)
    return out


def causal_attention(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, T: int, scale: float) -> torch.Tensor:
    """Causal attention of n new query rows over L = T + n keys, fp32.

    q [n, Hq, D] (new token i at position T + i); K, V [Hkv, L, D]; query head h reads
    kv head h // G. Key t is visible to row i when t <= T + i (the causal mask of the
    HF LlamaAttention forward the reference's kv_init runs). Returns fp32 [n, Hq, D]."""
    n, Hq, D = q.shape
    Hkv, L, _ = K.shape
    G = Hq // Hkv
    qg = q.float().permute(1, 0, 2).reshape(Hkv, G, n, D)
    scores = torch.einsum("kgnd,ktd->kgnt", qg, K.float()) * scale
    rows = torch.arange(n).view(n, 1) + T
    cols = torch.arange(L).view(1, L)
    scores = scores.masked_fill(cols > rows, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    out = torch.einsum("kgnt,ktd->kgnd", probs, V.float())
    return out.reshape(Hq, n, D).permute(1, 0, 2).contiguous()


def prefill_step(q, k_new, v_new, k_cache, v_cache, cu_seqlens_q, seq_lens, *, cu_seqlens_kv=None, scale=None,
                 theta: float = 10000.0, rotary_dim: Optional[int] = None, inplace: bool = False):
    """Causal prefill of the new tokens of B sequences, on copies of the caches.

    Restates the reference's kv_init (case4_graph_generator_server_ipc.py:1241-1262):
    the model forward over the prompt (rotate-half RoPE at positions T_b + i, causal
    softmax(q k^T * scale) v) and the copy of the rotated keys and the values into the
    arena rows T_b .. T_b + n_b - 1, after which the cached length is T_b + n_b.

    q [total, Hq, D], k_new / v_new [total, Hkv, D] fp16; sequence b owns rows
    cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1. Caches batched [B, Hkv, cap, D] or packed
    [Hkv, total_kv, D] with cu_seqlens_kv. A sequence whose T_b + n_b exceeds its
    capacity is skipped (out rows 0, ok False).
    Returns dict(out fp32 [total, Hq, D], q_rot fp16, k_cache, v_cache, seq_lens, ok)."""
    total, Hq, D = q.shape
    B = int(cu_seqlens_q.numel()) - 1
    if not inplace:
        k_cache = k_cache.clone()
        v_cache = v_cache.clone()
    scale = (1.0 / math.sqrt(D)) if scale is None else scale
    rot = D if rotary_dim is None else rotary_dim
    out = torch.zeros(total, Hq, D, dtype=torch.float32)
    q_rot = q.clone()
    new_lens = seq_lens.clone()
    ok = torch.zeros(B, dtype=torch.bool)
    for b in range(B):
        r0, r1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        n = r1 - r0
        T = int(seq_lens[b])
        if cu_seqlens_kv is None:
            cap = k_cache.shape[2]
        else:
            cap = int(cu_seqlens_kv[b + 1]) - int(cu_seqlens_kv[b])
        if T < 0 or T + n > cap:
            continue
        ok[b] = True
        new_lens[b] = T + n
        if n == 0:
            continue
        pos = torch.arange(T, T + n)
        qr = rope_positions(q[r0:r1], pos, rot, theta)
        kr = rope_positions(k_new[r0:r1], pos, rot, theta)
        q_rot[r0:r1] = qr
        if cu_seqlens_kv is None:
            k_cache[b, :, T:T + n] = kr.permute(1, 0, 2)
            v_cache[b, :, T:T + n] = v_new[r0:r1].permute(1, 0, 2)
        else:
            base = int(cu_seqlens_kv[b])
            k_cache[:, base + T: base + T + n] = kr.permute(1, 0, 2)
            v_cache[:, base + T: base + T + n] = v_new[r0:r1].permute(1, 0, 2)
        K = _rows(k_cache, b, 0, T + n, cu_seqlens_kv)
        V = _rows(v_cache, b, 0, T + n, cu_seqlens_kv)
        out[r0:r1] = causal_attention(qr, K, V, T, scale)
    return dict(out=out, q_rot=q_rot, k_cache=k_cache, v_cache=v_cache, seq_lens=new_lens, ok=ok)


def placeholder_step(ctrl: int, arena_k, arena_v, T: int, vocab: int):
    """capture_decode placeholder: zero rows [:, 0, :, T, :], one-hot logits, T+1.

    The remainder follows C (sign of the dividend); a negative index writes nothing.
    """
    arena_k = arena_k.clone()
    arena_v = arena_v.clone()
    if 0 <= T < arena_k.shape[3]:
        arena_k[:, 0, :, T, :] = 0
        arena_v[:, 0, :, T, :] = 0
    logits = torch.zeros(1, vocab, dtype=torch.float32)
    hot = int(math.fmod(ctrl, vocab))
    if hot >= 0:
        logits[0, hot] = 1.0
    return arena_k, arena_v, logits, T + 1


def compare(got: torch.Tensor, want: torch.Tensor) -> tuple[float, float]:
    """(max-abs, relative-L2) of got vs want, in fp64."""
    g = got.double().cpu()
    w = want.double().cpu()
    diff = g - w
    max_abs = float(diff.abs().max()) if diff.numel() else 0.0
    den = float(w.norm())
    rel = float(diff.norm()) / den if den > 0 else float(diff.norm())
    return max_abs, rel


# Tolerance of the decode-attention output against this fp32 oracle (fp16 in/out).
MAX_ABS_TOL = 2e-3
REL_L2_TOL = 1e-3
