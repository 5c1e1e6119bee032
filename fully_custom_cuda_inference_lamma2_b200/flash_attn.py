"""Single-query SDPA on the decode-attention kernel, with the reference's names.

The reference's custom_kernels/flash_attn.py defines `sdp_single_q(q, k, v, scale)`
(attention of one query position over T keys, computed in fp32 by its own kernel)
and `enable_flash_sdp_monkeypatch()`, which routes every
`torch.nn.functional.scaled_dot_product_attention` call with one query position and
no mask to it and leaves the others to torch (custom_kernels/flash_attn.py:18-36).

Here both names run the split-KV decode kernel of this library in fp16:
q [B, Hq, 1, D] over k, v [B, Hkv, T, D] read in place through their strides
(Hq a multiple of Hkv: a GQA group shares each K/V tile; HF's repeated K/V
[B, Hq, T, D] works too). Calls the kernel does not compute (other dtypes, head_dim
outside {64, 128, 256}, a mask, dropout, more than one query position) go to the
function that was patched, as the reference sends its masked and prefill calls.
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

from . import attn_varlen

_WORKSPACES: Dict[Tuple[int, int, int, int, int], torch.Tensor] = {}
_ORIGINAL_SDPA = None


def _workspace(device: torch.device, B: int, Hq: int, Hkv: int, D: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), B, Hq, Hkv, D)
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = attn_varlen.make_workspace(B, Hq, Hkv, D, device)
        _WORKSPACES[key] = ws
    return ws


def supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """True when the decode kernel computes this call: fp16 CUDA, q [B, Hq, 1, D],
    k/v [B, Hkv, T, D] with Hq % Hkv == 0, T >= 1, D in {64, 128, 256}."""
    if not (q.is_cuda and q.dtype == torch.float16 and k.dtype == torch.float16 and v.dtype == torch.float16):
        return False
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4 or q.size(2) != 1:
        return False
    B, Hq, _, D = q.shape
    if k.shape != v.shape or k.size(0) != B or k.size(3) != D or D not in (64, 128, 256):
        return False
    Hkv, T = k.size(1), k.size(2)
    return Hkv > 0 and Hq % Hkv == 0 and T >= 1 and (Hq // Hkv) <= 16


def sdp_single_q(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
    """softmax(q k^T * scale) v for q [B, H, 1, D] over k, v [B, Hkv, T, D] (fp16, CUDA);
    returns [B, H, 1, D] fp16. scale defaults to 1/sqrt(D)."""
    if not supported(q, k, v):
        raise ValueError("sdp_single_q: needs fp16 CUDA q [B, H, 1, D], k/v [B, Hkv, T, D], H % Hkv == 0, "
                         "D in {64, 128, 256}")
    B, Hq, _, D = q.shape
    Hkv, T = k.size(1), k.size(2)
    q3 = q[:, :, 0, :]
    if q3.stride(2) != 1:
        q3 = q3.contiguous()
    # the decode kernel reads the cache through TMA: head_dim contiguous, 16-byte strides
    kk = k if (k.stride(3) == 1 and all(s % 8 == 0 for s in k.stride()[:3]) and k.data_ptr() % 16 == 0) else k.contiguous()
    vv = v if (v.stride(3) == 1 and all(s % 8 == 0 for s in v.stride()[:3]) and v.data_ptr() % 16 == 0) else v.contiguous()
    out = torch.empty(B, Hq, 1, D, dtype=q.dtype, device=q.device)
    attn_varlen.decode(q3, kk, vv, out[:, :, 0, :], fixed_len=T,
                       scale=float(scale) if scale is not None else 1.0 / math.sqrt(D), rotary_dim=0,
                       workspace=_workspace(q.device, B, Hq, Hkv, D), split=True)
    return out


def enable_flash_sdp_monkeypatch():
    """Route single-query, unmasked `F.scaled_dot_product_attention` calls to sdp_single_q."""
    global _ORIGINAL_SDPA
    import torch.nn.functional as F

    if _ORIGINAL_SDPA is not None:
        return
    _ORIGINAL_SDPA = orig = F.scaled_dot_product_attention

    def _fn(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, **kwargs):
        if attn_mask is None and dropout_p == 0.0 and query.dim() == 4 and query.size(2) == 1 \
                and supported(query, key, value):
            return sdp_single_q(query, key, value, scale)
        return orig(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p, is_causal=is_causal, scale=scale,
                    **kwargs)

    F.scaled_dot_product_attention = _fn


def disable_flash_sdp_monkeypatch():
    """Restore the function enable_flash_sdp_monkeypatch replaced."""
    global _ORIGINAL_SDPA
    import torch.nn.functional as F

    if _ORIGINAL_SDPA is not None:
        F.scaled_dot_product_attention = _ORIGINAL_SDPA
        _ORIGINAL_SDPA = None
