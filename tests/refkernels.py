"""ctypes access to the reference's own CUDA kernels, built from its sources into
oracle/_ref/ by oracle/Makefile. Test and baseline infrastructure only."""
from __future__ import annotations

import ctypes
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def _load(name: str):
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is missing: build it with `make -C oracle` where the reference is present")
    return ctypes.CDLL(path)


_attn = None
_cds = None


def ref_attn_varlen():
    global _attn
    if _attn is None:
        lib = _load("libref_attn_varlen.so")
        lib.attn_varlen_host.restype = None
        lib.attn_varlen_host.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p,
                                         ctypes.c_void_p]
        _attn = lib
    return _attn


def ref_capture_decode():
    global _cds
    if _cds is None:
        lib = _load("libref_capture_decode.so")
        lib.capture_decode_host.restype = None
        lib.capture_decode_host.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int32] * 5 + [ctypes.c_void_p]
        _cds = lib
    return _cds


def ref_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_len: int, scale: float) -> torch.Tensor:
    """The reference kernel exactly as its attn_varlen.forward launches it (contiguous inputs)."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    H, D = q.shape
    ctx = torch.empty(H, D, dtype=torch.float16, device=q.device)
    stream = torch.cuda.current_stream().cuda_stream
    ref_attn_varlen().attn_varlen_host(q.data_ptr(), k.data_ptr(), v.data_ptr(), H, seq_len, D, float(scale),
                                       ctx.data_ptr(), stream)
    return ctx


def ref_capture_decode_step(ctrl, arena_k, arena_v, seq_len, pos, logits):
    L, _, H, max_len, D = arena_k.shape
    stream = torch.cuda.current_stream().cuda_stream
    ref_capture_decode().capture_decode_host(ctrl.data_ptr(), arena_k.data_ptr(), arena_v.data_ptr(),
                                             seq_len.data_ptr(), pos.data_ptr(), logits.data_ptr(), L, H, max_len,
                                             D, logits.shape[1], stream)
