"""ctypes binding of include/fcci_decode.h — what a non-pybind caller of the
library writes. Used by the C-ABI parity tests."""
from __future__ import annotations

import ctypes
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(ROOT, "fully_custom_cuda_inference_lamma2_b200", "libfcci_decode.so")
ABI_VERSION = 2
PREFETCH_KV = 1
CHECK_EARLY_READ = 2

c_i32, c_i64, c_vp, c_f32, c_sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float, ctypes.c_size_t


_DESC_V1_FIELDS = [
    ("abi_version", c_i32), ("B", c_i32), ("Hq", c_i32), ("Hkv", c_i32), ("D", c_i32),
    ("q", c_vp), ("q_stride_b", c_i64), ("q_stride_h", c_i64),
    ("k_new", c_vp), ("k_new_stride_b", c_i64), ("k_new_stride_h", c_i64),
    ("v_new", c_vp), ("v_new_stride_b", c_i64), ("v_new_stride_h", c_i64),
    ("k_cache", c_vp), ("k_stride_b", c_i64), ("k_stride_h", c_i64), ("k_stride_t", c_i64),
    ("v_cache", c_vp), ("v_stride_b", c_i64), ("v_stride_h", c_i64), ("v_stride_t", c_i64),
    ("capacity", c_i32), ("cu_seqlens", c_vp), ("seq_lens", c_vp), ("fixed_len", c_i32),
    ("out", c_vp), ("out_stride_b", c_i64), ("out_stride_h", c_i64), ("q_rot_out", c_vp),
    ("scale", c_f32), ("rope_theta", c_f32), ("rotary_dim", c_i32), ("advance", c_i32), ("split", c_i32),
    ("workspace", c_vp), ("workspace_bytes", c_sz),
]


class DecodeDescV1(ctypes.Structure):
    """fcci_decode_desc as version 1 of the ABI laid it out (no trailing flags)."""
    _fields_ = _DESC_V1_FIELDS


class DecodeDesc(ctypes.Structure):
    _fields_ = _DESC_V1_FIELDS + [("flags", ctypes.c_uint32)]


def load(path: str = LIB_PATH):
    lib = ctypes.CDLL(path)
    lib.fcci_decode_attention.argtypes = [ctypes.POINTER(DecodeDesc), c_vp]
    lib.fcci_decode_attention.restype = ctypes.c_int
    lib.fcci_rope_append.argtypes = [ctypes.POINTER(DecodeDesc), c_vp]
    lib.fcci_rope_append.restype = ctypes.c_int
    lib.fcci_decode_workspace_bytes.argtypes = [c_i32, c_i32, c_i32, c_i32, ctypes.c_int]
    lib.fcci_decode_workspace_bytes.restype = c_sz
    lib.fcci_decode_workspace_init.argtypes = [c_vp, c_sz, c_vp]
    lib.fcci_decode_workspace_init.restype = ctypes.c_int
    lib.fcci_decode_read_error.argtypes = [c_vp, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, c_vp]
    lib.fcci_decode_read_error.restype = ctypes.c_int
    lib.fcci_last_error_string.restype = ctypes.c_char_p
    lib.fcci_last_status.restype = ctypes.c_int
    lib.attn_varlen_host.argtypes = [c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_f32, c_vp, c_vp]
    lib.attn_varlen_host.restype = None
    return lib


def batched_desc(q, k_cache, v_cache, out, *, k_new=None, v_new=None, seq_lens=None, fixed_len=0, scale=None,
                 rope_theta=10000.0, rotary_dim=None, advance=False, split=True, workspace=None, q_rot_out=None,
                 flags=0):
    """Descriptor for torch CUDA tensors: q [B,Hq,D], caches [B,Hkv,cap,D], out [B,Hq,D]."""
    B, Hq, D = q.shape
    Hkv, cap = k_cache.shape[1], k_cache.shape[2]
    d = DecodeDesc()
    d.abi_version, d.B, d.Hq, d.Hkv, d.D = ABI_VERSION, B, Hq, Hkv, D
    d.q, d.q_stride_b, d.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    if k_new is not None:
        d.k_new, d.k_new_stride_b, d.k_new_stride_h = k_new.data_ptr(), k_new.stride(0), k_new.stride(1)
        d.v_new, d.v_new_stride_b, d.v_new_stride_h = v_new.data_ptr(), v_new.stride(0), v_new.stride(1)
    d.k_cache, d.k_stride_b, d.k_stride_h, d.k_stride_t = k_cache.data_ptr(), *k_cache.stride()[:3]
    d.v_cache, d.v_stride_b, d.v_stride_h, d.v_stride_t = v_cache.data_ptr(), *v_cache.stride()[:3]
    d.capacity = cap
    d.seq_lens = seq_lens.data_ptr() if seq_lens is not None else None
    d.fixed_len = fixed_len
    d.out, d.out_stride_b, d.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    d.q_rot_out = q_rot_out.data_ptr() if q_rot_out is not None else None
    d.scale = scale if scale is not None else D ** -0.5
    d.rope_theta = rope_theta
    d.rotary_dim = (D if k_new is not None else 0) if rotary_dim is None else rotary_dim
    d.advance, d.split, d.flags = int(advance), int(split), int(flags)
    if workspace is not None:
        d.workspace, d.workspace_bytes = workspace.data_ptr(), workspace.numel()
    return d
