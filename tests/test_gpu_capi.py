"""GPU parity through the C ABI itself (ctypes, no pybind): what a caller in
another language binds. Same tolerances as tests/test_gpu_decode.py."""
import ctypes
import math

import pytest
import torch

import capi_ctypes as C
from helpers import randn_half
from oracle import decode_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def lib():
    return C.load()


def close(got, want):
    return O.compare(got.float().cpu(), want)


@pytest.mark.parametrize("T", [1, 70, 513, 3000])
def test_attn_varlen_host_symbol(lib, T):
    H, D = 32, 128
    q, k, v = randn_half((H, D), 1), randn_half((H, T, D), 2), randn_half((H, T, D), 3)
    dq, dk, dv = q.to(DEV), k.to(DEV), v.to(DEV)
    ctx = torch.empty(H, D, dtype=torch.float16, device=DEV)
    lib.attn_varlen_host(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), H, T, D, 1 / math.sqrt(D), ctx.data_ptr(),
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert lib.fcci_last_status() == 0, lib.fcci_last_error_string()
    ma, rl = close(ctx, O.attn_varlen_forward(q, k, v, T, 1 / math.sqrt(D)))
    assert ma <= O.MAX_ABS_TOL and rl <= O.REL_L2_TOL, (ma, rl)


@pytest.mark.parametrize("split", [0, 1])
def test_decode_descriptor(lib, split):
    B, Hkv, G, D, cap = 3, 4, 8, 128, 700
    lens = [5, 300, 640]
    q, kn, vn = randn_half((B, Hkv * G, D), 10), randn_half((B, Hkv, D), 11), randn_half((B, Hkv, D), 12)
    kc, vc = randn_half((B, Hkv, cap, D), 13), randn_half((B, Hkv, cap, D), 14)
    T = torch.tensor(lens, dtype=torch.int32)
    dq, dkn, dvn, dk, dv, dT = q.to(DEV), kn.to(DEV), vn.to(DEV), kc.to(DEV), vc.to(DEV), T.to(DEV)
    out = torch.empty(B, Hkv * G, D, dtype=torch.float16, device=DEV)
    nbytes = lib.fcci_decode_workspace_bytes(B, Hkv * G, Hkv, D, torch.cuda.current_device())
    assert nbytes > 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.fcci_decode_workspace_init(ws.data_ptr(), nbytes, stream) == 0
    d = C.batched_desc(dq, dk, dv, out, k_new=dkn, v_new=dvn, seq_lens=dT, advance=True, split=bool(split),
                       workspace=ws)
    assert lib.fcci_decode_attention(ctypes.byref(d), stream) == 0, lib.fcci_last_error_string()
    flags = ctypes.c_uint32(99)
    assert lib.fcci_decode_read_error(ws.data_ptr(), ctypes.byref(flags), 1, stream) == 0
    assert flags.value == 0
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn)
    ma, rl = close(out, want["ctx"])
    assert ma <= O.MAX_ABS_TOL and rl <= O.REL_L2_TOL, (ma, rl)
    assert dT.cpu().tolist() == [t + 1 for t in lens]


def test_descriptor_errors_are_status_codes(lib):
    d = C.DecodeDesc()
    d.abi_version = 99
    assert lib.fcci_decode_attention(ctypes.byref(d), None) == 1
    assert b"abi_version" in lib.fcci_last_error_string()
    q = torch.zeros(1, 8, 96, dtype=torch.float16, device=DEV)  # head_dim 96 is not compiled
    kc = torch.zeros(1, 8, 16, 96, dtype=torch.float16, device=DEV)
    d = C.batched_desc(q, kc, kc, q.clone(), fixed_len=4, split=False)
    assert lib.fcci_decode_attention(ctypes.byref(d), None) == 2
    assert b"unsupported" in lib.fcci_last_error_string()
    q = torch.zeros(1, 8, 128, dtype=torch.float16, device=DEV)
    kc = torch.zeros(1, 8, 16, 128, dtype=torch.float16, device=DEV)
    d = C.batched_desc(q, kc, kc, q.clone(), fixed_len=4, split=True)  # split needs a workspace
    assert lib.fcci_decode_attention(ctypes.byref(d), None) == 3


def test_descriptor_versions_and_flags(lib):
    """A version-1 descriptor (no flags field) still works; FCCI_DECODE_PREFETCH_KV gives
    the same bits, with or without FCCI_DECODE_CHECK_EARLY_READ; unknown flag bits are rejected
    with a status code."""
    B, Hkv, G, D, cap = 4, 2, 8, 128, 900
    lens = [3, 200, 880, 64]
    q, kn, vn = randn_half((B, Hkv * G, D), 20), randn_half((B, Hkv, D), 21), randn_half((B, Hkv, D), 22)
    kc, vc = randn_half((B, Hkv, cap, D), 23), randn_half((B, Hkv, cap, D), 24)
    T = torch.tensor(lens, dtype=torch.int32)
    nbytes = lib.fcci_decode_workspace_bytes(B, Hkv * G, Hkv, D, torch.cuda.current_device())
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.fcci_decode_workspace_init(ws.data_ptr(), nbytes, stream) == 0
    outs = []
    for version, flags in ((2, 0), (2, C.PREFETCH_KV), (2, C.PREFETCH_KV | C.CHECK_EARLY_READ), (1, 0)):
        dk, dv, dT = kc.to(DEV), vc.to(DEV), T.to(DEV)
        out = torch.empty(B, Hkv * G, D, dtype=torch.float16, device=DEV)
        d = C.batched_desc(q.to(DEV), dk, dv, out, k_new=kn.to(DEV), v_new=vn.to(DEV), seq_lens=dT, advance=True,
                           workspace=ws, flags=flags)
        if version == 1:
            v1 = C.DecodeDescV1()
            ctypes.memmove(ctypes.byref(v1), ctypes.byref(d), ctypes.sizeof(v1))
            v1.abi_version = 1
            rc = lib.fcci_decode_attention(ctypes.cast(ctypes.byref(v1), ctypes.POINTER(C.DecodeDesc)), stream)
        else:
            rc = lib.fcci_decode_attention(ctypes.byref(d), stream)
        assert rc == 0, lib.fcci_last_error_string()
        torch.cuda.synchronize()
        assert dT.cpu().tolist() == [t + 1 for t in lens]
        outs.append(out.cpu())
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    ma, rl = close(outs[0], O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn)["ctx"])
    assert ma <= O.MAX_ABS_TOL and rl <= O.REL_L2_TOL, (ma, rl)
    d = C.batched_desc(q.to(DEV), kc.to(DEV), vc.to(DEV), torch.empty(B, Hkv * G, D, dtype=torch.float16, device=DEV),
                       fixed_len=5, workspace=ws, flags=4)
    assert lib.fcci_decode_attention(ctypes.byref(d), stream) == 1
    assert b"flags" in lib.fcci_last_error_string()
