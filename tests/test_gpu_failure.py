"""Failure detection on the GPU without a fault: the bounded wait that every
pipeline wait of the kernels uses gives up after its limit on a barrier nothing
arrives on, reports the timeout bit, the kernel returns, and the same context then
runs a decode step correctly."""
import ctypes
import math

import pytest
import torch

import capi_ctypes as C
from helpers import randn_half
from oracle import decode_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_stays_usable():
    lib = C.load()
    f = lib.fcci_selftest_bounded_wait
    f.argtypes = [ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint32), ctypes.c_void_p]
    f.restype = ctypes.c_int
    res = (ctypes.c_uint32 * 2)()
    assert f(50_000_000, res, torch.cuda.current_stream().cuda_stream) == 0, lib.fcci_last_error_string()
    assert res[0] == 2, "the wait did not report a timeout"
    assert 45 <= res[1] < 1000, f"waited {res[1]} ms for a 50 ms limit"
    assert f(2_000_000_000, res, None) == 1  # limits above 1 s are refused
    # the context still works: one decode step against the oracle
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    q, kn, vn = randn_half((1, 8, 128), 1), randn_half((1, 8, 128), 2), randn_half((1, 8, 128), 3)
    kc, vc = randn_half((1, 8, 64, 128), 4), randn_half((1, 8, 64, 128), 5)
    T = torch.tensor([40], dtype=torch.int32)
    dk, dv, dT = kc.cuda(), vc.cuda(), T.cuda()
    out = torch.empty(1, 8, 128, dtype=torch.float16, device="cuda")
    pkg.attn_varlen.decode(q.cuda(), dk, dv, out, k_new=kn.cuda(), v_new=vn.cuda(), seq_lens=dT)
    torch.cuda.synchronize()
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn, scale=1 / math.sqrt(128))
    max_abs, rel = O.compare(out.float().cpu(), want["ctx"])
    assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL
