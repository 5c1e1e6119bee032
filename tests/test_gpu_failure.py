"""Failure detection on the GPU without a fault: the bounded wait that every
pipeline wait of the kernels uses gives up after its limit on a barrier nothing
arrives on, reports the timeout bit, the kernel returns, and the same context then
runs a decode step correctly."""
import ctypes
import math
import time

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


def test_exchange_wait_times_out_and_reports():
    """The ctx exchange's wait on one GPU with flags that nothing raises: the one-CTA wait
    kernel gives up after its limit, sets FCCI_DEV_ERR_TIMEOUT (2) in the exchange's error
    word and returns; the context stays usable (a decode step afterwards is correct)."""
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    av = pkg.attn_varlen
    mem, _ = av.ipc_alloc(1024)
    flags, epoch, err = mem[0:16], mem[256:260], mem[512:516]
    epoch.view(torch.int32).fill_(1)  # every flag is 0: the epoch is never reached
    t0 = time.time()
    av.exchange_wait(flags, 4, epoch, err, 50_000_000)  # 50 ms
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert int(err.view(torch.int32).item()) & 2
    assert 0.04 < waited < 5.0
    # the context still works
    q = torch.randn(1, 8, 128, device="cuda").half()
    kc = torch.randn(1, 1, 100, 128, device="cuda").half()
    out = torch.empty_like(q)
    av.decode(q, kc, kc, out, fixed_len=100, split=False)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
