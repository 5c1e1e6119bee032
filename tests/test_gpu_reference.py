"""Side by side on the GPU: the reference's own kernels (built from its sources
into oracle/_ref), the fp32 oracle, and this library, on identical inputs.

This pins the oracle to the reference implementation (reference vs oracle) and
checks the drop-in claim directly (this library vs reference)."""
import math

import pytest
import torch

from helpers import randn_half
from oracle import decode_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ref():
    import refkernels

    refkernels.ref_attn_varlen()
    return refkernels


@pytest.fixture(scope="module")
def av():
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    return pkg.attn_varlen


def close(a, b):
    return O.compare(a.float().cpu(), b.float().cpu())


@pytest.mark.parametrize("H,T,D", [(32, 1, 128), (32, 2, 128), (32, 64, 128), (32, 65, 128), (32, 513, 128),
                                   (8, 300, 64), (4, 200, 256)])
def test_reference_kernel_vs_oracle_vs_ours(ref, av, H, T, D):
    q = randn_half((H, D), 31 + T)
    k = randn_half((H, T, D), 32 + T)
    v = randn_half((H, T, D), 33 + T)
    scale = 1.0 / math.sqrt(D)
    want = O.attn_varlen_forward(q, k, v, T, scale)
    got_ref = ref.ref_forward(q.to(DEV), k.to(DEV), v.to(DEV), T, scale)
    got = av.forward(q.to(DEV), k.to(DEV), v.to(DEV), T, scale)
    torch.cuda.synchronize()
    ma, rl = close(got_ref, want)
    assert ma <= O.MAX_ABS_TOL and rl <= O.REL_L2_TOL, f"reference vs oracle {ma} {rl}"
    ma, rl = close(got, got_ref)
    assert ma <= O.MAX_ABS_TOL and rl <= O.REL_L2_TOL, f"ours vs reference {ma} {rl}"


def test_reference_driver_gqa_path_vs_ours(ref, av):
    """The driver's GQA path (contiguous slice + repeat_interleave + forward,
    direct_custom_decode_500.py:241-249) against one decode() call."""
    Hkv, G, D, T, max_len = 4, 8, 128, 300, 512
    q = randn_half((Hkv * G, D), 41)
    arena_k = randn_half((Hkv, max_len, D), 42).to(DEV)
    arena_v = randn_half((Hkv, max_len, D), 43).to(DEV)
    Ks = arena_k[:, :T].contiguous().repeat_interleave(G, dim=0)
    Vs = arena_v[:, :T].contiguous().repeat_interleave(G, dim=0)
    got_ref = ref.ref_forward(q.to(DEV), Ks, Vs, T, 1 / math.sqrt(D))
    out = torch.empty(1, Hkv * G, D, dtype=torch.float16, device=DEV)
    av.decode(q.view(1, Hkv * G, D).to(DEV), arena_k.unsqueeze(0), arena_v.unsqueeze(0), out, fixed_len=T)
    torch.cuda.synchronize()
    ma, rl = close(out[0], got_ref)
    assert ma <= O.MAX_ABS_TOL and rl <= O.REL_L2_TOL, f"{ma} {rl}"


@pytest.mark.parametrize("T,ctrl", [(5, 1234567), (0, 3), (15, 42)])
def test_placeholder_identical_to_reference(ref, T, ctrl):
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    L, H, max_len, D, vocab = 2, 4, 16, 128, 1000
    ak = randn_half((L, 1, H, max_len, D), 51).to(DEV)
    avv = randn_half((L, 1, H, max_len, D), 52).to(DEV)
    outs = []
    for which in ("ref", "ours"):
        k, v = ak.clone(), avv.clone()
        c = torch.tensor([[ctrl]], dtype=torch.int64, device=DEV)
        sl = torch.tensor([T], dtype=torch.int32, device=DEV)
        pos = sl.clone()
        lg = torch.full((1, vocab), 3.0, device=DEV)
        if which == "ref":
            ref.ref_capture_decode_step(c, k, v, sl, pos, lg)
        else:
            pkg.capture_decode_step.capture_decode(c, k, v, sl, pos, lg)
        torch.cuda.synchronize()
        outs.append((k.cpu(), v.cpu(), lg.cpu(), int(sl.item())))
    for a, b in zip(outs[0], outs[1]):
        if isinstance(a, int):
            assert a == b
        else:
            assert torch.equal(a, b)
