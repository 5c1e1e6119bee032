"""GPU tests of the `capture_decode_step` surface: the reference's placeholder
step (identical results), the attention step added through keyword arguments,
and its use inside one CUDA graph across many sequence lengths."""
import math

import pytest
import torch

from helpers import fp16_ulp_diff, randn_half
from oracle import decode_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def cds():
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    return pkg.capture_decode_step


@pytest.fixture(scope="module")
def av():
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    return pkg.attn_varlen


def assert_close(got, want, what=""):
    max_abs, rel = O.compare(got.float().cpu(), want)
    assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL, f"{what}: max_abs={max_abs:.3g} rel_l2={rel:.3g}"


@pytest.mark.parametrize("T,ctrl", [(5, 1234567), (0, 3), (15, -7), (16, 99)])
def test_placeholder_step_matches_reference_semantics(cds, T, ctrl):
    L, H, max_len, D, vocab = 3, 4, 16, 128, 1000
    ak = randn_half((L, 1, H, max_len, D), 11)
    av_ = randn_half((L, 1, H, max_len, D), 12)
    dk, dv = ak.to(DEV), av_.to(DEV)
    c = torch.tensor([[ctrl]], dtype=torch.int64, device=DEV)
    sl = torch.tensor([T], dtype=torch.int32, device=DEV)
    pos = torch.tensor([T], dtype=torch.int32, device=DEV)
    logits = torch.full((1, vocab), 7.0, device=DEV)
    cds.capture_decode(c, dk, dv, sl, pos, logits)
    torch.cuda.synchronize()
    wk, wv, wl, wT = O.placeholder_step(ctrl, ak, av_, T, vocab)
    assert torch.equal(dk.cpu(), wk) and torch.equal(dv.cpu(), wv)
    assert torch.equal(logits.cpu(), wl)
    assert int(sl.item()) == wT


def test_capture_decode_ext_without_weights(cds):
    L, H, max_len, D, vocab, I = 2, 4, 8, 128, 64, 32
    ak = torch.zeros(L, 1, H, max_len, D, dtype=torch.float16, device=DEV)
    c = torch.zeros(1, 1, dtype=torch.int64, device=DEV)
    sl = torch.tensor([3], dtype=torch.int32, device=DEV)
    pos = sl.clone()
    logits = torch.full((1, vocab), 5.0, device=DEV)
    scr = [torch.full((n,), 1.0, dtype=torch.float16, device=DEV) for n in (H * D, I, I, I, H * D)]
    cds.capture_decode_ext(c, ak, ak.clone(), sl, pos, logits, *scr, 0, 0, 0, 0, 0, 0, 0, I, 1e-5)
    torch.cuda.synchronize()
    assert int(sl.item()) == 4
    assert torch.count_nonzero(logits) == 0
    # as in the reference, `H` of the _ext step is the arena's head count
    # (capture_decode_step.cpp:104): x_norm/mlp_out are zeroed over H entries, gate/up/act over I
    for s, n in zip(scr, (H, I, I, I, H)):
        assert torch.count_nonzero(s[:n]) == 0 and torch.count_nonzero(s[n:]) == s.numel() - n


def test_attention_step_per_layer_with_advance_on_last(cds):
    L, Hkv, G, max_len, D = 3, 4, 2, 256, 128
    Hq = Hkv * G
    T = 100
    ak = randn_half((L, 1, Hkv, max_len, D), 21)
    av_ = randn_half((L, 1, Hkv, max_len, D), 22)
    dk, dv = ak.to(DEV), av_.to(DEV)
    sl = torch.tensor([T], dtype=torch.int32, device=DEV)
    c = torch.zeros(1, 1, dtype=torch.int64, device=DEV)
    logits = torch.zeros(1, 10, device=DEV)
    for l in range(L):
        q = randn_half((Hq * D,), 30 + l)
        kn = randn_half((Hkv * D,), 40 + l)
        vn = randn_half((Hkv * D,), 50 + l)
        ctx = torch.empty(Hq * D, dtype=torch.float16, device=DEV)
        cds.capture_decode(c, dk, dv, sl, sl, logits, q=q.to(DEV), k_new=kn.to(DEV), v_new=vn.to(DEV),
                           ctx_out=ctx, layer=l, advance=(l == L - 1))
        torch.cuda.synchronize()
        want = O.decode_step(q.view(1, Hq, D), ak[l, 0:1], av_[l, 0:1], torch.tensor([T], dtype=torch.int32),
                             k_new=kn.view(1, Hkv, D), v_new=vn.view(1, Hkv, D))
        assert_close(ctx.view(1, Hq, D), want["ctx"], f"layer {l}")
        dev_rot = O.rope_rotate_half(kn.view(Hkv, D).to(DEV), T, D).cpu()
        assert torch.equal(dk.cpu()[l, 0, :, T], dev_rot)
        assert float((dk.cpu()[l, 0, :, T].float() - want["k_cache"][0, :, T].float()).abs().max()) <= 2e-3
        assert torch.equal(dv.cpu()[l, 0, :, T], want["v_cache"][0, :, T])
        assert int(sl.item()) == (T + 1 if l == L - 1 else T)
    assert torch.count_nonzero(logits) == 0  # the attention step leaves logits alone


def test_one_graph_serves_every_length(cds, av):
    """Capture the per-layer attention steps of a whole token once; replay it as T grows."""
    L, Hkv, G, max_len, D = 2, 2, 4, 128, 128
    Hq = Hkv * G
    T0 = 50
    ak = randn_half((L, 1, Hkv, max_len, D), 61)
    av_ = randn_half((L, 1, Hkv, max_len, D), 62)
    dk, dv = ak.to(DEV), av_.to(DEV)
    sl = torch.tensor([T0], dtype=torch.int32, device=DEV)
    c = torch.zeros(1, 1, dtype=torch.int64, device=DEV)
    logits = torch.zeros(1, 10, device=DEV)
    sq = torch.empty(L, Hq * D, dtype=torch.float16, device=DEV)
    skn = torch.empty(L, Hkv * D, dtype=torch.float16, device=DEV)
    svn = torch.empty_like(skn)
    ctx = torch.empty(L, Hq * D, dtype=torch.float16, device=DEV)
    ws = av.make_workspace(1, Hq, Hkv, D)

    def step():
        for l in range(L):
            cds.capture_decode(c, dk, dv, sl, sl, logits, q=sq[l], k_new=skn[l], v_new=svn[l], ctx_out=ctx[l],
                               layer=l, advance=(l == L - 1), workspace=ws)

    # warm-up on copies so the real arena and seq_len stay at T0
    saved = (dk.clone(), dv.clone(), sl.clone())
    step()
    torch.cuda.synchronize()
    dk.copy_(saved[0]); dv.copy_(saved[1]); sl.copy_(saved[2])
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            step()
    torch.cuda.synchronize()
    rk, rv, rT = ak.clone(), av_.clone(), T0
    mem0 = torch.cuda.memory_allocated()
    for it in range(5):
        qs = [randn_half((Hq * D,), 100 + 10 * it + l) for l in range(L)]
        kns = [randn_half((Hkv * D,), 200 + 10 * it + l) for l in range(L)]
        vns = [randn_half((Hkv * D,), 300 + 10 * it + l) for l in range(L)]
        for l in range(L):
            sq[l].copy_(qs[l]); skn[l].copy_(kns[l]); svn[l].copy_(vns[l])
        g.replay()
        torch.cuda.synchronize()
        for l in range(L):
            want = O.decode_step(qs[l].view(1, Hq, D), rk[l, 0:1], rv[l, 0:1], torch.tensor([rT], dtype=torch.int32),
                                 k_new=kns[l].view(1, Hkv, D), v_new=vns[l].view(1, Hkv, D))
            assert_close(ctx[l].view(1, Hq, D), want["ctx"], f"replay {it} layer {l}")
            rk[l, 0] = want["k_cache"][0]
            rv[l, 0] = want["v_cache"][0]
        rT += 1
        assert int(sl.item()) == rT
    assert torch.cuda.memory_allocated() == mem0
    assert av.read_error(ws) == 0


def test_gemv_helpers_match_torch(cds):
    H, I, V = 256, 512, 1000
    x = randn_half((H,), 71).to(DEV)
    wg = (randn_half((I, H), 72) * 0.05).to(DEV)
    wu = (randn_half((I, H), 73) * 0.05).to(DEV)
    wd = (randn_half((H, I), 74) * 0.05).to(DEV)
    wv = (randn_half((V, H), 75) * 0.05).to(DEV)
    g = torch.empty(I, dtype=torch.float16, device=DEV)
    u = torch.empty_like(g)
    cds.gate_up_gemm(x, g, u, wg.data_ptr(), wu.data_ptr(), H, I)
    a = torch.empty_like(g)
    cds.swiglu(g, u, a)
    o = torch.empty(H, dtype=torch.float16, device=DEV)
    cds.down_gemm(a, o, wd.data_ptr(), I, H)
    lg = torch.empty(V, dtype=torch.float32, device=DEV)
    cds.logits_gemm_vocab(x, lg, wv.data_ptr(), H, V)
    rw = torch.ones(H, dtype=torch.float16, device=DEV)
    y = torch.empty_like(x)
    cds.rmsnorm(x, rw, y, 1e-5)
    torch.cuda.synchronize()
    xf = x.float()
    gf, uf = wg.float() @ xf, wu.float() @ xf
    assert torch.allclose(g.float(), gf, atol=2e-2, rtol=1e-2)
    assert torch.allclose(u.float(), uf, atol=2e-2, rtol=1e-2)
    af = torch.nn.functional.silu(g.float()) * u.float()
    assert torch.allclose(a.float(), af, atol=1e-2, rtol=1e-2)
    assert torch.allclose(o.float(), wd.float() @ a.float(), atol=2e-2, rtol=1e-2)
    assert torch.allclose(lg, wv.float() @ xf, atol=2e-2, rtol=1e-2)
    yf = xf * torch.rsqrt(xf.pow(2).mean() + 1e-5)
    assert torch.allclose(y.float(), yf, atol=1e-2, rtol=1e-2)
