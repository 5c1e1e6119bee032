"""GPU parity at the exact workload shapes the benchmark times, against the fp32 oracle.

Shapes (the decode configurations of the benchmark, one layer each):
  gqa70b      batch 32, 64 query heads, 8 kv heads, head_dim 128, 4096 cached keys + 1 appended
  gqa70b_32k  batch 4, same heads, 32768 cached keys + 1 (split-KV across many CTAs)
  varlen7b    64 sequences with the benchmark's seeded lengths U[128, 8192] (seed 3), 32 heads,
              packed arena with cu_seqlens
  mha7b       one sequence, 32 heads, 512 cached keys + 1, as the reference's decode driver runs
              it (scripts/direct_custom_decode_500.py:229-250): through attn_varlen.decode, the
              reference surfaces attn_varlen.forward and capture_decode_step.capture_decode
and the prefill and the whole model step at their shapes:
  prefill16   the benchmark's 16 seeded prompt lengths U[256, 4096] (seed 5), on 2 of the 32 heads
              so that the CPU oracle stays cheap (per-head work is independent)
  llama7b     the full 32-layer Llama-2-7B shape, teacher-forced decode steps after a 16-token
              prompt; layers 0, 15 and 31 and the logits checked against the fp32 oracle from the
              GPU's own layer inputs

Every decode shape runs in split mode, then again as a CUDA-graph replay with the early reads
(prefetch_kv); the replays must equal the eager result bit for bit. Tolerances: ctx within
max-abs 2e-3 and relative-L2 1e-3 of the oracle; appended rows bit-exact with the RoPE formula
evaluated on the GPU; rows past each sequence are NaN so a leak shows.
"""
import math

import pytest
import torch

from oracle import decode_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def av():
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    return pkg.attn_varlen


def assert_close(got, want, what=""):
    max_abs, rel = O.compare(got.float().cpu(), want)
    assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL, f"{what}: max_abs={max_abs:.3g} rel_l2={rel:.3g}"


def varlen7b_lengths():
    g = torch.Generator().manual_seed(3)
    return torch.randint(128, 8193, (64,), generator=g).tolist()


def prefill16_lengths():
    g = torch.Generator().manual_seed(5)
    return torch.randint(256, 4097, (16,), generator=g).tolist()


SHAPES = {
    "gqa70b": dict(B=32, Hq=64, Hkv=8, lens=[4096] * 32, packed=False),
    "gqa70b_32k": dict(B=4, Hq=64, Hkv=8, lens=[32768] * 4, packed=False),
    "varlen7b": dict(B=64, Hq=32, Hkv=32, lens=None, packed=True),
    "mha7b": dict(B=1, Hq=32, Hkv=32, lens=[512], packed=False),
}


def make_decode_case(name, seed, D=128, slack=3):
    """Inputs generated on the device from a seed; rows at and past each T_b are NaN."""
    s = SHAPES[name]
    lens = s["lens"] if s["lens"] is not None else varlen7b_lengths()
    B, Hq, Hkv = len(lens), s["Hq"], s["Hkv"]
    g = torch.Generator(device=DEV).manual_seed(seed)
    rn = lambda *shape: torch.randn(*shape, generator=g, device=DEV, dtype=torch.float16)
    q, kn, vn = rn(B, Hq, D), rn(B, Hkv, D), rn(B, Hkv, D)
    if s["packed"]:
        caps = [t + 1 + slack for t in lens]
        cu = torch.tensor([0] + torch.tensor(caps).cumsum(0).tolist(), dtype=torch.int32)
        kc, vc = rn(Hkv, int(cu[-1]), D), rn(Hkv, int(cu[-1]), D)
        for b, t in enumerate(lens):
            kc[:, int(cu[b]) + t:int(cu[b + 1])] = float("nan")
            vc[:, int(cu[b]) + t:int(cu[b + 1])] = float("nan")
    else:
        cu = None
        cap = max(lens) + 1 + slack
        kc, vc = rn(B, Hkv, cap, D), rn(B, Hkv, cap, D)
        for b, t in enumerate(lens):
            kc[b, :, t:] = float("nan")
            vc[b, :, t:] = float("nan")
    return dict(q=q, kn=kn, vn=vn, kc=kc, vc=vc, lens=lens, cu=cu, T=torch.tensor(lens, dtype=torch.int32))


def check_appended_rows(case, k_after, v_after, what):
    """Appended K rows: bit-exact with the reference's fp32 RoPE formula on the device; V copied."""
    D = case["q"].shape[-1]
    for b, t in enumerate(case["lens"]):
        if case["cu"] is None:
            krow, vrow = k_after[b, :, t], v_after[b, :, t]
        else:
            row = int(case["cu"][b]) + t
            krow, vrow = k_after[:, row], v_after[:, row]
        assert torch.equal(krow, O.rope_rotate_half(case["kn"][b], t, D)), f"{what}: k row of sequence {b}"
        assert torch.equal(vrow, case["vn"][b]), f"{what}: v row of sequence {b}"


@pytest.mark.parametrize("name", ["gqa70b", "gqa70b_32k", "varlen7b", "mha7b"])
def test_decode_at_benchmark_shape(av, name):
    c = make_decode_case(name, seed={"gqa70b": 1, "gqa70b_32k": 2, "varlen7b": 3, "mha7b": 4}[name])
    B, Hq, D = c["q"].shape
    Hkv = c["kn"].shape[1]
    cu_dev = c["cu"].to(DEV) if c["cu"] is not None else None
    # the oracle works on host copies of the inputs taken before the kernel appends
    kc_h, vc_h = c["kc"].cpu(), c["vc"].cpu()
    want = O.decode_step(c["q"].cpu(), kc_h, vc_h, c["T"], k_new=c["kn"].cpu(), v_new=c["vn"].cpu(),
                         cu_seqlens=c["cu"], inplace=True)
    assert want["ok"].all()
    ws = av.make_workspace(B, Hq, Hkv, D)
    lens0 = c["T"].to(DEV)
    T = lens0.clone()
    out = torch.full((B, Hq, D), float("nan"), dtype=torch.float16, device=DEV)
    av.decode(c["q"], c["kc"], c["vc"], out, k_new=c["kn"], v_new=c["vn"], seq_lens=T, cu_seqlens=cu_dev,
              advance=True, workspace=ws, split=True)
    torch.cuda.synchronize()
    assert av.read_error(ws) == 0
    assert_close(out, want["ctx"], f"{name} split")
    assert T.cpu().tolist() == [t + 1 for t in c["lens"]]
    check_appended_rows(c, c["kc"], c["vc"], name)
    eager = out.clone()

    # the same step replayed from a CUDA graph with the early reads: the length is restored
    # by a copy inside the graph, so every replay repeats the step (the appended row is
    # rewritten with the same value)
    out.fill_(float("nan"))
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            T.copy_(lens0)
            av.decode(c["q"], c["kc"], c["vc"], out, k_new=c["kn"], v_new=c["vn"], seq_lens=T, cu_seqlens=cu_dev,
                      advance=True, workspace=ws, split=True, prefetch_kv=True)
    torch.cuda.synchronize()
    for rep in range(2):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager), f"{name}: graph replay {rep} with prefetch_kv differs from the eager step"
    assert av.read_error(ws) == 0
    assert T.cpu().tolist() == [t + 1 for t in c["lens"]]
    del g


def test_mha7b_through_the_reference_surfaces(av):
    """Config 1 as the reference's decode driver runs it: torch RoPE and append at T = 512,
    then attn_varlen.forward(q, K[:T+1], V[:T+1], T+1, 1/sqrt(D)); and the same step through
    capture_decode_step.capture_decode on the server's arena [L, 1, H, max_len, D]."""
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    c = make_decode_case("mha7b", seed=11)
    H, D, T = 32, 128, 512
    scale = 1.0 / math.sqrt(D)
    want = O.decode_step(c["q"].cpu(), c["kc"].cpu(), c["vc"].cpu(), c["T"], k_new=c["kn"].cpu(),
                         v_new=c["vn"].cpu(), scale=scale)
    # the driver's own steps around forward()
    qr = O.rope_rotate_half(c["q"][0], T, D)
    kr = O.rope_rotate_half(c["kn"][0], T, D)
    K = c["kc"][0].clone()
    V = c["vc"][0].clone()
    K[:, T] = kr
    V[:, T] = c["vn"][0]
    ctx = av.forward(qr, K[:, :T + 1].contiguous(), V[:, :T + 1].contiguous(), T + 1, scale)
    assert_close(ctx, want["ctx"][0], "forward")
    # the server's in-graph surface: layer 1 of a 2-layer arena with max_len 1024
    ak = torch.full((2, 1, H, 1024, D), float("nan"), dtype=torch.float16, device=DEV)
    avv = torch.full_like(ak, float("nan"))
    ak[1, 0, :, :T] = c["kc"][0, :, :T]
    avv[1, 0, :, :T] = c["vc"][0, :, :T]
    sl = torch.tensor([T], dtype=torch.int32, device=DEV)
    pos = torch.zeros(1, dtype=torch.int32, device=DEV)
    ctrl = torch.zeros(1, 1, dtype=torch.int64, device=DEV)
    logits = torch.zeros(1, 8, dtype=torch.float32, device=DEV)
    out = torch.empty(H, D, dtype=torch.float16, device=DEV)
    pkg.capture_decode_step.capture_decode(ctrl, ak, avv, sl, pos, logits, q=c["q"][0], k_new=c["kn"][0],
                                           v_new=c["vn"][0], ctx_out=out, layer=1, advance=True)
    torch.cuda.synchronize()
    assert_close(out, want["ctx"][0], "capture_decode")
    assert int(sl.item()) == T + 1
    assert torch.equal(ak[1, 0, :, T], kr) and torch.equal(avv[1, 0, :, T], c["vn"][0])


def test_prefill_at_benchmark_lengths(av):
    """The benchmark's 16 prompt lengths (seed 5), causal, RoPE, into an empty arena, on 2 heads."""
    lens = prefill16_lengths()
    Hq = Hkv = 2
    D = 128
    B = len(lens)
    cap = (max(lens) + 127) // 128 * 128
    total = sum(lens)
    g = torch.Generator(device=DEV).manual_seed(55)
    rn = lambda *shape: torch.randn(*shape, generator=g, device=DEV, dtype=torch.float16)
    q, kn, vn = rn(total, Hq, D), rn(total, Hkv, D), rn(total, Hkv, D)
    kc = torch.full((B, Hkv, cap, D), float("nan"), dtype=torch.float16, device=DEV)
    vc = torch.full_like(kc, float("nan"))
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32)
    T = torch.zeros(B, dtype=torch.int32, device=DEV)
    out = torch.full((total, Hq, D), float("nan"), dtype=torch.float16, device=DEV)
    want = O.prefill_step(q.cpu(), kn.cpu(), vn.cpu(), kc.cpu(), vc.cpu(), cu, torch.zeros(B, dtype=torch.int32))
    av.prefill_varlen(q, kn, vn, kc, vc, out, cu.to(DEV), max(lens), seq_lens=T, advance=True)
    torch.cuda.synchronize()
    assert_close(out, want["out"], "prefill16 lengths")
    assert T.cpu().tolist() == lens
    for b in range(B):
        r0, r1 = int(cu[b]), int(cu[b + 1])
        k_dev = O.rope_positions(kn[r0:r1], torch.arange(r1 - r0), D).permute(1, 0, 2)
        assert torch.equal(kc[b, :, :r1 - r0], k_dev), f"appended keys of prompt {b}"
        assert torch.equal(vc[b, :, :r1 - r0], vn[r0:r1].permute(1, 0, 2)), f"appended values of prompt {b}"


def _oracle_layer(w, l, x_in, k_rows, v_rows, T):
    """fp32 oracle of one decoder layer for one token at position T: RMSNorm, QKV, RoPE,
    attention over the cached rows [0, T) plus the new row, O projection + residual,
    RMSNorm, SwiGLU MLP + residual (the model of llama_oracle, one step)."""
    from oracle import llama_oracle as LO

    s = w.shape
    f = lambda t: t.detach().float().cpu()
    Hq, Hkv, D, I = s.heads, s.kv_heads, s.head_dim, s.intermediate
    x = f(x_in)
    h = LO.rms(x, f(w.rms_in[l]), s.eps)
    qkv = h @ f(w.w_qkv[l]).t()
    q = O.rope_rotate_half(qkv[: Hq * D].view(Hq, D), T, D, s.rope_theta)
    k = O.rope_rotate_half(qkv[Hq * D:(Hq + Hkv) * D].view(Hkv, D), T, D, s.rope_theta)
    v = qkv[(Hq + Hkv) * D:].view(Hkv, D)
    K = torch.cat([f(k_rows[:, :T]), k.unsqueeze(1)], dim=1)
    V = torch.cat([f(v_rows[:, :T]), v.unsqueeze(1)], dim=1)
    ctx = O.attention(q, K, V, 1.0 / math.sqrt(D)).reshape(-1)
    x = x + ctx @ f(w.w_o[l]).t()
    h = LO.rms(x, f(w.rms_post[l]), s.eps)
    gu = h @ f(w.w_gu[l]).t()
    x = x + (torch.nn.functional.silu(gu[:I]) * gu[I:]) @ f(w.w_down[l]).t()
    return qkv, x


def test_llama7b_full_shape_layers_against_oracle():
    """The whole 32-layer Llama-2-7B-shaped step (fused projections, decode attention), two
    teacher-forced tokens after a 16-token prompt. For layers 0, 15 and 31 the GPU's own layer
    input is run through the fp32 oracle layer: QKV within relative-L2 3e-3, the attention
    output within the decode tolerance of the oracle attention on the GPU's q/k/v, and the
    layer's update of the residual within relative-L2 1e-2; the logits within relative-L2
    3e-3 of the oracle on the GPU's final residual."""
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import LLAMA2_7B, GreedyDecoder, LlamaWeights
    from oracle import llama_oracle as LO

    s = LLAMA2_7B
    w = LlamaWeights(s, seed=21)
    dec = GreedyDecoder(w, capacity=32, max_new_tokens=8)
    gen = torch.Generator().manual_seed(22)
    prompt = torch.randint(0, s.vocab, (16,), generator=gen).cuda()
    forced = torch.randint(0, s.vocab, (2,), generator=gen).tolist()
    dec.arena.seq_lens.zero_()
    dec.prefill(prompt)
    Hq, Hkv, D = s.heads, s.kv_heads, s.head_dim
    check = (0, 15, s.layers - 1)
    for step, tok in enumerate(forced):
        T = int(dec.arena.seq_lens.item())
        assert T == 16 + step
        dec.token.fill_(tok)
        torch.index_select(w.embed, 0, dec.token, out=dec.x.view(1, -1))
        rec = {}
        for l in range(s.layers):
            x_in = dec.x.clone() if l in check else None
            dec._layer(l)
            if l in check:
                rec[l] = (x_in, dec.qkv.clone(), dec.ctx.clone(), dec.x.clone())
        torch.cuda.synchronize()
        assert int(dec.arena.seq_lens.item()) == T + 1
        for l, (x_in, qkv, ctx, x_out) in rec.items():
            kl, vl = dec.arena.layer(l)
            qkv_ref, x_ref = _oracle_layer(w, l, x_in, kl[0, :, :T + 1], vl[0, :, :T + 1], T)
            _, rel = O.compare(qkv.float(), qkv_ref)
            assert rel <= 3e-3, f"step {step} layer {l}: qkv rel_l2={rel:.3g}"
            # attention on the GPU's own q/k/v against the oracle attention step
            q = qkv[: Hq * D].view(1, Hq, D).cpu()
            kn = qkv[Hq * D:(Hq + Hkv) * D].view(1, Hkv, D).cpu()
            vn = qkv[(Hq + Hkv) * D:].view(1, Hkv, D).cpu()
            want = O.decode_step(q, kl[:, :, :T + 1].cpu(), vl[:, :, :T + 1].cpu(), torch.tensor([T]),
                                 k_new=kn, v_new=vn, capacity=T + 1)
            assert_close(ctx.view(1, Hq, D), want["ctx"], f"step {step} layer {l} attention")
            upd_gpu = x_out.float().cpu() - x_in.float().cpu()
            upd_ref = x_ref - x_in.float().cpu()
            rel = float((upd_gpu - upd_ref).norm() / upd_ref.norm())
            assert rel <= 1e-2, f"step {step} layer {l}: residual update rel_l2={rel:.3g}"
        from fully_custom_cuda_inference_lamma2_b200 import capture_decode_step as cds

        cds.gemv_fused(w.embed, dec.x, dec.logits, "store", w.rms_final, s.eps)
        torch.cuda.synchronize()
        ref = LO.rms(dec.x.float().cpu(), w.rms_final.float().cpu(), s.eps) @ w.embed.float().cpu().t()
        rel = float((dec.logits.float().cpu() - ref).norm() / ref.norm())
        assert rel <= 3e-3, f"step {step}: logits rel_l2={rel:.3g}"
