"""GPU parity of the decode-attention path against the fp32 oracle.

Tolerances: ctx within max-abs 2e-3 and relative-L2 1e-3 of the fp32 oracle
(fp16 inputs and output). Rotated q and appended K rows bit-exact with the
reference driver's RoPE formula evaluated by torch on the GPU (where the
reference evaluates it), and within 2e-3 of the CPU oracle, whose powf/cosf/sinf
differ from the GPU's in the last fp32 bits. Appended V rows and untouched arena
rows bit-exact.
"""
import gc
import math

import pytest
import torch

from helpers import fp16_ulp_diff, randn_half
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


def rope_on_device(x, pos, rot, theta=10000.0):
    """The reference driver's RoPE evaluated by torch on the GPU, where the reference runs it."""
    return O.rope_rotate_half(x.to(DEV), pos, rot, theta).cpu()


def assert_rope(got, x, pos, rot, theta=10000.0, what=""):
    """Rotated fp16 rows: bit-exact with the reference formula on the device, and within
    2e-3 of the CPU oracle (the CPU's powf/cosf/sinf differ from the GPU's in the last bits)."""
    dev = rope_on_device(x, pos, rot, theta)
    assert torch.equal(got, dev), f"{what}: {fp16_ulp_diff(got, dev)} ulp from the device formula"
    cpu = O.rope_rotate_half(x, pos, rot, theta)
    assert float((got.float() - cpu.float()).abs().max()) <= O.MAX_ABS_TOL, what


# ------------------------------------------------------------------ forward (reference surface)

@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 513, 4097])
def test_forward_matches_oracle(av, T):
    H, D = 32, 128
    q = randn_half((H, D), 1)
    k = randn_half((H, T, D), 2)
    v = randn_half((H, T, D), 3)
    scale = 1.0 / math.sqrt(D)
    ctx = av.forward(q.to(DEV), k.to(DEV), v.to(DEV), T, scale)
    torch.cuda.synchronize()
    assert ctx.shape == (H, D) and ctx.dtype == torch.float16
    assert_close(ctx, O.attn_varlen_forward(q, k, v, T, scale), f"T={T}")


@pytest.mark.parametrize("D", [64, 256])
def test_forward_head_dims(av, D):
    H, T = 8, 300
    q, k, v = randn_half((H, D), 4), randn_half((H, T, D), 5), randn_half((H, T, D), 6)
    scale = 1.0 / math.sqrt(D)
    ctx = av.forward(q.to(DEV), k.to(DEV), v.to(DEV), T, scale)
    assert_close(ctx, O.attn_varlen_forward(q, k, v, T, scale), f"D={D}")


def test_forward_honours_strides_and_seq_len(av):
    # a slice of an arena [H, max_len, D]: row stride D, head stride max_len*D,
    # attended over seq_len < k.size(1) (the reference needed exact copies here)
    H, D, max_len, T, seq_len = 16, 128, 1024, 700, 333
    arena_k = randn_half((H, max_len, D), 7)
    arena_v = randn_half((H, max_len, D), 8)
    q = randn_half((H, D), 9)
    k = arena_k.to(DEV)[:, :T]
    v = arena_v.to(DEV)[:, :T]
    assert not k.is_contiguous()
    ctx = av.forward(q.to(DEV), k, v, seq_len, 0.0883883)
    assert_close(ctx, O.attn_varlen_forward(q, arena_k[:, :T], arena_v[:, :T], seq_len, 0.0883883), "strided")


def test_forward_out_no_alloc_with_workspace(av):
    H, D, T = 32, 128, 2000
    q, k, v = randn_half((H, D), 10).to(DEV), randn_half((H, T, D), 11).to(DEV), randn_half((H, T, D), 12).to(DEV)
    out = torch.empty(H, D, dtype=torch.float16, device=DEV)
    ws = av.make_workspace(1, H, H, D)
    av.forward_out(q, k, v, T, 0.0883883, out, ws)  # warm up (first launch sets kernel attributes)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    av.forward_out(q, k, v, T, 0.0883883, out, ws)
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == before
    assert_close(out, O.attn_varlen_forward(q.cpu(), k.cpu(), v.cpu(), T, 0.0883883), "forward_out")


def test_repeated_reference_calls_neither_allocate_nor_memset(av):
    """forward() past 256 keys and capture_decode(..., q=...) without a workspace reuse one
    zeroed workspace per (device, stream, shape): after the first call, further calls
    change torch.cuda.memory_allocated() by the returned ctx alone and issue no memset."""
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    H, D, T = 32, 128, 2000
    q, k, v = randn_half((H, D), 13).to(DEV), randn_half((H, T, D), 14).to(DEV), randn_half((H, T, D), 15).to(DEV)
    first = av.forward(q, k, v, T, 0.0883883)
    ak = randn_half((1, 1, H, 600, D), 16).to(DEV)
    avv = randn_half((1, 1, H, 600, D), 17).to(DEV)
    sl = torch.tensor([500], dtype=torch.int32, device=DEV)
    z32 = torch.zeros(1, dtype=torch.int32, device=DEV)
    ctrl = torch.zeros(1, 1, dtype=torch.int64, device=DEV)
    logits = torch.zeros(1, 8, device=DEV)
    kn, vn, ctx = torch.zeros(H, D, dtype=torch.float16, device=DEV), torch.zeros_like(q), torch.empty_like(q)
    cds = pkg.capture_decode_step
    cds.capture_decode(ctrl, ak, avv, sl, z32, logits, q=q, k_new=kn, v_new=vn, ctx_out=ctx, advance=False)
    torch.cuda.synchronize()
    # Tensors of earlier tests held by reference cycles (a failed test's traceback frames)
    # would otherwise be freed by a collection inside the measured loop.
    gc.collect()
    gc.disable()
    try:
        before = torch.cuda.memory_allocated()
        kept = []
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(4):
                kept.append(av.forward(q, k, v, T, 0.0883883))
                cds.capture_decode(ctrl, ak, avv, sl, z32, logits, q=q, k_new=kn, v_new=vn, ctx_out=ctx,
                                   advance=False)
            torch.cuda.synchronize()
        grown = torch.cuda.memory_allocated() - before
    finally:
        gc.enable()
    assert grown == sum(t.numel() * 2 for t in kept)
    names = [e.name for e in prof.events()]
    assert any("decode_attn_kernel" in n for n in names), "profiler recorded no kernels"
    assert not any("memset" in n.lower() for n in names), "a memset ran inside the repeated calls"
    assert all(torch.equal(t, first) for t in kept)


def test_forward_rejects_bad_inputs(av):
    q = torch.zeros(4, 128, dtype=torch.float16, device=DEV)
    k = torch.zeros(4, 10, 128, dtype=torch.float16, device=DEV)
    with pytest.raises(RuntimeError, match="invalid seq_len"):
        av.forward(q, k, k, 11, 1.0)
    with pytest.raises(RuntimeError, match="invalid seq_len"):
        av.forward(q, k, k, 0, 1.0)
    with pytest.raises(RuntimeError, match="fp16"):
        av.forward(q.float(), k, k, 5, 1.0)
    with pytest.raises(RuntimeError, match="head mismatch"):
        av.forward(q[:3], k, k, 5, 1.0)
    with pytest.raises(RuntimeError, match="must be CUDA"):
        av.forward(q.cpu(), k, k, 5, 1.0)


# ------------------------------------------------------------------ batched / varlen decode step

def make_case(B, Hkv, G, D, lens, cap, seed, packed=False, slack=5):
    """Seeded decode inputs; rows past each sequence's T are NaN so any leak shows."""
    Hq = Hkv * G
    q = randn_half((B, Hq, D), seed)
    k_new = randn_half((B, Hkv, D), seed + 1)
    v_new = randn_half((B, Hkv, D), seed + 2)
    if packed:
        caps = [t + 1 + slack for t in lens]
        cu = torch.tensor([0] + list(torch.tensor(caps).cumsum(0)), dtype=torch.int32)
        total = int(cu[-1])
        kc = randn_half((Hkv, total, D), seed + 3)
        vc = randn_half((Hkv, total, D), seed + 4)
        for b, t in enumerate(lens):
            kc[:, int(cu[b]) + t:int(cu[b + 1])] = float("nan")
            vc[:, int(cu[b]) + t:int(cu[b + 1])] = float("nan")
    else:
        cu = None
        kc = randn_half((B, Hkv, cap, D), seed + 3)
        vc = randn_half((B, Hkv, cap, D), seed + 4)
        for b, t in enumerate(lens):
            kc[b, :, t:] = float("nan")
            vc[b, :, t:] = float("nan")
    return q, k_new, v_new, kc, vc, torch.tensor(lens, dtype=torch.int32), cu


def run_decode(av, q, k_new, v_new, kc, vc, lens, cu, *, split=True, advance=True, q_rot=True):
    B, Hq, D = q.shape
    dk, dv = kc.to(DEV), vc.to(DEV)
    dlens = lens.to(DEV)
    out = torch.full((B, Hq, D), float("nan"), dtype=torch.float16, device=DEV)
    qr = torch.empty_like(q, device=DEV) if q_rot else None
    ws = av.make_workspace(B, Hq, kc.shape[1] if cu is None else kc.shape[0], D)
    av.decode(q.to(DEV), dk, dv, out, k_new=k_new.to(DEV) if k_new is not None else None,
              v_new=v_new.to(DEV) if v_new is not None else None, seq_lens=dlens,
              cu_seqlens=cu.to(DEV) if cu is not None else None, advance=advance, workspace=ws,
              q_rot_out=qr, split=split)
    torch.cuda.synchronize()
    err = av.read_error(ws)
    return dict(out=out.cpu(), q_rot=qr.cpu() if qr is not None else None, k=dk.cpu(), v=dv.cpu(),
                lens=dlens.cpu(), err=err)


@pytest.mark.parametrize("G", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("split", [True, False])
def test_decode_batched_append_gqa(av, G, split):
    B, Hkv, D, cap = 4, 2, 128, 400
    lens = [0, 70, 255, 398]
    q, kn, vn, kc, vc, T, cu = make_case(B, Hkv, G, D, lens, cap, seed=100 + G)
    got = run_decode(av, q, kn, vn, kc, vc, T, cu, split=split)
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn)
    assert got["err"] == 0
    assert_close(got["out"], want["ctx"], f"G={G} split={split}")
    for b, t in enumerate(lens):
        assert_rope(got["q_rot"][b], q[b], t, D, what=f"q_rot b={b}")
        assert_rope(got["k"][b, :, t], kn[b], t, D, what=f"k row b={b}")
        assert torch.equal(got["v"][b, :, t], want["v_cache"][b, :, t])
        assert torch.equal(got["k"][b, :, :t], kc[b, :, :t])  # cached rows untouched
    assert got["lens"].tolist() == [t + 1 for t in lens]


@pytest.mark.parametrize("split", [True, False])
def test_decode_packed_varlen(av, split):
    # ragged lengths including the one-key sequence (T=0) and tile edges
    lens = [0, 1, 15, 16, 17, 63, 64, 65, 127, 128, 129, 1000, 3]
    B, Hkv, G, D = len(lens), 4, 8, 128
    q, kn, vn, kc, vc, T, cu = make_case(B, Hkv, G, D, lens, None, seed=200, packed=True)
    got = run_decode(av, q, kn, vn, kc, vc, T, cu, split=split)
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn, cu_seqlens=cu)
    assert got["err"] == 0
    assert_close(got["out"], want["ctx"], f"packed split={split}")
    for b, t in enumerate(lens):
        row = int(cu[b]) + t
        assert_rope(got["q_rot"][b], q[b], t, D, what=f"q_rot b={b}")
        assert_rope(got["k"][:, row], kn[b], t, D, what=f"k row b={b}")
        assert torch.equal(got["v"][:, row], want["v_cache"][:, row])
    assert got["lens"].tolist() == [t + 1 for t in lens]


def test_decode_attention_only(av):
    # no append: attend to the first T_b keys with q as given (no RoPE)
    lens = [1, 64, 500, 77]
    B, Hkv, G, D, cap = 4, 8, 8, 128, 512
    q, _, _, kc, vc, T, cu = make_case(B, Hkv, G, D, lens, cap, seed=300)
    got = run_decode(av, q, None, None, kc, vc, T, cu, advance=False, q_rot=False)
    want = O.decode_step(q, kc, vc, T)
    assert got["err"] == 0
    assert_close(got["out"], want["ctx"], "attention-only")
    assert got["lens"].tolist() == lens


def test_decode_long_split_kv(av):
    # one long sequence per kv head pair: the stream-K split cuts every pair
    lens = [32768, 20000]
    B, Hkv, G, D, cap = 2, 8, 8, 128, 32800
    q, kn, vn, kc, vc, T, cu = make_case(B, Hkv, G, D, lens, cap, seed=400)
    got = run_decode(av, q, kn, vn, kc, vc, T, cu)
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn)
    assert got["err"] == 0
    assert_close(got["out"], want["ctx"], "split-kv 32k")


@pytest.mark.parametrize("max_cluster", [0, 8, 2, 1])
@pytest.mark.parametrize("B,Hkv,G,T", [(32, 1, 8, 4095), (32, 2, 8, 4095), (1, 32, 1, 1000), (4, 8, 8, 4095)])
def test_decode_few_pairs_cluster_and_stream_k(av, B, Hkv, G, T, max_cluster):
    """Few (sequence, kv head) pairs: the split grid is launched as one thread-block cluster
    per pair (up to max_cluster CTAs; 0 = automatic, 1 = no clusters). With uniform lengths
    the CTAs of a cluster split the pair's tiles and merge their pieces through distributed
    shared memory; calls alternate with ragged lengths (stream-K pieces, last-arriver merge)
    on one workspace, so the pair counters must come back to zero."""
    D, cap = 128, T + 8
    ws = av.make_workspace(B, Hkv * G, Hkv, D)
    av.set_tuning(max_cluster=max_cluster)
    try:
        for i, lens in enumerate([[T] * B, [max(1, T - 977 * b % T) for b in range(B)], [T] * B]):
            q, kn, vn, kc, vc, lt, _ = make_case(B, Hkv, G, D, lens, cap, seed=700 + i)
            dk, dv, dl = kc.to(DEV), vc.to(DEV), lt.to(DEV)
            out = torch.full((B, Hkv * G, D), float("nan"), dtype=torch.float16, device=DEV)
            av.decode(q.to(DEV), dk, dv, out, k_new=kn.to(DEV), v_new=vn.to(DEV), seq_lens=dl, advance=True,
                      workspace=ws, split=True)
            torch.cuda.synchronize()
            assert av.read_error(ws) == 0
            want = O.decode_step(q, kc, vc, lt, k_new=kn, v_new=vn)
            assert_close(out.cpu(), want["ctx"], f"B={B} Hkv={Hkv} G={G} max_cluster={max_cluster} call {i}")
            assert dl.cpu().tolist() == [t + 1 for t in lens]
    finally:
        av.set_tuning()


@pytest.mark.parametrize("T", [0, 63, 64, 100, 700])
def test_decode_cluster_short_pairs(av, T):
    """Pairs of 1 to 12 tiles in a cluster launch: k_eff = min(k, tiles) CTAs carry the
    pair (one tile each at most), the others only join the cluster barriers."""
    B, Hkv, G, D = 2, 8, 8, 128
    q, kn, vn, kc, vc, lt, _ = make_case(B, Hkv, G, D, [T] * B, T + 4, seed=750 + T)
    got = run_decode(av, q, kn, vn, kc, vc, lt, None)
    want = O.decode_step(q, kc, vc, lt, k_new=kn, v_new=vn)
    assert got["err"] == 0
    assert_close(got["out"], want["ctx"], f"T={T}")
    assert got["lens"].tolist() == [T + 1] * B


@pytest.mark.parametrize("split", [True, False])
def test_early_read_guard_reports_a_broken_contract(av, split):
    """FCCI_DECODE_PREFETCH_KV lets a launch read the lengths before the kernel ahead of it on
    the stream has finished; the caller promises that no such kernel writes them. Here the
    kernel ahead breaks that promise on purpose: a decode step that advances the very lengths
    the next (early-reading) step uses. With the check on (FCCI_DECODE_CHECK_EARLY_READ),
    whatever the timing, the second step must never be silently wrong: if its ctx differs
    from the step at the advanced lengths, its error word carries FCCI_DEV_ERR_EARLY_READ (4);
    without the bit, its ctx is the right one."""
    B, Hkv, G, D, T = 32, 8, 8, 128, 1000
    qa, kna, vna, kca, vca, lens, _ = make_case(B, Hkv, G, D, [T] * B, T + 8, seed=1200)
    qb = randn_half((B, Hkv * G, D), 1210)
    kcb, vcb = randn_half((B, Hkv, T + 8, D), 1211), randn_half((B, Hkv, T + 8, D), 1212)
    want = O.decode_step(qb, kcb, vcb, torch.tensor([T + 1] * B, dtype=torch.int32))["ctx"]
    dqa, dkna, dvna, dqb = qa.to(DEV), kna.to(DEV), vna.to(DEV), qb.to(DEV)
    dkcb, dvcb = kcb.to(DEV), vcb.to(DEV)
    flagged = 0
    for trial in range(8):
        dka, dva = kca.to(DEV), vca.to(DEV)
        seq = lens.to(DEV)
        wsa, wsb = av.make_workspace(B, Hkv * G, Hkv, D), av.make_workspace(B, Hkv * G, Hkv, D)
        out_a = torch.empty(B, Hkv * G, D, dtype=torch.float16, device=DEV)
        out_b = torch.full((B, Hkv * G, D), float("nan"), dtype=torch.float16, device=DEV)
        torch.cuda.synchronize()
        av.decode(dqa, dka, dva, out_a, k_new=dkna, v_new=dvna, seq_lens=seq, advance=True, workspace=wsa,
                  split=True)
        av.decode(dqb, dkcb, dvcb, out_b, seq_lens=seq, workspace=wsb, split=split, prefetch_kv=True,
                  check_early_read=True)
        torch.cuda.synchronize()
        err = av.read_error(wsb)
        max_abs, rel = O.compare(out_b.float().cpu(), want)
        right = max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL
        assert right or (err & 4), f"trial {trial}: stale lengths used silently (max_abs={max_abs:.3g})"
        flagged += bool(err & 4)
        assert seq.cpu().tolist() == [T + 1] * B
    print(f"split={split}: {flagged} of 8 steps read stale lengths and reported it")


def test_decode_capacity_overflow_sets_error(av):
    lens = [10, 400, 20]  # 400 + 1 > cap 400
    B, Hkv, G, D, cap = 3, 2, 4, 128, 400
    q, kn, vn, kc, vc, T, cu = make_case(B, Hkv, G, D, lens, cap, seed=500)
    got = run_decode(av, q, kn, vn, kc, vc, T, cu)
    assert got["err"] & 1
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn)
    assert not bool(want["ok"][1])
    assert torch.count_nonzero(got["out"][1]) == 0
    assert_close(got["out"][[0, 2]], want["ctx"][[0, 2]], "valid sequences")
    assert got["lens"].tolist() == [11, 400, 21]


@pytest.mark.parametrize("rotary_dim", [0, 64])
def test_decode_partial_rotary(av, rotary_dim):
    lens = [5, 300]
    B, Hkv, G, D, cap = 2, 2, 4, 128, 320
    q, kn, vn, kc, vc, T, cu = make_case(B, Hkv, G, D, lens, cap, seed=600)
    dk, dv = kc.to(DEV), vc.to(DEV)
    out = torch.empty(B, Hkv * G, D, dtype=torch.float16, device=DEV)
    av.decode(q.to(DEV), dk, dv, out, k_new=kn.to(DEV), v_new=vn.to(DEV), seq_lens=T.to(DEV),
              rotary_dim=rotary_dim, rope_theta=500000.0)
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn, rotary_dim=rotary_dim, theta=500000.0)
    assert_close(out, want["ctx"], f"rotary_dim={rotary_dim}")


def test_rope_append_standalone(av):
    lens = [0, 9, 130]
    B, Hkv, G, D, cap = 3, 4, 2, 128, 200
    q, kn, vn, kc, vc, T, cu = make_case(B, Hkv, G, D, lens, cap, seed=700)
    dk, dv, dT = kc.to(DEV), vc.to(DEV), T.to(DEV)
    qr = torch.empty(B, Hkv * G, D, dtype=torch.float16, device=DEV)
    av.rope_append(q.to(DEV), kn.to(DEV), vn.to(DEV), dk, dv, dT, advance=True, q_rot_out=qr)
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn)
    for b, t in enumerate(lens):
        assert_rope(qr.cpu()[b], q[b], t, D, what=f"q_rot b={b}")
        assert_rope(dk.cpu()[b, :, t], kn[b], t, D, what=f"k row b={b}")
        assert torch.equal(dv.cpu()[b, :, t], want["v_cache"][b, :, t])
    assert dT.cpu().tolist() == [t + 1 for t in lens]


def test_decode_graph_replays_across_lengths(av):
    """One CUDA graph serves every length: capture once, replay as T grows, no allocation."""
    B, Hkv, G, D, cap = 3, 2, 8, 128, 300
    lens = [40, 120, 7]
    _, _, _, kc, vc, T, _ = make_case(B, Hkv, G, D, lens, cap, seed=800)
    dk, dv, dT = kc.to(DEV), vc.to(DEV), T.to(DEV)
    sq = torch.empty(B, Hkv * G, D, dtype=torch.float16, device=DEV)
    skn = torch.empty(B, Hkv, D, dtype=torch.float16, device=DEV)
    svn = torch.empty_like(skn)
    out = torch.empty(B, Hkv * G, D, dtype=torch.float16, device=DEV)
    ws = av.make_workspace(B, Hkv * G, Hkv, D)
    # warm-up outside capture on a scratch copy, then restore
    av.decode(sq, dk.clone(), dv.clone(), out, k_new=skn, v_new=svn, seq_lens=dT.clone(), advance=True, workspace=ws)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            av.decode(sq, dk, dv, out, k_new=skn, v_new=svn, seq_lens=dT, advance=True, workspace=ws)
    torch.cuda.synchronize()
    ref_k, ref_v, ref_T = kc.clone(), vc.clone(), T.clone()
    mem0 = torch.cuda.memory_allocated()
    for step in range(4):
        q = randn_half((B, Hkv * G, D), 900 + step)
        kn = randn_half((B, Hkv, D), 950 + step)
        vn = randn_half((B, Hkv, D), 980 + step)
        sq.copy_(q)
        skn.copy_(kn)
        svn.copy_(vn)
        g.replay()
        torch.cuda.synchronize()
        want = O.decode_step(q, ref_k, ref_v, ref_T, k_new=kn, v_new=vn)
        assert_close(out.cpu(), want["ctx"], f"replay {step}")
        ref_k, ref_v, ref_T = want["k_cache"], want["v_cache"], want["seq_lens"]
        assert dT.cpu().tolist() == ref_T.tolist()
    assert torch.cuda.memory_allocated() == mem0
    assert av.read_error(ws) == 0


def test_nan_past_end_does_not_leak(av):
    # every row past T is NaN (make_case); the output must be finite everywhere
    lens = [3, 17, 200]
    q, kn, vn, kc, vc, T, cu = make_case(3, 2, 8, 128, lens, 256, seed=1000)
    got = run_decode(av, q, kn, vn, kc, vc, T, cu)
    assert torch.isfinite(got["out"].float()).all()


@pytest.mark.parametrize("lens_kind", ["uniform", "ragged", "packed"])
def test_prefetch_kv_layer_chain(av, lens_kind):
    """A chain of decode steps over four layers' arenas, as one token of a model runs them
    (only the last advances seq_lens), captured in one graph. With prefetch_kv each launch
    reads the lengths and its first cached K/V tiles before waiting for the previous
    layer's launch. Outputs, arenas and lengths must be bit-identical to the same chain
    without it, and each layer's output within tolerance of the oracle."""
    L, B, Hkv, G, D = 4, 8, 2, 8, 128
    lens = [1500] * B if lens_kind == "uniform" else [5, 64, 700, 1500, 129, 3000, 1, 2048]
    cap = max(lens) + 4
    packed = lens_kind == "packed"
    cases = [make_case(B, Hkv, G, D, lens, None if packed else cap, seed=1100 + 10 * l, packed=packed)
             for l in range(L)]
    lens0 = torch.tensor(lens, dtype=torch.int32, device=DEV)
    cu = cases[0][6].to(DEV) if packed else None
    results = {}
    for prefetch in (False, True):
        dq = [c[0].to(DEV) for c in cases]
        dkn = [c[1].to(DEV) for c in cases]
        dvn = [c[2].to(DEV) for c in cases]
        dk = [c[3].to(DEV) for c in cases]
        dv = [c[4].to(DEV) for c in cases]
        dT = lens0.clone()
        out = torch.full((L, B, Hkv * G, D), float("nan"), dtype=torch.float16, device=DEV)
        ws = av.make_workspace(B, Hkv * G, Hkv, D)

        def chain():
            dT.copy_(lens0)
            for l in range(L):
                av.decode(dq[l], dk[l], dv[l], out[l], k_new=dkn[l], v_new=dvn[l], seq_lens=dT, cu_seqlens=cu,
                          advance=(l == L - 1), workspace=ws, split=True, prefetch_kv=prefetch)

        chain()  # eager run (kernel attributes), then the same chain from a graph, twice
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                chain()
        torch.cuda.synchronize()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        assert av.read_error(ws) == 0
        results[prefetch] = (out.cpu(), [k.cpu() for k in dk], [v.cpu() for v in dv], dT.cpu())
    plain, pre = results[False], results[True]
    assert torch.equal(plain[0], pre[0])
    # bit patterns: the rows past each sequence hold NaN
    assert all(torch.equal(a.view(torch.int16), b.view(torch.int16)) for a, b in zip(plain[1] + plain[2],
                                                                                      pre[1] + pre[2]))
    assert pre[3].tolist() == [t + 1 for t in lens]
    for l, (q, kn, vn, kc, vc, T, cu_l) in enumerate(cases):
        want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn, cu_seqlens=cu_l)
        assert_close(pre[0][l], want["ctx"], f"layer {l} prefetch_kv")
