"""GPU parity of the causal varlen prefill (tcgen05 attention) against the oracle
and against HF transformers' own Llama functions.

Tolerances (the decode path's): attention output within max-abs 2e-3 and
relative-L2 1e-3 of the fp32 oracle. Rotated keys written into the arena are
bit-exact with the reference driver's fp32 RoPE formula evaluated by torch on the
GPU; values are copied bit-exactly; arena rows outside [T_b, T_b + n_b) are left
untouched. seq_lens advances by n_b.
"""
import pytest
import torch

from helpers import randn_half
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


def make_batch(lens, T, Hq, Hkv, cap, seed, packed=False, poison=True, qscale=1.0):
    """Seeded new tokens for sequences of n_b = lens[b] tokens after T[b] cached ones."""
    D = 128
    B = len(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)
    total = int(cu[-1])
    q = (randn_half((total, Hq, D), seed).float() * qscale).half()
    kn, vn = randn_half((total, Hkv, D), seed + 1), randn_half((total, Hkv, D), seed + 2)
    if packed:
        caps = [cap] * B
        cu_kv = torch.tensor([0] + [cap * (b + 1) for b in range(B)], dtype=torch.int32)
        kc = randn_half((Hkv, cap * B, D), seed + 3)
        vc = randn_half((Hkv, cap * B, D), seed + 4)
    else:
        cu_kv = None
        kc = randn_half((B, Hkv, cap, D), seed + 3)
        vc = randn_half((B, Hkv, cap, D), seed + 4)
    if poison:
        # rows past each sequence's new length hold NaN: the kernel must not let them leak
        for b in range(B):
            end = T[b] + lens[b]
            if packed:
                vc[:, cap * b + end: cap * (b + 1)] = float("nan")
                kc[:, cap * b + end: cap * (b + 1)] = float("nan")
            else:
                vc[b, :, end:] = float("nan")
                kc[b, :, end:] = float("nan")
    return dict(q=q, kn=kn, vn=vn, kc=kc, vc=vc, cu=cu, cu_kv=cu_kv, T=torch.tensor(T, dtype=torch.int32),
                max_q=max(lens) if lens else 0)


def run_prefill(av, c, advance=True, workspace=None):
    dq, dkn, dvn = c["q"].to(DEV), c["kn"].to(DEV), c["vn"].to(DEV)
    dk, dv = c["kc"].to(DEV), c["vc"].to(DEV)
    dcu, dT = c["cu"].to(DEV), c["T"].to(DEV)
    dcukv = c["cu_kv"].to(DEV) if c["cu_kv"] is not None else None
    out = torch.full_like(dq, float("nan"))
    av.prefill_varlen(dq, dkn, dvn, dk, dv, out, dcu, c["max_q"], seq_lens=dT, cu_seqlens_kv=dcukv,
                      advance=advance, workspace=workspace)
    torch.cuda.synchronize()
    return out.cpu(), dk.cpu(), dv.cpu(), dT.cpu()


def check_against_oracle(av, c, what):
    out, k, v, T = run_prefill(av, c)
    want = O.prefill_step(c["q"], c["kn"], c["vn"], c["kc"], c["vc"], c["cu"], c["T"], cu_seqlens_kv=c["cu_kv"])
    assert want["ok"].all()
    assert_close(out, want["out"], what)
    # rotated keys: bit-exact with the fp32 formula evaluated on the GPU
    B = c["cu"].numel() - 1
    for b in range(B):
        r0, r1 = int(c["cu"][b]), int(c["cu"][b + 1])
        t0 = int(c["T"][b])
        if r1 == r0:
            continue
        pos = torch.arange(t0, t0 + r1 - r0)
        k_dev = O.rope_positions(c["kn"][r0:r1].to(DEV), pos, 128).cpu().permute(1, 0, 2)
        if c["cu_kv"] is None:
            got_k, got_v = k[b, :, t0:t0 + r1 - r0], v[b, :, t0:t0 + r1 - r0]
        else:
            base = int(c["cu_kv"][b])
            got_k, got_v = k[:, base + t0: base + t0 + r1 - r0], v[:, base + t0: base + t0 + r1 - r0]
        assert torch.equal(got_k, k_dev), f"{what}: appended keys of sequence {b} differ"
        assert torch.equal(got_v, c["vn"][r0:r1].permute(1, 0, 2)), f"{what}: appended values of sequence {b}"
    # rows outside [T_b, T_b + n_b) keep their bit patterns (NaN poison included)
    new_rows = torch.zeros(k.shape[:-1], dtype=torch.bool)
    for b in range(B):
        t0, n = int(c["T"][b]), int(c["cu"][b + 1] - c["cu"][b])
        if c["cu_kv"] is None:
            new_rows[b, :, t0:t0 + n] = True
        else:
            base = int(c["cu_kv"][b])
            new_rows[:, base + t0: base + t0 + n] = True
    keep = ~new_rows
    assert torch.equal(k.view(torch.int16)[keep], c["kc"].view(torch.int16)[keep]), f"{what}: other key rows changed"
    assert torch.equal(v.view(torch.int16)[keep], c["vc"].view(torch.int16)[keep]), f"{what}: other value rows changed"
    assert T.tolist() == want["seq_lens"].tolist()


def test_prefill_hf_golden(av):
    """Fresh prompt and a second chunk from HF transformers' LlamaRotaryEmbedding,
    apply_rotary_pos_emb and eager_attention_forward (tests/golden/prefill_hf.pt)."""
    import os

    d = torch.load(os.path.join(os.path.dirname(__file__), "golden", "prefill_hf.pt"))
    for i, c in enumerate(d["cases"]):
        n, Hq, D = c["q"].shape
        total, Hkv, _ = c["k"].shape
        past = c["past"]
        cap = total + 40
        kc = torch.zeros(1, Hkv, cap, D, dtype=torch.float16)
        vc = torch.zeros_like(kc)
        kc[0, :, :past] = c["k_rot"][:past].half().permute(1, 0, 2)
        vc[0, :, :past] = c["v"][:past].permute(1, 0, 2)
        dk, dv = kc.to(DEV), vc.to(DEV)
        out = torch.empty(n, Hq, D, dtype=torch.float16, device=DEV)
        T = torch.tensor([past], dtype=torch.int32, device=DEV)
        av.prefill_varlen(c["q"].to(DEV), c["k"][past:].to(DEV), c["v"][past:].to(DEV), dk, dv, out,
                          torch.tensor([0, n], dtype=torch.int32, device=DEV), n, seq_lens=T, advance=True)
        torch.cuda.synchronize()
        assert_close(out, c["out"], f"HF case {i}")
        got_k = dk[0, :, past:total].permute(1, 0, 2).float().cpu()
        assert (got_k - c["k_rot"][past:]).abs().max().item() <= 4e-3, f"HF case {i}: rotated keys"
        assert int(T.item()) == total


@pytest.mark.parametrize("packed", [False, True])
def test_prefill_varlen_fresh(av, packed):
    lens = [1, 127, 128, 129, 300, 0, 256, 257]
    c = make_batch(lens, [0] * len(lens), Hq=4, Hkv=2, cap=320, seed=100, packed=packed)
    check_against_oracle(av, c, f"fresh packed={packed}")


def test_prefill_chunked_after_cache(av):
    """Later chunks: T_b > 0 cached tokens (not a multiple of the tile), GQA 4."""
    lens = [90, 1, 200, 33]
    T = [37, 500, 128, 0]
    c = make_batch(lens, T, Hq=8, Hkv=2, cap=704, seed=200)
    check_against_oracle(av, c, "chunked")


def test_prefill_long_rescale(av):
    """Two long sequences with sharp scores so the running maximum moves often."""
    c = make_batch([2048, 1500], [0, 0], Hq=2, Hkv=2, cap=2048, seed=300, qscale=3.0)
    check_against_oracle(av, c, "long")


def test_prefill_then_decode_matches_oracle_chain(av):
    lens = [200, 77]
    c = make_batch(lens, [0, 0], Hq=4, Hkv=4, cap=400, seed=400, poison=False)
    out, k, v, T = run_prefill(av, c)
    want = O.prefill_step(c["q"], c["kn"], c["vn"], c["kc"], c["vc"], c["cu"], c["T"])
    assert T.tolist() == lens
    B, Hq, D = 2, 4, 128
    q1, kn1, vn1 = randn_half((B, Hq, D), 401), randn_half((B, 4, D), 402), randn_half((B, 4, D), 403)
    dk, dv, dT = k.to(DEV), v.to(DEV), T.to(DEV)
    ctx = torch.empty(B, Hq, D, dtype=torch.float16, device=DEV)
    av.decode(q1.to(DEV), dk, dv, ctx, k_new=kn1.to(DEV), v_new=vn1.to(DEV), seq_lens=dT, advance=True)
    torch.cuda.synchronize()
    ref = O.decode_step(q1, want["k_cache"], want["v_cache"], want["seq_lens"], k_new=kn1, v_new=vn1)
    assert_close(ctx, ref["ctx"], "decode after prefill")
    assert dT.cpu().tolist() == [201, 78]


def test_prefill_reuses_workspace_and_flags_capacity(av):
    """One workspace across calls of different sizes; a sequence that does not fit
    its capacity sets the device error word and the others are still correct."""
    ws = av.make_prefill_workspace(3, 4, 2, 128, 600, 300, 320)
    c = make_batch([100, 300, 50], [0, 30, 0], Hq=4, Hkv=2, cap=320, seed=500)
    out, *_ = run_prefill(av, c, workspace=ws)
    assert av.prefill_read_error(ws) & 1, "capacity overflow of sequence 1 not flagged"
    want = O.prefill_step(c["q"], c["kn"], c["vn"], c["kc"], c["vc"], c["cu"], c["T"])
    assert want["ok"].tolist() == [True, False, True]
    keep = torch.cat([torch.arange(0, 100), torch.arange(400, 450)])
    assert_close(out[keep], want["out"][keep], "valid sequences next to an overflowing one")
    c2 = make_batch([64, 64, 64], [5, 5, 5], Hq=4, Hkv=2, cap=320, seed=501)
    out2, *_ = run_prefill(av, c2, workspace=ws)
    assert av.prefill_read_error(ws) == 0
    want2 = O.prefill_step(c2["q"], c2["kn"], c2["vn"], c2["kc"], c2["vc"], c2["cu"], c2["T"])
    assert_close(out2, want2["out"], "second call on the same workspace")
