"""CPU checks of the oracle: golden vectors from the reference's own code and
known-answer properties of RoPE, softmax attention, GQA and the placeholder step."""
import math
import os

import pytest
import torch

from helpers import randn_half
from oracle import decode_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.fail(f"golden fixture {name} missing")
    return torch.load(path)


def test_rope_matches_reference_driver_bit_exact():
    d = golden("rope_reference.pt")
    cases = [c for c in d["cases"] if c["kind"] == "driver"]
    assert len(cases) >= 40
    for c in cases:
        got = O.rope_rotate_half(c["x"], c["pos"], c["rotary_dim"], c["theta"])
        assert torch.equal(got, c["out"]), (c["pos"], c["rotary_dim"], c["theta"])


def test_server_rope_fixture_and_its_aliasing():
    d = golden("rope_reference.pt")
    for c in (c for c in d["cases"] if c["kind"] == "server"):
        got = O.rope_server_inplace(c["x"], c["pos"], c["theta"])
        assert torch.allclose(got, c["out"], atol=2e-5, rtol=1e-5), c["pos"]
        if c["pos"] > 0:  # the server result is not a rotation: norms are not preserved
            rot = O.rope_rotate_half(c["x"].float(), c["pos"], 128, c["theta"])
            assert not torch.allclose(rot, c["out"], atol=1e-3)


def test_rope_position_zero_is_identity():
    x = randn_half((16, 128), 1)
    assert torch.equal(O.rope_rotate_half(x, 0, 128), x)


def test_rope_preserves_pair_norms():
    x = torch.randn(8, 128, dtype=torch.float32, generator=torch.Generator().manual_seed(2))
    for pos in (1, 100, 4096, 32768):
        y = O.rope_rotate_half(x, pos, 128)
        n0 = x[:, :64] ** 2 + x[:, 64:] ** 2
        n1 = y[:, :64] ** 2 + y[:, 64:] ** 2
        assert torch.allclose(n0, n1, rtol=1e-4, atol=1e-4)


def test_rope_partial_leaves_tail():
    x = randn_half((4, 128), 3)
    y = O.rope_rotate_half(x, 77, 64)
    assert torch.equal(y[:, 64:], x[:, 64:])
    assert not torch.equal(y[:, :64], x[:, :64])


def test_attention_single_key_returns_value():
    q, k, v = randn_half((4, 128), 4), randn_half((4, 1, 128), 5), randn_half((4, 1, 128), 6)
    assert torch.allclose(O.attention(q, k, v, 0.1), v[:, 0].float())


def test_attention_constant_values_normalise():
    q, k = randn_half((8, 64), 7), randn_half((8, 300, 64), 8)
    v = torch.ones(8, 300, 64, dtype=torch.float16)
    assert torch.allclose(O.attention(q, k, v, 0.125), torch.ones(8, 64), atol=1e-6)


def test_attention_matches_reference_einsum_form():
    # case4_graph_generator_server_ipc.py:1000-1006 on MHA
    q, k, v = randn_half((32, 128), 9), randn_half((32, 513, 128), 10), randn_half((32, 513, 128), 11)
    s = torch.einsum("hd,htd->ht", q.float(), k.float()) * (1 / math.sqrt(128))
    want = torch.einsum("ht,htd->hd", torch.softmax(s, -1), v.float())
    assert torch.allclose(O.attention(q, k, v, 1 / math.sqrt(128)), want, atol=1e-5)


def test_gqa_equals_repeat_interleave():
    Hkv, G = 4, 8
    q, k, v = randn_half((Hkv * G, 64), 12), randn_half((Hkv, 100, 64), 13), randn_half((Hkv, 100, 64), 14)
    ks, vs = k.repeat_interleave(G, 0), v.repeat_interleave(G, 0)
    assert torch.allclose(O.attention(q, k, v, 0.125), O.attention(q, ks, vs, 0.125), atol=1e-6)


def test_decode_step_appends_and_advances():
    B, Hkv, G, D, cap = 2, 2, 2, 64, 10
    q, kn, vn = randn_half((B, Hkv * G, D), 15), randn_half((B, Hkv, D), 16), randn_half((B, Hkv, D), 17)
    kc, vc = randn_half((B, Hkv, cap, D), 18), randn_half((B, Hkv, cap, D), 19)
    r = O.decode_step(q, kc, vc, torch.tensor([3, 9], dtype=torch.int32), k_new=kn, v_new=vn)
    assert r["seq_lens"].tolist() == [4, 10]
    assert torch.equal(r["v_cache"][1, :, 9], vn[1])
    assert torch.equal(r["k_cache"][0, :, 3], O.rope_rotate_half(kn[0], 3, D))
    assert torch.equal(kc[0, :, 3], randn_half((B, Hkv, cap, D), 18)[0, :, 3])  # inputs untouched


def test_decode_step_capacity_overflow():
    B, Hkv, D, cap = 1, 1, 64, 4
    q, kn, vn = randn_half((B, Hkv, D), 20), randn_half((B, Hkv, D), 21), randn_half((B, Hkv, D), 22)
    kc = randn_half((B, Hkv, cap, D), 23)
    r = O.decode_step(q, kc, kc, torch.tensor([4], dtype=torch.int32), k_new=kn, v_new=vn)
    assert not bool(r["ok"][0]) and torch.count_nonzero(r["ctx"]) == 0 and r["seq_lens"].tolist() == [4]


def test_packed_layout_equals_batched():
    lens = [5, 17, 1]
    B, Hkv, G, D = 3, 2, 4, 64
    q, kn, vn = randn_half((B, Hkv * G, D), 24), randn_half((B, Hkv, D), 25), randn_half((B, Hkv, D), 26)
    cap = 20
    kb, vb = randn_half((B, Hkv, cap, D), 27), randn_half((B, Hkv, cap, D), 28)
    cu = torch.tensor([0, cap, 2 * cap, 3 * cap], dtype=torch.int32)
    kp = kb.permute(1, 0, 2, 3).reshape(Hkv, B * cap, D).contiguous()
    vp = vb.permute(1, 0, 2, 3).reshape(Hkv, B * cap, D).contiguous()
    T = torch.tensor(lens, dtype=torch.int32)
    a = O.decode_step(q, kb, vb, T, k_new=kn, v_new=vn)
    b = O.decode_step(q, kp, vp, T, k_new=kn, v_new=vn, cu_seqlens=cu)
    assert torch.equal(a["ctx"], b["ctx"])


@pytest.mark.parametrize("T,ctrl", [(3, 12345), (0, -3), (9, 7)])
def test_placeholder_step(T, ctrl):
    ak = randn_half((2, 1, 3, 10, 8), 29)
    nk, nv, lg, nT = O.placeholder_step(ctrl, ak, ak, T, 100)
    assert nT == T + 1
    assert torch.count_nonzero(nk[:, 0, :, T]) == 0
    other = [t for t in range(10) if t != T]
    assert torch.equal(nk[:, :, :, other], ak[:, :, :, other])
    hot = int(math.fmod(ctrl, 100))
    assert float(lg.sum()) == (1.0 if hot >= 0 else 0.0)
    if hot >= 0:
        assert float(lg[0, hot]) == 1.0


def test_compare_metric():
    a = torch.tensor([1.0, 2.0, 3.0], dtype=torch.float64)
    ma, rel = O.compare(a + 1e-3, a)
    assert abs(ma - 1e-3) < 1e-9 and rel < 1e-3


def test_oracle_matches_reference_cuda_kernel_golden():
    """Outputs of the reference's attn_varlen kernel, built from its sources and run on a
    B200 (tests/golden/make_golden_gpu.py), against the oracle on the same seeded inputs."""
    from helpers import sha256_of

    d = golden("ref_kernels.pt")
    assert len(d["attn_varlen"]) >= 9
    for c in d["attn_varlen"]:
        H, T, D, seed = c["H"], c["T"], c["D"], c["seed"]
        q = randn_half((H, D), 1000 * seed + 1)
        k = randn_half((H, T, D), 1000 * seed + 2)
        v = randn_half((H, T, D), 1000 * seed + 3)
        assert (sha256_of(q), sha256_of(k), sha256_of(v)) == (c["sha_q"], c["sha_k"], c["sha_v"])
        ma, rel = O.compare(O.attn_varlen_forward(q, k, v, T, c["scale"]), c["ctx"].float())
        assert ma <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL, (H, T, D, ma, rel)


def test_oracle_placeholder_matches_reference_kernel_golden():
    from helpers import sha256_of

    d = golden("ref_kernels.pt")
    for c in d["capture_decode"]:
        L, H, ml, D, seed = c["L"], c["H"], c["max_len"], c["D"], c["seed"]
        ak = randn_half((L, 1, H, ml, D), 1000 * seed + 1)
        av = randn_half((L, 1, H, ml, D), 1000 * seed + 2)
        nk, nv, lg, nT = O.placeholder_step(c["ctrl"], ak, av, c["T"], c["vocab"])
        assert sha256_of(nk) == c["sha_k_out"] and sha256_of(nv) == c["sha_v_out"]
        assert torch.nonzero(lg[0]).flatten().tolist() == c["logits_nonzero"].tolist()
        assert float(lg.sum()) == c["logits_sum"] and nT == c["seq_len_out"]
