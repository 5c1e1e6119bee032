"""CPU checks of the prefill oracle and of the prefill C ABI (no GPU).

The oracle's prefill_step is pinned two ways:
  - against HF transformers' own LlamaRotaryEmbedding / apply_rotary_pos_emb /
    eager_attention_forward (the code the reference's kv_init runs), evaluated in
    fp32 by tests/golden/make_golden_prefill.py: rotated q/k within fp16 rounding
    of HF's fp32 values, attention output within the decode tolerance;
  - against the decode oracle (itself pinned to the reference's RoPE and kernel
    outputs): n new tokens prefilled at once equal n consecutive decode steps.
"""
import ctypes
import os

import torch

from helpers import randn_half
from oracle import decode_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _hf_cases():
    return torch.load(os.path.join(ROOT, "tests", "golden", "prefill_hf.pt"))["cases"]


def test_prefill_oracle_matches_hf_llama_functions():
    for c in _hf_cases():
        n, Hq, D = c["q"].shape
        total, Hkv, _ = c["k"].shape
        past = c["past"]
        kc = torch.zeros(1, Hkv, total + 8, D, dtype=torch.float16)
        vc = torch.zeros_like(kc)
        kc[0, :, :past] = c["k_rot"][:past].half().permute(1, 0, 2)
        vc[0, :, :past] = c["v"][:past].permute(1, 0, 2)
        r = O.prefill_step(c["q"], c["k"][past:], c["v"][past:], kc, vc, torch.tensor([0, n]), torch.tensor([past]))
        # fp16 rounding of values below 8 in magnitude: at most 2^-8 apart
        assert (r["q_rot"].float() - c["q_rot"]).abs().max() <= 2.0 ** -8
        got_k = r["k_cache"][0, :, past:total].permute(1, 0, 2).float()
        assert (got_k - c["k_rot"][past:]).abs().max() <= 2.0 ** -8
        assert torch.equal(r["v_cache"][0, :, past:total], c["v"][past:].permute(1, 0, 2))
        max_abs, rel = O.compare(r["out"], c["out"])
        assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL
        assert int(r["seq_lens"][0]) == total


def test_prefill_equals_chain_of_decode_steps():
    B, Hq, Hkv, D, cap = 3, 4, 2, 128, 48
    lens, T0 = [5, 9, 0], [3, 0, 7]
    cu = torch.tensor([0, 5, 14, 14], dtype=torch.int32)
    q, kn, vn = randn_half((14, Hq, D), 1), randn_half((14, Hkv, D), 2), randn_half((14, Hkv, D), 3)
    kc, vc = randn_half((B, Hkv, cap, D), 4), randn_half((B, Hkv, cap, D), 5)
    T = torch.tensor(T0, dtype=torch.int32)
    r = O.prefill_step(q, kn, vn, kc, vc, cu, T)
    k2, v2, T2 = kc.clone(), vc.clone(), T.clone()
    for b in range(B):
        for i in range(lens[b]):
            row = int(cu[b]) + i
            qq, kk, vv = (torch.zeros(B, h, D, dtype=torch.float16) for h in (Hq, Hkv, Hkv))
            qq[b], kk[b], vv[b] = q[row], kn[row], vn[row]
            d = O.decode_step(qq, k2, v2, T2, k_new=kk, v_new=vv)
            k2[b], v2[b], T2[b] = d["k_cache"][b], d["v_cache"][b], d["seq_lens"][b]
            assert (d["ctx"][b] - r["out"][row]).abs().max() <= 1e-5
    assert torch.equal(k2, r["k_cache"]) and torch.equal(v2, r["v_cache"])
    assert T2.tolist() == r["seq_lens"].tolist() == [8, 9, 7]


def test_prefill_oracle_packed_layout_and_overflow():
    Hq, Hkv, D = 2, 1, 128
    cu = torch.tensor([0, 4, 10], dtype=torch.int32)
    cu_kv = torch.tensor([0, 8, 12], dtype=torch.int32)  # capacities 8 and 4
    q, kn, vn = randn_half((10, Hq, D), 7), randn_half((10, Hkv, D), 8), randn_half((10, Hkv, D), 9)
    kc, vc = randn_half((Hkv, 12, D), 10), randn_half((Hkv, 12, D), 11)
    r = O.prefill_step(q, kn, vn, kc, vc, cu, torch.tensor([2, 0]), cu_seqlens_kv=cu_kv)
    assert r["ok"].tolist() == [True, False]  # 0 + 6 > 4
    assert r["seq_lens"].tolist() == [6, 0]
    assert torch.equal(r["k_cache"][:, 8:], kc[:, 8:]) and r["out"][4:].abs().max() == 0


def test_prefill_workspace_bytes_abi():
    lib = ctypes.CDLL(os.path.join(ROOT, "fully_custom_cuda_inference_lamma2_b200", "libfcci_decode.so"))
    f = lib.fcci_prefill_workspace_bytes
    f.restype = ctypes.c_size_t
    f.argtypes = [ctypes.c_int32] * 8
    n = f(16, 32, 32, 128, 34816, 4096, 4096, 128)
    # rotated queries + table + work list + header
    assert n >= 34816 * 32 * 128 * 2 + 4096 * 64 * 8 + 16 * 16 * 32 * 16
    assert f(16, 32, 32, 64, 100, 100, 100, 64) == 0  # head_dim 64 is not compiled
    assert f(0, 32, 32, 128, 100, 100, 100, 128) == 0
    lib.fcci_prefill_attention.restype = ctypes.c_int
    lib.fcci_prefill_attention.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    assert lib.fcci_prefill_attention(None, None) == 1
