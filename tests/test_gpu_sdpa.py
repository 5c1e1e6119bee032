"""GPU checks of the single-query SDPA route (the reference's flash_attn.py names:
sdp_single_q and enable_flash_sdp_monkeypatch) on the decode-attention kernel.

sdp_single_q matches torch SDPA computed in fp32 within the decode tolerance
(max-abs 2e-3, rel-L2 1e-3) for MHA, GQA and strided caches; the patched
F.scaled_dot_product_attention runs the decode kernel for single-query unmasked
calls (the library's launch counter moves), hands every other call to torch, and an
HF Llama decoding greedily with the patch gives the logits it gives without it.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from oracle import decode_oracle as O

pytestmark = pytest.mark.gpu


def _ref(q, k, v, scale):
    G = q.size(1) // k.size(1)
    kk = k.float().repeat_interleave(G, dim=1)
    vv = v.float().repeat_interleave(G, dim=1)
    return F.scaled_dot_product_attention(q.float(), kk, vv, scale=scale)


@pytest.mark.parametrize("B,Hq,Hkv,T,D", [(1, 32, 32, 1, 128), (2, 32, 32, 517, 128), (3, 64, 8, 2049, 128),
                                          (4, 16, 4, 300, 64), (1, 8, 8, 1000, 256)])
def test_sdp_single_q_matches_fp32(B, Hq, Hkv, T, D):
    from fully_custom_cuda_inference_lamma2_b200 import flash_attn as FA

    g = torch.Generator(device="cuda").manual_seed(T + D)
    q = torch.randn(B, Hq, 1, D, device="cuda", generator=g).half()
    k = torch.randn(B, Hkv, T, D, device="cuda", generator=g).half()
    v = torch.randn(B, Hkv, T, D, device="cuda", generator=g).half()
    scale = 1.0 / math.sqrt(D)
    out = FA.sdp_single_q(q, k, v)
    torch.cuda.synchronize()
    max_abs, rel = O.compare(out.float().cpu(), _ref(q, k, v, scale).cpu())
    assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL, (max_abs, rel)


def test_sdp_single_q_strided_cache_and_scale():
    from fully_custom_cuda_inference_lamma2_b200 import flash_attn as FA

    g = torch.Generator(device="cuda").manual_seed(9)
    cache_k = torch.randn(2, 8, 1024, 128, device="cuda", generator=g).half()
    cache_v = torch.randn(2, 8, 1024, 128, device="cuda", generator=g).half()
    k, v = cache_k[:, :, :333], cache_v[:, :, :333]  # a prefix view of a larger cache
    q = torch.randn(2, 8, 1, 128, device="cuda", generator=g).half()
    out = FA.sdp_single_q(q, k, v, scale=0.05)
    torch.cuda.synchronize()
    max_abs, rel = O.compare(out.float().cpu(), _ref(q, k, v, 0.05).cpu())
    assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL, (max_abs, rel)


def test_monkeypatch_routes_only_single_query_calls():
    import fully_custom_cuda_inference_lamma2_b200 as pkg
    from fully_custom_cuda_inference_lamma2_b200 import flash_attn as FA

    av = pkg.attn_varlen
    g = torch.Generator(device="cuda").manual_seed(10)
    q1 = torch.randn(1, 8, 1, 128, device="cuda", generator=g).half()
    q4 = torch.randn(1, 8, 4, 128, device="cuda", generator=g).half()
    k = torch.randn(1, 8, 64, 128, device="cuda", generator=g).half()
    v = torch.randn(1, 8, 64, 128, device="cuda", generator=g).half()
    FA.enable_flash_sdp_monkeypatch()
    try:
        n0 = av.launch_count()
        a = F.scaled_dot_product_attention(q1, k, v)
        torch.cuda.synchronize()
        assert av.launch_count() > n0, "single-query call did not reach the decode kernel"
        n1 = av.launch_count()
        b = F.scaled_dot_product_attention(q4, k, v, is_causal=True)
        c = F.scaled_dot_product_attention(q1.float(), k.float(), v.float())
        torch.cuda.synchronize()
        assert av.launch_count() == n1, "multi-query / fp32 calls must go to torch"
    finally:
        FA.disable_flash_sdp_monkeypatch()
    assert F.scaled_dot_product_attention is not None
    max_abs, rel = O.compare(a.float().cpu(), _ref(q1, k, v, 1 / math.sqrt(128)).cpu())
    assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL
    assert torch.allclose(b, F.scaled_dot_product_attention(q4, k, v, is_causal=True))


def test_hf_llama_decode_with_the_patch():
    from transformers import LlamaConfig, LlamaForCausalLM

    from fully_custom_cuda_inference_lamma2_b200 import flash_attn as FA

    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=1000, max_position_embeddings=256)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = LlamaForCausalLM(cfg).half().eval()
    prompt = torch.randint(0, 1000, (1, 12), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        ref = model(prompt, use_cache=True)
        ref_step = model(prompt[:, -1:] * 0 + 5, past_key_values=ref.past_key_values, use_cache=True).logits
        FA.enable_flash_sdp_monkeypatch()
        try:
            out = model(prompt, use_cache=True)
            out_step = model(prompt[:, -1:] * 0 + 5, past_key_values=out.past_key_values, use_cache=True).logits
        finally:
            FA.disable_flash_sdp_monkeypatch()
    torch.cuda.synchronize()
    assert torch.equal(out.logits, ref.logits)  # the prompt pass is multi-query: torch in both runs
    max_abs, rel = O.compare(out_step.float().cpu(), ref_step.float().cpu())
    assert rel <= 2e-3, (max_abs, rel)
