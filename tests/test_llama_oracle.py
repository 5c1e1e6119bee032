"""CPU pin of the model oracle (oracle/llama_oracle.py) against HF transformers'
own LlamaForCausalLM, the model the reference decodes: the same small random
weights loaded into both, logits at every position of a sequence compared in fp32."""
import torch

from oracle import llama_oracle as LO


class _W:
    pass


def test_llama_oracle_matches_hf_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    H, I, V, L, heads, kv, D = 256, 512, 300, 2, 4, 2, 64
    cfg = LlamaConfig(hidden_size=H, intermediate_size=I, num_hidden_layers=L, num_attention_heads=heads,
                      num_key_value_heads=kv, head_dim=D, vocab_size=V, rms_norm_eps=1e-5,
                      tie_word_embeddings=True, rope_theta=10000.0, max_position_embeddings=128)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).float().eval()
    with torch.no_grad():  # non-trivial RMSNorm weights too
        for layer in model.model.layers:
            layer.input_layernorm.weight.uniform_(0.5, 1.5)
            layer.post_attention_layernorm.weight.uniform_(0.5, 1.5)
        model.model.norm.weight.uniform_(0.5, 1.5)
    w = _W()
    w.shape = type("S", (), dict(layers=L, hidden=H, heads=heads, kv_heads=kv, head_dim=D, intermediate=I,
                                 vocab=V, eps=1e-5, rope_theta=10000.0))
    ly = model.model.layers
    w.embed = model.model.embed_tokens.weight.detach()
    w.w_qkv = torch.stack([torch.cat([l.self_attn.q_proj.weight, l.self_attn.k_proj.weight,
                                      l.self_attn.v_proj.weight]) for l in ly]).detach()
    w.w_o = torch.stack([l.self_attn.o_proj.weight for l in ly]).detach()
    w.w_gu = torch.stack([torch.cat([l.mlp.gate_proj.weight, l.mlp.up_proj.weight]) for l in ly]).detach()
    w.w_down = torch.stack([l.mlp.down_proj.weight for l in ly]).detach()
    w.rms_in = torch.stack([l.input_layernorm.weight for l in ly]).detach()
    w.rms_post = torch.stack([l.post_attention_layernorm.weight for l in ly]).detach()
    w.rms_final = model.model.norm.weight.detach()
    tokens = torch.randint(0, V, (20,), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        hf = model(tokens.view(1, -1)).logits[0]
    ours = LO.logits_for(w, tokens)
    assert torch.allclose(ours, hf, rtol=1e-4, atol=1e-4), float((ours - hf).abs().max())
