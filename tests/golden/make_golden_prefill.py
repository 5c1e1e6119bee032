"""Golden vectors for the prefill path from HF transformers' own Llama functions.

The reference's prefill (kv_init, case4_graph_generator_server_ipc.py:1241-1262)
runs the HF LlamaForCausalLM forward over the prompt: LlamaRotaryEmbedding +
apply_rotary_pos_emb (rotate-half RoPE at positions past_len + i) and the causal
eager attention (eager_attention_forward with an additive causal mask, softmax in
fp32), then copies each layer's rotated keys and values into the arena. This
script evaluates exactly those transformers functions, in fp32 on the CPU, on
seeded fp16-representable inputs, and stores inputs and outputs in
tests/golden/prefill_hf.pt. transformers is the reference's unpinned dependency;
the version used is recorded in the file.

Cases: a fresh prompt (past_len 0) with GQA, and a second chunk (past_len > 0)
whose cached keys are HF's own rotation of the earlier positions.

Run from the repository root: python tests/golden/make_golden_prefill.py
"""
import os

import torch
import transformers
from transformers import LlamaConfig
from transformers.models.llama import modeling_llama as M

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "prefill_hf.pt")


class _Stub(torch.nn.Module):
    def __init__(self, groups):
        super().__init__()
        self.num_key_value_groups = groups


def hf_case(seed, Hq, Hkv, D, past, n, theta=10000.0):
    g = torch.Generator().manual_seed(seed)
    total = past + n
    q = torch.randn(n, Hq, D, generator=g).half()
    k = torch.randn(total, Hkv, D, generator=g).half()  # un-rotated keys of positions 0 .. total-1
    v = torch.randn(total, Hkv, D, generator=g).half()
    cfg = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=D,
                      max_position_embeddings=4096, rope_theta=theta)
    rope = M.LlamaRotaryEmbedding(cfg)
    x = torch.zeros(1, total, Hq * D)
    pos_all = torch.arange(total).view(1, -1)
    cos, sin = rope(x, pos_all)  # [1, total, D] fp32
    qh = q.float().permute(1, 0, 2).unsqueeze(0)  # [1, Hq, n, D]
    kh = k.float().permute(1, 0, 2).unsqueeze(0)  # [1, Hkv, total, D]
    q_rot, _ = M.apply_rotary_pos_emb(qh, qh, cos[:, past:], sin[:, past:])
    _, k_rot = M.apply_rotary_pos_emb(kh, kh, cos, sin)
    vh = v.float().permute(1, 0, 2).unsqueeze(0)
    mask = torch.full((n, total), float("-inf"))
    rows = torch.arange(n).view(-1, 1) + past
    mask = mask.masked_fill(torch.arange(total).view(1, -1) <= rows, 0.0).view(1, 1, n, total)
    out, _ = M.eager_attention_forward(_Stub(Hq // Hkv), q_rot, k_rot, vh, mask, scaling=D ** -0.5)
    return dict(q=q, k=k, v=v, past=past, theta=theta, q_rot=q_rot[0].permute(1, 0, 2).contiguous(),
                k_rot=k_rot[0].permute(1, 0, 2).contiguous(), out=out[0].contiguous())


def main():
    cases = [hf_case(11, 2, 1, 128, 0, 160), hf_case(12, 2, 1, 128, 137, 90)]
    torch.save(dict(transformers=transformers.__version__, cases=cases), OUT)
    print("wrote", OUT, "transformers", transformers.__version__)


if __name__ == "__main__":
    main()
