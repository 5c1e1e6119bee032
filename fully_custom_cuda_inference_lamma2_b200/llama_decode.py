"""Greedy decode of a Llama-2-shaped model around the decode-attention path.

The reference decodes in CUDA graphs captured per exact sequence length
(case4_graph_generator_server_ipc.py:2341-2607; scripts/direct_custom_decode_500.py),
with the attention of each layer done in torch around `attn_varlen.forward`, and
its in-graph step `capture_decode_ext` (custom_kernels/capture_decode_step_kernel.cu:137-274)
runs only layer 0 of the MLP on x = 0. Here one token step is the whole model:

    x = embed[token]
    per layer l:  h = RMSNorm(x) ; qkv = W_qkv h                       (cuBLAS)
                  RoPE(q, k) at T, append (k, v) at T, attention over T+1 keys,
                  T += 1 after the last layer                          (decode_attn_kernel)
                  x += W_o ctx                                          (cuBLAS)
                  h = RMSNorm(x) ; g, u = W_gu h ; x += W_down (SiLU(g) * u)
    logits = embed . RMSNorm(x)   (tied embeddings) ; token = argmax(logits)

T lives on the device (`KVArena.seq_lens`), so ONE captured graph serves every
length; a step neither allocates nor synchronises the host. The prompt is filled
into the arena by the causal varlen prefill (`attn_varlen.prefill_varlen`), whose
rows are the same the decode step would have appended.

Projections (default) are this library's fused batch-1 GEMVs
(`capture_decode_step.gemv_fused`): RMSNorm in the QKV and gate/up prologues, SwiGLU
in the gate/up epilogue, the residual adds in the O and down epilogues, five
launches per layer. `projections="cublas"` runs them as torch/cuBLAS products with
the separate RMSNorm / SwiGLU kernels instead. All fp16, as the reference's model.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from . import attn_varlen, capture_decode_step
from .arena import KVArena, decode_attention


@dataclass(frozen=True)
class LlamaShape:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 32
    head_dim: int = 128
    intermediate: int = 11008
    vocab: int = 32000
    eps: float = 1e-5
    rope_theta: float = 10000.0

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    def weight_bytes(self) -> int:
        """fp16 bytes one token step reads: every projection once, plus the tied vocab matrix."""
        H, I = self.hidden, self.intermediate
        per_layer = (self.qkv_rows * H + H * self.heads * self.head_dim + 2 * I * H + H * I + 2 * H) * 2
        return self.layers * per_layer + (self.vocab * H + H) * 2


LLAMA2_7B = LlamaShape()


class LlamaWeights:
    """Random-init weights (N(0, 0.02), RMSNorm weights 1) generated on the device from a seed;
    no checkpoint is needed or read. Layer tensors are stacked on a leading layer axis."""

    def __init__(self, shape: LlamaShape = LLAMA2_7B, seed: int = 0, device=None, std: float = 0.02):
        self.shape = s = shape
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(seed)

        def rand(*dims):
            t = torch.empty(*dims, dtype=torch.float16, device=dev)
            flat = t.view(-1)
            step = 1 << 28
            for i in range(0, flat.numel(), step):
                flat[i:i + step].normal_(0.0, std, generator=g)
            return t

        H, I, L = s.hidden, s.intermediate, s.layers
        self.embed = rand(s.vocab, H)
        self.w_qkv = rand(L, s.qkv_rows, H)
        self.w_o = rand(L, H, s.heads * s.head_dim)
        self.w_gu = rand(L, 2 * I, H)
        self.w_down = rand(L, H, I)
        self.rms_in = torch.ones(L, H, dtype=torch.float16, device=dev)
        self.rms_post = torch.ones(L, H, dtype=torch.float16, device=dev)
        self.rms_final = torch.ones(H, dtype=torch.float16, device=dev)

    @classmethod
    def from_tensors(cls, shape: LlamaShape, *, embed, w_qkv, w_o, w_gu, w_down, rms_in, rms_post, rms_final):
        self = cls.__new__(cls)
        self.shape = shape
        self.embed, self.w_qkv, self.w_o, self.w_gu, self.w_down = embed, w_qkv, w_o, w_gu, w_down
        self.rms_in, self.rms_post, self.rms_final = rms_in, rms_post, rms_final
        return self


class GreedyDecoder:
    """Batch-1 greedy decoding with a persistent KV arena and one CUDA graph per token step."""

    def __init__(self, weights: LlamaWeights, capacity: int, max_new_tokens: int = 1024, projections: str = "fused"):
        if projections not in ("fused", "cublas"):
            raise ValueError("projections must be 'fused' or 'cublas'")
        self.projections = projections
        self.w = weights
        s = self.s = weights.shape
        dev = weights.embed.device
        self.device = dev
        self.arena = KVArena(s.layers, 1, s.kv_heads, s.head_dim, capacity=capacity, q_heads=s.heads, device=dev)
        H, I = s.hidden, s.intermediate
        f16 = dict(dtype=torch.float16, device=dev)
        self.x = torch.zeros(H, **f16)
        self.h = torch.zeros(H, **f16)
        self.qkv = torch.zeros(s.qkv_rows, **f16)
        self.ctx = torch.zeros(s.heads * s.head_dim, **f16)
        self.tmp = torch.zeros(H, **f16)
        self.gu = torch.zeros(2 * I, **f16)
        self.act = torch.zeros(I, **f16)
        self.logits = torch.zeros(s.vocab, **f16)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)  # input of the next step
        self.step_idx = torch.zeros(1, dtype=torch.int64, device=dev)
        self.generated = torch.zeros(max_new_tokens, dtype=torch.int64, device=dev)
        self._slot = torch.zeros(1, dtype=torch.int64, device=dev)  # write position in `generated`
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self._prefill_ws = None

    # ------------------------------------------------------------------ one token step
    def _layer(self, l: int):
        if self.projections == "fused":
            return self._layer_fused(l)
        s, w = self.s, self.w
        Hq, Hkv, D = s.heads, s.kv_heads, s.head_dim
        capture_decode_step.rmsnorm(self.x, w.rms_in[l], self.h, s.eps)
        torch.mv(w.w_qkv[l], self.h, out=self.qkv)
        q = self.qkv[: Hq * D].view(1, Hq, D)
        k = self.qkv[Hq * D: (Hq + Hkv) * D].view(1, Hkv, D)
        v = self.qkv[(Hq + Hkv) * D:].view(1, Hkv, D)
        decode_attention(self.arena, l, q, self.ctx.view(1, Hq, D), k_new=k, v_new=v,
                         advance=(l == s.layers - 1), rope_theta=s.rope_theta, prefetch_kv=True)
        torch.mv(w.w_o[l], self.ctx, out=self.tmp)
        self.x.add_(self.tmp)
        capture_decode_step.rmsnorm(self.x, w.rms_post[l], self.h, s.eps)
        torch.mv(w.w_gu[l], self.h, out=self.gu)
        I = s.intermediate
        capture_decode_step.swiglu(self.gu[:I], self.gu[I:], self.act)
        torch.mv(w.w_down[l], self.act, out=self.tmp)
        self.x.add_(self.tmp)

    def _layer_fused(self, l: int):
        """The same layer in five launches: RMSNorm folded into the QKV and gate/up
        projections, SwiGLU into gate/up, the residual adds into O and down."""
        s, w = self.s, self.w
        Hq, Hkv, D = s.heads, s.kv_heads, s.head_dim
        gemv = capture_decode_step.gemv_fused
        gemv(w.w_qkv[l], self.x, self.qkv, "store", w.rms_in[l], s.eps)
        q = self.qkv[: Hq * D].view(1, Hq, D)
        k = self.qkv[Hq * D: (Hq + Hkv) * D].view(1, Hkv, D)
        v = self.qkv[(Hq + Hkv) * D:].view(1, Hkv, D)
        decode_attention(self.arena, l, q, self.ctx.view(1, Hq, D), k_new=k, v_new=v,
                         advance=(l == s.layers - 1), rope_theta=s.rope_theta, prefetch_kv=True)
        gemv(w.w_o[l], self.ctx, self.x, "residual")
        gemv(w.w_gu[l], self.x, self.act, "swiglu", w.rms_post[l], s.eps)
        gemv(w.w_down[l], self.act, self.x, "residual")

    def _step(self):
        """Consumes self.token, leaves the argmax token in self.token and in generated[step_idx]."""
        torch.index_select(self.w.embed, 0, self.token, out=self.x.view(1, -1))
        for l in range(self.s.layers):
            self._layer(l)
        if self.projections == "fused":
            capture_decode_step.gemv_fused(self.w.embed, self.x, self.logits, "store", self.w.rms_final, self.s.eps)
        else:
            capture_decode_step.rmsnorm(self.x, self.w.rms_final, self.h, self.s.eps)
            torch.mv(self.w.embed, self.h, out=self.logits)
        torch.argmax(self.logits.view(1, -1), dim=1, out=self.token)
        # the record of generated tokens wraps around: replays beyond max_new_tokens
        # overwrite the oldest entries instead of indexing past the buffer
        torch.remainder(self.step_idx, self.generated.numel(), out=self._slot)
        self.generated.index_copy_(0, self._slot, self.token)
        self.step_idx.add_(1)

    def capture(self, warmup: int = 0):
        """Capture one token step into a CUDA graph (the arena's seq_len is read on the device, so
        the graph is valid for every length). The caller's state (T, token) is restored."""
        saved_T = self.arena.seq_lens.clone()
        saved_tok, saved_idx = self.token.clone(), self.step_idx.clone()
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):  # first launches set kernel attributes outside the capture
                self._step()
        torch.cuda.current_stream().wait_stream(side)
        self.arena.seq_lens.copy_(saved_T)
        self.token.copy_(saved_tok)
        self.step_idx.copy_(saved_idx)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            self._step()
        torch.cuda.current_stream().wait_stream(side)
        self.arena.seq_lens.copy_(saved_T)
        self.token.copy_(saved_tok)
        self.step_idx.copy_(saved_idx)
        self.graph = g
        return g

    def step(self):
        if self.graph is None:
            self._step()
        else:
            self.graph.replay()

    # ------------------------------------------------------------------ prompt
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Run the prompt (int64 [n] on the device) through the model with the causal varlen
        prefill filling the arena rows [T, T + n); sets self.token to the greedy next token."""
        s, w = self.s, self.w
        n = int(prompt.numel())
        Hq, Hkv, D, H, I = s.heads, s.kv_heads, s.head_dim, s.hidden, s.intermediate
        if self._prefill_ws is None or self._prefill_ws[1] < n:
            ws = attn_varlen.make_prefill_workspace(1, Hq, Hkv, D, n, n, self.arena.capacity, D, self.device)
            self._prefill_ws = (ws, n)
        ws = self._prefill_ws[0]
        cu = torch.tensor([0, n], dtype=torch.int32, device=self.device)
        x = w.embed.index_select(0, prompt)
        h = torch.empty_like(x)
        for l in range(s.layers):
            for i in range(n):  # RMSNorm kernel works one row at a time
                capture_decode_step.rmsnorm(x[i], w.rms_in[l], h[i], s.eps)
            qkv = h @ w.w_qkv[l].t()
            q = qkv[:, : Hq * D].reshape(n, Hq, D)
            k = qkv[:, Hq * D: (Hq + Hkv) * D].reshape(n, Hkv, D)
            v = qkv[:, (Hq + Hkv) * D:].reshape(n, Hkv, D)
            ctx = torch.empty(n, Hq, D, dtype=torch.float16, device=self.device)
            kl, vl = self.arena.layer(l)
            attn_varlen.prefill_varlen(q.contiguous(), k.contiguous(), v.contiguous(), kl, vl, ctx, cu, n,
                                       seq_lens=self.arena.seq_lens, advance=(l == s.layers - 1),
                                       rope_theta=s.rope_theta, workspace=ws)
            x = x + ctx.reshape(n, Hq * D) @ w.w_o[l].t()
            for i in range(n):
                capture_decode_step.rmsnorm(x[i], w.rms_post[l], h[i], s.eps)
            gu = h @ w.w_gu[l].t()
            act = torch.empty(n, I, dtype=torch.float16, device=self.device)
            for i in range(n):
                capture_decode_step.swiglu(gu[i, :I], gu[i, I:], act[i])
            x = x + act @ w.w_down[l].t()
        capture_decode_step.rmsnorm(x[n - 1], w.rms_final, self.h, s.eps)
        torch.mv(w.embed, self.h, out=self.logits)
        torch.argmax(self.logits.view(1, -1), dim=1, out=self.token)
        return self.token

    def generate(self, prompt: torch.Tensor, new_tokens: int) -> List[int]:
        """Greedy continuation of `prompt`: the token after the prompt, then new_tokens - 1 graph steps."""
        if new_tokens > self.generated.numel():
            raise ValueError("new_tokens exceeds max_new_tokens")
        self.arena.seq_lens.zero_()
        self.step_idx.zero_()
        first = self.prefill(prompt)
        self.generated[0:1].copy_(first)
        self.step_idx.fill_(1)
        if self.graph is None:
            self.capture()
        for _ in range(new_tokens - 1):
            self.graph.replay()
        return self.generated[:new_tokens].tolist()
