"""GPU checks of the Llama-2-shaped greedy decode built on the decode-attention path
(one CUDA graph per token step, device-side sequence length, prompt through the
causal prefill).

Against the fp32 oracle (oracle/llama_oracle.py) under teacher forcing: the logits
of every step within relative-L2 2e-2 (fp16 weights and activations through the
whole model, fp32 oracle), and the greedy token equal wherever the oracle's top-2
margin exceeds the largest logit error seen. Graph replays and eager steps give
bit-identical tokens and logits; the arena length advances by one per step.
"""
import pytest
import torch

from oracle import llama_oracle as LO

pytestmark = pytest.mark.gpu


def _small():
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import LlamaShape

    return LlamaShape(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, intermediate=1024, vocab=1000)


def _run(dec, prompt, steps, use_graph):
    dec.arena.seq_lens.zero_()
    dec.step_idx.zero_()
    dec.prefill(prompt)
    dec.generated[0:1].copy_(dec.token)
    dec.step_idx.fill_(1)
    logits, toks = [dec.logits.float().cpu().clone()], [int(dec.token.item())]
    if use_graph and dec.graph is None:
        dec.capture()
    for _ in range(steps):
        if use_graph:
            dec.graph.replay()
        else:
            dec._step()
        logits.append(dec.logits.float().cpu().clone())
        toks.append(int(dec.token.item()))
    return torch.stack(logits), toks


@pytest.mark.parametrize("projections", ["fused", "cublas"])
def test_llama_graph_decode_matches_oracle(projections):
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import GreedyDecoder, LlamaWeights

    shape = _small()
    w = LlamaWeights(shape, seed=3, std=0.05)
    dec = GreedyDecoder(w, capacity=64, max_new_tokens=32, projections=projections)
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, shape.vocab, (9,), generator=g)
    steps = 12
    logits, toks = _run(dec, prompt.cuda(), steps, use_graph=True)
    assert int(dec.arena.seq_lens.item()) == prompt.numel() + steps
    assert dec.generated[: steps + 1].tolist() == toks
    fed = prompt.tolist() + toks[:-1]
    ref = LO.logits_for(w, fed)[prompt.numel() - 1:]
    assert ref.shape == logits.shape
    err = (logits - ref).abs()
    rel = float((logits - ref).norm() / ref.norm())
    assert rel <= 2e-2, f"logits rel-L2 {rel:.3g}"
    top2 = ref.topk(2, dim=1).values
    margin = top2[:, 0] - top2[:, 1]
    sure = margin > 2 * float(err.max())
    assert sure.any()
    assert (ref.argmax(1)[sure] == torch.tensor(toks)[sure]).all()


@pytest.mark.parametrize("projections", ["fused", "cublas"])
def test_llama_graph_replay_equals_eager_steps(projections):
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import GreedyDecoder, LlamaWeights

    shape = _small()
    w = LlamaWeights(shape, seed=5, std=0.05)
    prompt = torch.randint(0, shape.vocab, (7,), generator=torch.Generator().manual_seed(6)).cuda()
    eager = GreedyDecoder(w, capacity=48, max_new_tokens=32, projections=projections)
    graph = GreedyDecoder(w, capacity=48, max_new_tokens=32, projections=projections)
    le, te = _run(eager, prompt, 10, use_graph=False)
    lg, tg = _run(graph, prompt, 10, use_graph=True)
    assert te == tg
    assert torch.equal(le, lg)
    # a second generation with the same graph (lengths restart on the device)
    lg2, tg2 = _run(graph, prompt, 10, use_graph=True)
    assert tg2 == tg and torch.equal(lg2, lg)


@pytest.mark.parametrize("K", [512, 4096, 11008])
def test_gemv_fused_modes_against_torch(K):
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    cds = pkg.capture_decode_step
    g = torch.Generator(device="cuda").manual_seed(K)
    N = 1000
    W = (torch.randn(2 * N, K, device="cuda", generator=g) * 0.05).half()
    x = torch.randn(K, device="cuda", generator=g).half()
    rw = (1 + 0.1 * torch.randn(K, device="cuda", generator=g)).half()
    eps = 1e-5
    # the prologue reproduces the RMSNorm kernel bit for bit
    h = torch.empty_like(x)
    cds.rmsnorm(x, rw, h, eps)
    a = h.float()
    ref = W[:N].float() @ a
    y = torch.empty(N, dtype=torch.float16, device="cuda")
    cds.gemv_fused(W[:N], x, y, "store", rw, eps)
    assert torch.allclose(y.float(), ref, rtol=2e-3, atol=2e-3)
    y0 = torch.empty(N, dtype=torch.float16, device="cuda")
    cds.gemv_fused(W[:N], h, y0, "store")
    assert torch.equal(y0, y), "RMSNorm prologue differs from the RMSNorm kernel"
    # residual: out += fp16(W a)
    base = torch.randn(N, device="cuda", generator=g).half()
    r = base.clone()
    cds.gemv_fused(W[:N], h, r, "residual")
    assert torch.equal(r, (base.float() + y0.float()).half())
    # SwiGLU over gate rows [0, N) and up rows [N, 2N), as the separate kernels on the same fp16 values
    gu = torch.empty(2 * N, dtype=torch.float16, device="cuda")
    cds.gemv_fused(W, h, gu, "store")
    act_ref = torch.empty(N, dtype=torch.float16, device="cuda")
    cds.swiglu(gu[:N], gu[N:], act_ref)
    act = torch.empty(N, dtype=torch.float16, device="cuda")
    cds.gemv_fused(W, x, act, "swiglu", rw, eps)
    assert torch.equal(act, act_ref)
    torch.cuda.synchronize()


def test_gemv_fused_rejects_bad_shapes():
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    cds = pkg.capture_decode_step
    W = torch.zeros(8, 100, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        cds.gemv_fused(W, torch.zeros(100, dtype=torch.float16, device="cuda"),
                       torch.zeros(8, dtype=torch.float16, device="cuda"))  # K not a multiple of 8
    with pytest.raises(RuntimeError):
        cds.gemv_fused(W[:, :96], torch.zeros(96, dtype=torch.float16, device="cuda"),
                       torch.zeros(8, dtype=torch.float16, device="cuda"), "swiglu")  # needs 2N rows
