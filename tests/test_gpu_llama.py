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


def test_llama_graph_decode_matches_oracle():
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import GreedyDecoder, LlamaWeights

    shape = _small()
    w = LlamaWeights(shape, seed=3, std=0.05)
    dec = GreedyDecoder(w, capacity=64, max_new_tokens=32)
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


def test_llama_graph_replay_equals_eager_steps():
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import GreedyDecoder, LlamaWeights

    shape = _small()
    w = LlamaWeights(shape, seed=5, std=0.05)
    prompt = torch.randint(0, shape.vocab, (7,), generator=torch.Generator().manual_seed(6)).cuda()
    eager = GreedyDecoder(w, capacity=48, max_new_tokens=32)
    graph = GreedyDecoder(w, capacity=48, max_new_tokens=32)
    le, te = _run(eager, prompt, 10, use_graph=False)
    lg, tg = _run(graph, prompt, 10, use_graph=True)
    assert te == tg
    assert torch.equal(le, lg)
    # a second generation with the same graph (lengths restart on the device)
    lg2, tg2 = _run(graph, prompt, 10, use_graph=True)
    assert tg2 == tg and torch.equal(lg2, lg)
