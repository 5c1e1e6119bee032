"""The whole token step behind capture_decode_step.capture_decode_ext.

The reference's server captures capture_decode_ext once per sequence length
(case4_graph_generator_server_ipc.py:2261, 2291, 2405, 2526), and the reference's
own step behind it runs layer 0's MLP on x = 0. Given the per-layer weight lists of
the reference's weight loader (qkv_ptrs, o_ptrs, mlp_gate_ptrs, mlp_up_ptrs,
mlp_down_ptrs, rms_in_ptrs, rms_post_ptrs, emb_ptr), the same call here runs the
whole model for the token in ctrl_input: one graph is captured once and replayed
for every length (the length lives on the device), and its fp32 logits must match
the model oracle under teacher forcing within relative-L2 2e-2 (fp16 weights and
activations against fp32), with the greedy token equal wherever the oracle's top-2
margin exceeds twice the largest logit error seen. Without the lists the call keeps
the reference's placeholder behaviour, in its 20-argument form and in the 25-argument
form the server passes.
"""
import pytest
import torch

from oracle import llama_oracle as LO

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _shape():
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import LlamaShape

    return LlamaShape(layers=2, hidden=512, heads=4, kv_heads=2, head_dim=128, intermediate=1024, vocab=1000)


def _weights_kwargs(w):
    s = w.shape
    I = s.intermediate
    L = s.layers
    return dict(qkv_ptrs=[w.w_qkv[l].data_ptr() for l in range(L)],
                o_ptrs=[w.w_o[l].data_ptr() for l in range(L)],
                mlp_gate_ptrs=[w.w_gu[l, :I].data_ptr() for l in range(L)],
                mlp_up_ptrs=[w.w_gu[l, I:].data_ptr() for l in range(L)],
                mlp_down_ptrs=[w.w_down[l].data_ptr() for l in range(L)],
                rms_in_ptrs=[w.rms_in[l].data_ptr() for l in range(L)],
                rms_post_ptrs=[w.rms_post[l].data_ptr() for l in range(L)],
                emb_ptr=w.embed.data_ptr())


def _buffers(s, max_len):
    f16 = dict(dtype=torch.float16, device=DEV)
    return dict(
        ctrl=torch.zeros(1, 1, dtype=torch.int64, device=DEV),
        ak=torch.full((s.layers, 1, s.kv_heads, max_len, s.head_dim), float("nan"), **f16),
        av=torch.full((s.layers, 1, s.kv_heads, max_len, s.head_dim), float("nan"), **f16),
        seq=torch.zeros(1, dtype=torch.int32, device=DEV),
        pos=torch.zeros(1, dtype=torch.int32, device=DEV),
        logits=torch.zeros(1, s.vocab, dtype=torch.float32, device=DEV),
        x_norm=torch.zeros(s.heads * s.head_dim, **f16),
        gate=torch.zeros(s.intermediate, **f16),
        up=torch.zeros(s.intermediate, **f16),
        act=torch.zeros(s.intermediate, **f16),
        mlp_out=torch.zeros(s.hidden, **f16),
        qkv=torch.zeros((s.heads + 2 * s.kv_heads) * s.head_dim, **f16),
    )


def _call(cds, s, w, b, kw, ws, form=20):
    I = s.intermediate
    head = [b["ctrl"], b["ak"], b["av"], b["seq"], b["pos"], b["logits"], b["x_norm"], b["gate"], b["up"], b["act"],
            b["mlp_out"], w.rms_in[0].data_ptr(), w.rms_post[0].data_ptr(), w.rms_final.data_ptr(),
            w.w_gu[0, :I].data_ptr(), w.w_gu[0, I:].data_ptr(), w.w_down[0].data_ptr(), w.embed.data_ptr()]
    if form == 25:
        head += [s.layers, s.hidden, b["ak"].shape[3], s.head_dim, s.vocab]
    cds.capture_decode_ext(*head, I, s.eps, workspace=ws, qkv_s=b["qkv"], q_heads=s.heads, **kw)


def test_capture_decode_ext_whole_step_graph_matches_oracle():
    import fully_custom_cuda_inference_lamma2_b200 as pkg
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import LlamaWeights

    cds, av = pkg.capture_decode_step, pkg.attn_varlen
    s = _shape()
    w = LlamaWeights(s, seed=31, std=0.05)
    b = _buffers(s, max_len=64)
    kw = _weights_kwargs(w)
    ws = av.make_workspace(1, s.heads, s.kv_heads, s.head_dim)
    # one eager step first (kernel attributes are set outside the capture), then from T = 0
    _call(cds, s, w, b, kw, ws)
    torch.cuda.synchronize()
    b["seq"].zero_()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            _call(cds, s, w, b, kw, ws)
    torch.cuda.synchronize()
    tokens = torch.randint(0, s.vocab, (20,), generator=torch.Generator().manual_seed(32)).tolist()
    mem0 = torch.cuda.memory_allocated()
    got = []
    for t, tok in enumerate(tokens):  # teacher forcing: the graph consumes ctrl_input
        b["ctrl"].fill_(tok)
        g.replay()
        torch.cuda.synchronize()
        assert int(b["seq"].item()) == t + 1
        got.append(b["logits"][0].cpu().clone())
    assert torch.cuda.memory_allocated() == mem0
    got = torch.stack(got)
    ref = LO.logits_for(w, tokens)
    rel = float((got - ref).norm() / ref.norm())
    assert rel <= 2e-2, f"logits rel-L2 {rel:.3g}"
    err = float((got - ref).abs().max())
    top2 = ref.topk(2, dim=1).values
    sure = (top2[:, 0] - top2[:, 1]) > 2 * err
    assert sure.any()
    assert (got.argmax(1)[sure] == ref.argmax(1)[sure]).all()
    assert av.read_error(ws) == 0


def test_capture_decode_ext_whole_step_equals_model_decoder():
    """The C-ABI step and the Python-composed step of GreedyDecoder (same kernels) give
    bit-identical logits and arenas for the same tokens."""
    import fully_custom_cuda_inference_lamma2_b200 as pkg
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import GreedyDecoder, LlamaWeights

    cds, av = pkg.capture_decode_step, pkg.attn_varlen
    s = _shape()
    w = LlamaWeights(s, seed=33, std=0.05)
    max_len = 32
    b = _buffers(s, max_len)
    b["ak"].zero_()
    b["av"].zero_()
    kw = _weights_kwargs(w)
    ws = av.make_workspace(1, s.heads, s.kv_heads, s.head_dim)
    dec = GreedyDecoder(w, capacity=max_len, max_new_tokens=16)
    dec.arena.k.zero_()
    dec.arena.v.zero_()
    dec.arena.seq_lens.zero_()
    tokens = torch.randint(0, s.vocab, (6,), generator=torch.Generator().manual_seed(34)).tolist()
    for tok in tokens:
        b["ctrl"].fill_(tok)
        _call(cds, s, w, b, kw, ws, form=25)
        dec.token.fill_(tok)
        dec._step()
        torch.cuda.synchronize()
        assert torch.equal(b["logits"][0].half(), dec.logits)
    assert torch.equal(b["ak"][:, 0], dec.arena.k[:, 0]) and torch.equal(b["av"][:, 0], dec.arena.v[:, 0])
    assert int(b["seq"].item()) == int(dec.arena.seq_lens.item()) == len(tokens)


def test_capture_decode_ext_server_form_keeps_the_placeholder():
    """The 25 positional arguments of the server's calls, without weight lists: the same
    placeholder result as the reference module's 20-argument form."""
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    cds = pkg.capture_decode_step
    L, H, max_len, D, vocab, I = 2, 4, 8, 128, 64, 32
    outs = []
    for form in (20, 25):
        ak = torch.ones(L, 1, H, max_len, D, dtype=torch.float16, device=DEV)
        c = torch.full((1, 1), 5, dtype=torch.int64, device=DEV)
        sl = torch.tensor([3], dtype=torch.int32, device=DEV)
        logits = torch.full((1, vocab), 5.0, device=DEV)
        scr = [torch.full((n,), 1.0, dtype=torch.float16, device=DEV) for n in (H * D, I, I, I, H * D)]
        args = [c, ak, ak.clone(), sl, sl.clone(), logits, *scr, 0, 0, 0, 0, 0, 0, 0]
        if form == 25:
            args += [L, H * D, max_len, D, vocab]
        cds.capture_decode_ext(*args, I, 1e-5)
        torch.cuda.synchronize()
        outs.append((ak.cpu(), logits.cpu(), int(sl.item()), [t.cpu() for t in scr]))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert outs[0][2] == outs[1][2] == 4
    assert all(torch.equal(a, b) for a, b in zip(outs[0][3], outs[1][3]))
    with pytest.raises((RuntimeError, TypeError)):
        bad = [c, ak, ak, sl, sl, logits, *scr, 0, 0, 0, 0, 0, 0, 0, L + 1, H, max_len, D, vocab, I, 1e-5]
        cds.capture_decode_ext(*bad)
