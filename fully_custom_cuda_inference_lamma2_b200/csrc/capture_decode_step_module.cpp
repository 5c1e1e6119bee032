// Python module `capture_decode_step`: the reference's surface
// (custom_kernels/capture_decode_step.cpp:61-325) with the decode-attention step
// added to capture_decode / capture_decode_ext as optional keyword arguments.
// Existing 6-argument and 20-argument calls behave as in the reference.
#include <pybind11/stl.h>

#include <vector>

#include "binding_common.h"
#include "fcci_compat.h"

using namespace fcci_py;

namespace {

void check_arena(const at::Tensor& ak, const at::Tensor& av) {
    check_half_cuda(ak, "arena_k");
    check_half_cuda(av, "arena_v");
    TORCH_CHECK(ak.dim() == 5 && av.dim() == 5, "arena must be [L, 1, H, max_len, D]");
    TORCH_CHECK(ak.sizes() == av.sizes(), "arena_k and arena_v shapes differ");
}

// The attention step of one layer: with T = seq_len_dev[0], rotate q/k_new at T,
// store k_rot/v_new at arena[layer, 0, :, T, :], write ctx_out = attention of the
// rotated q over keys 0..T, and (advance) seq_len_dev[0] = T + 1 after the reads.
void attention_step(const at::Tensor& arena_k, const at::Tensor& arena_v, const at::Tensor& seq_len_dev,
                    const at::Tensor& q, const at::Tensor& k_new, const at::Tensor& v_new, const at::Tensor& ctx_out,
                    int64_t layer, bool advance, const c10::optional<at::Tensor>& workspace, double scale,
                    double rope_theta, int64_t rotary_dim, const c10::optional<at::Tensor>& q_rot_out) {
    check_arena(arena_k, arena_v);
    TORCH_CHECK(arena_k.size(1) == 1, "arena batch dimension must be 1");
    const int64_t L = arena_k.size(0), Hkv = arena_k.size(2), max_len = arena_k.size(3), D = arena_k.size(4);
    TORCH_CHECK(layer >= 0 && layer < L, "layer out of range");
    TORCH_CHECK(tma_compatible(arena_k) && tma_compatible(arena_v),
                "arena must have a contiguous head_dim and 16-byte aligned strides");
    check_int32_cuda(seq_len_dev, "seq_len_dev");
    TORCH_CHECK(seq_len_dev.numel() >= 1, "seq_len_dev must hold one int32");
    TORCH_CHECK(q.numel() % D == 0, "q must hold Hq * head_dim values");
    const int64_t Hq = q.numel() / D;
    check_rows(q, Hq * D, "q");
    check_rows(k_new, Hkv * D, "k_new");
    check_rows(v_new, Hkv * D, "v_new");
    check_rows(ctx_out, Hq * D, "ctx_out");
    TORCH_CHECK(Hq % Hkv == 0, "query heads must be a multiple of the arena's kv heads");
    fcci_decode_desc d = blank_desc();
    d.B = 1;
    d.Hq = (int32_t)Hq;
    d.Hkv = (int32_t)Hkv;
    d.D = (int32_t)D;
    d.q = q.data_ptr();
    d.q_stride_b = Hq * D;
    d.q_stride_h = D;
    d.k_new = k_new.data_ptr();
    d.k_new_stride_b = Hkv * D;
    d.k_new_stride_h = D;
    d.v_new = v_new.data_ptr();
    d.v_new_stride_b = Hkv * D;
    d.v_new_stride_h = D;
    d.k_cache = static_cast<at::Half*>(arena_k.data_ptr()) + layer * arena_k.stride(0);
    d.k_stride_b = arena_k.stride(1);
    d.k_stride_h = arena_k.stride(2);
    d.k_stride_t = arena_k.stride(3);
    d.v_cache = static_cast<at::Half*>(arena_v.data_ptr()) + layer * arena_v.stride(0);
    d.v_stride_b = arena_v.stride(1);
    d.v_stride_h = arena_v.stride(2);
    d.v_stride_t = arena_v.stride(3);
    d.capacity = (int32_t)max_len;
    d.seq_lens = seq_len_dev.data_ptr<int32_t>();
    d.out = ctx_out.data_ptr();
    d.out_stride_b = Hq * D;
    d.out_stride_h = D;
    if (q_rot_out.has_value() && q_rot_out->defined()) {
        check_rows(*q_rot_out, Hq * D, "q_rot_out");
        d.q_rot_out = q_rot_out->data_ptr();
    }
    d.scale = scale > 0 ? (float)scale : (float)(1.0 / std::sqrt((double)D));
    d.rope_theta = (float)rope_theta;
    d.rotary_dim = (int32_t)(rotary_dim < 0 ? D : rotary_dim);
    d.advance = advance ? 1 : 0;
    at::Tensor ws;
    if (workspace.has_value() && workspace->defined()) ws = *workspace;
    else ws = cached_workspace(1, Hq, Hkv, D, q.device());
    bind_workspace(d, ws);
    d.split = 1;
    check_rc(fcci_decode_attention(&d, current_stream()), "capture_decode_step.attention_step");
}

bool given(const c10::optional<at::Tensor>& t) { return t.has_value() && t->defined(); }

void capture_decode(at::Tensor ctrl_input, at::Tensor arena_k, at::Tensor arena_v, at::Tensor seq_len_dev,
                    at::Tensor pos_dev, at::Tensor logits_out, c10::optional<at::Tensor> q,
                    c10::optional<at::Tensor> k_new, c10::optional<at::Tensor> v_new,
                    c10::optional<at::Tensor> ctx_out, int64_t layer, bool advance,
                    c10::optional<at::Tensor> workspace, double scale, double rope_theta, int64_t rotary_dim,
                    c10::optional<at::Tensor> q_rot_out) {
    TORCH_CHECK(ctrl_input.is_cuda() && arena_k.is_cuda() && arena_v.is_cuda() && seq_len_dev.is_cuda() &&
                    pos_dev.is_cuda() && logits_out.is_cuda(),
                "all tensors must be CUDA");
    c10::cuda::CUDAGuard guard(arena_k.device());
    if (given(q)) {
        TORCH_CHECK(given(k_new) && given(v_new) && given(ctx_out), "the attention step needs q, k_new, v_new and ctx_out");
        attention_step(arena_k, arena_v, seq_len_dev, *q, *k_new, *v_new, *ctx_out, layer, advance, workspace, scale,
                       rope_theta, rotary_dim, q_rot_out);
        return;
    }
    TORCH_CHECK(ctrl_input.scalar_type() == at::kLong && seq_len_dev.scalar_type() == at::kInt &&
                    pos_dev.scalar_type() == at::kInt && logits_out.scalar_type() == at::kFloat,
                "ctrl_input int64, seq_len_dev/pos_dev int32, logits_out fp32");
    check_arena(arena_k, arena_v);
    TORCH_CHECK(arena_k.is_contiguous() && arena_v.is_contiguous(), "arena must be contiguous");
    TORCH_CHECK(logits_out.dim() == 2, "logits_out must be [1, vocab]");
    capture_decode_host(ctrl_input.data_ptr<int64_t>(), arena_k.data_ptr(), arena_v.data_ptr(),
                        seq_len_dev.data_ptr<int32_t>(), pos_dev.data_ptr<int32_t>(), logits_out.data_ptr<float>(),
                        (int32_t)arena_k.size(0), (int32_t)arena_k.size(2), (int32_t)arena_k.size(3),
                        (int32_t)arena_k.size(4), (int32_t)logits_out.size(1), current_stream());
    check_rc(fcci_last_status(), "capture_decode");
}

// Per-layer weights of the whole step, named as the keys of the reference's
// weight_loader.load_and_pack dictionary (custom_kernels/weight_loader.py:367-393).
struct LayerWeights {
    std::vector<uint64_t> qkv_ptrs, o_ptrs, mlp_gate_ptrs, mlp_up_ptrs, mlp_down_ptrs, rms_in_ptrs, rms_post_ptrs;
    uint64_t emb_ptr = 0;
    bool given() const { return !qkv_ptrs.empty(); }
};

// The whole token step behind capture_decode_ext (fcci_llama_decode_step): the token
// from ctrl_input, the residual in mlp_out_s, ctx in x_norm_s, SwiGLU output in act_s,
// q/k/v in qkv_s, fp32 logits in logits_out; seq_len_dev advances by one.
void full_step(const at::Tensor& ctrl_input, const at::Tensor& arena_k, const at::Tensor& arena_v,
               const at::Tensor& seq_len_dev, const at::Tensor& logits_out, const at::Tensor& x_norm_s,
               const at::Tensor& act_s, const at::Tensor& mlp_out_s, uint64_t rms_final_w, uint64_t w_vocab,
               int64_t I, double rms_eps, const LayerWeights& w, const c10::optional<at::Tensor>& qkv_s,
               int64_t q_heads, const c10::optional<at::Tensor>& workspace, double rope_theta, int64_t rotary_dim) {
    check_arena(arena_k, arena_v);
    TORCH_CHECK(arena_k.size(1) == 1, "arena batch dimension must be 1");
    TORCH_CHECK(arena_k.is_contiguous() && arena_v.is_contiguous(), "arena must be contiguous");
    const int64_t L = arena_k.size(0), Hkv = arena_k.size(2), max_len = arena_k.size(3), D = arena_k.size(4);
    const int64_t Hq = q_heads > 0 ? q_heads : Hkv;
    const int64_t H = mlp_out_s.numel(), V = logits_out.size(1);
    TORCH_CHECK(ctrl_input.scalar_type() == at::kLong && ctrl_input.numel() >= 1, "ctrl_input must hold one int64");
    check_int32_cuda(seq_len_dev, "seq_len_dev");
    TORCH_CHECK(logits_out.scalar_type() == at::kFloat && logits_out.dim() == 2 && logits_out.is_contiguous(),
                "logits_out must be a contiguous fp32 [1, vocab]");
    TORCH_CHECK(Hq % Hkv == 0, "q_heads must be a multiple of the arena's kv heads");
    TORCH_CHECK(given(qkv_s), "the whole step needs qkv_s ((q_heads + 2 kv_heads) * head_dim fp16)");
    check_rows(*qkv_s, (Hq + 2 * Hkv) * D, "qkv_s");
    check_rows(x_norm_s, Hq * D, "x_norm_s (holds ctx)");
    check_rows(act_s, I, "act_s");
    check_rows(mlp_out_s, H, "mlp_out_s (holds the residual)");
    auto n_ok = [&](const std::vector<uint64_t>& v) { return (int64_t)v.size() == L; };
    TORCH_CHECK(n_ok(w.qkv_ptrs) && n_ok(w.o_ptrs) && n_ok(w.mlp_gate_ptrs) && n_ok(w.mlp_up_ptrs) &&
                    n_ok(w.mlp_down_ptrs) && n_ok(w.rms_in_ptrs) && n_ok(w.rms_post_ptrs),
                "every per-layer pointer list needs one entry per arena layer (", L, ")");
    TORCH_CHECK(w.emb_ptr != 0 && rms_final_w != 0, "the whole step needs emb_ptr and rms_final_w");
    std::vector<const void*> qkv(L), o(L), gate(L), up(L), down(L), rin(L), rpost(L);
    for (int64_t l = 0; l < L; ++l) {
        qkv[l] = reinterpret_cast<const void*>(w.qkv_ptrs[l]);
        o[l] = reinterpret_cast<const void*>(w.o_ptrs[l]);
        gate[l] = reinterpret_cast<const void*>(w.mlp_gate_ptrs[l]);
        up[l] = reinterpret_cast<const void*>(w.mlp_up_ptrs[l]);
        down[l] = reinterpret_cast<const void*>(w.mlp_down_ptrs[l]);
        rin[l] = reinterpret_cast<const void*>(w.rms_in_ptrs[l]);
        rpost[l] = reinterpret_cast<const void*>(w.rms_post_ptrs[l]);
    }
    at::Tensor ws = given(workspace) ? *workspace : cached_workspace(1, Hq, Hkv, D, arena_k.device());
    TORCH_CHECK(ws.is_cuda() && ws.scalar_type() == at::kByte && ws.is_contiguous(),
                "workspace must be a contiguous uint8 CUDA tensor from attn_varlen.make_workspace()");
    fcci_llama_step_desc d;
    std::memset(&d, 0, sizeof(d));
    d.abi_version = FCCI_LLAMA_STEP_ABI_VERSION;
    d.layers = (int32_t)L;
    d.hidden = (int32_t)H;
    d.q_heads = (int32_t)Hq;
    d.kv_heads = (int32_t)Hkv;
    d.head_dim = (int32_t)D;
    d.intermediate = (int32_t)I;
    d.vocab = (int32_t)V;
    d.rms_eps = (float)rms_eps;
    d.rope_theta = (float)rope_theta;
    d.rotary_dim = (int32_t)rotary_dim;
    d.token = ctrl_input.data_ptr<int64_t>();
    d.embed = reinterpret_cast<const void*>(w.emb_ptr);
    d.w_qkv = qkv.data();
    d.w_o = o.data();
    d.w_gate = gate.data();
    d.w_up = up.data();
    d.w_down = down.data();
    d.rms_in = rin.data();
    d.rms_post = rpost.data();
    d.rms_final = reinterpret_cast<const void*>(rms_final_w);
    d.lm_head = reinterpret_cast<const void*>(w_vocab);
    d.arena_k = arena_k.data_ptr();
    d.arena_v = arena_v.data_ptr();
    d.max_len = (int32_t)max_len;
    d.seq_len = seq_len_dev.data_ptr<int32_t>();
    d.x = mlp_out_s.data_ptr();
    d.qkv = qkv_s->data_ptr();
    d.ctx = x_norm_s.data_ptr();
    d.act = act_s.data_ptr();
    d.logits = logits_out.data_ptr<float>();
    d.workspace = ws.data_ptr();
    d.workspace_bytes = (size_t)ws.numel();
    check_rc(fcci_llama_decode_step(&d, current_stream()), "capture_decode_ext (whole step)");
}

void capture_decode_ext(at::Tensor ctrl_input, at::Tensor arena_k, at::Tensor arena_v, at::Tensor seq_len_dev,
                        at::Tensor pos_dev, at::Tensor logits_out, at::Tensor x_norm_s, at::Tensor gate_out_s,
                        at::Tensor up_out_s, at::Tensor act_s, at::Tensor mlp_out_s, uint64_t rms_in_w,
                        uint64_t rms_post_w, uint64_t rms_final_w, uint64_t w_gate, uint64_t w_up, uint64_t w_down,
                        uint64_t w_vocab, int64_t I, double rms_eps, c10::optional<at::Tensor> q,
                        c10::optional<at::Tensor> k_new, c10::optional<at::Tensor> v_new,
                        c10::optional<at::Tensor> ctx_out, int64_t layer, c10::optional<at::Tensor> workspace,
                        double scale, double rope_theta, int64_t rotary_dim, c10::optional<at::Tensor> q_rot_out,
                        const LayerWeights& lw, c10::optional<at::Tensor> qkv_s, int64_t q_heads) {
    TORCH_CHECK(ctrl_input.is_cuda() && arena_k.is_cuda() && arena_v.is_cuda() && seq_len_dev.is_cuda() &&
                    pos_dev.is_cuda() && logits_out.is_cuda(),
                "all tensors must be CUDA");
    TORCH_CHECK(x_norm_s.is_cuda() && gate_out_s.is_cuda() && up_out_s.is_cuda() && act_s.is_cuda() &&
                    mlp_out_s.is_cuda(),
                "scratch must be CUDA");
    TORCH_CHECK(x_norm_s.scalar_type() == at::kHalf && gate_out_s.scalar_type() == at::kHalf &&
                    up_out_s.scalar_type() == at::kHalf && act_s.scalar_type() == at::kHalf &&
                    mlp_out_s.scalar_type() == at::kHalf,
                "scratch must be fp16");
    c10::cuda::CUDAGuard guard(arena_k.device());
    if (lw.given()) {
        TORCH_CHECK(!given(q), "give either the per-layer weights (whole step) or q/k_new/v_new (one attention step)");
        full_step(ctrl_input, arena_k, arena_v, seq_len_dev, logits_out, x_norm_s, act_s, mlp_out_s, rms_final_w,
                  w_vocab, I, rms_eps, lw, qkv_s, q_heads, workspace, rope_theta, rotary_dim);
        return;
    }
    if (given(q)) {
        TORCH_CHECK(given(k_new) && given(v_new) && given(ctx_out), "the attention step needs q, k_new, v_new and ctx_out");
        // the _ext step bumps seq_len itself (below), so the attention step does not
        attention_step(arena_k, arena_v, seq_len_dev, *q, *k_new, *v_new, *ctx_out, layer, false, workspace, scale,
                       rope_theta, rotary_dim, q_rot_out);
    }
    const int64_t H = arena_k.size(2);
    capture_decode_host_ext(
        ctrl_input.data_ptr<int64_t>(), arena_k.data_ptr(), arena_v.data_ptr(), seq_len_dev.data_ptr<int32_t>(),
        pos_dev.data_ptr<int32_t>(), logits_out.data_ptr<float>(), x_norm_s.data_ptr(), gate_out_s.data_ptr(),
        up_out_s.data_ptr(), act_s.data_ptr(), mlp_out_s.data_ptr(), reinterpret_cast<const void*>(rms_in_w),
        reinterpret_cast<const void*>(rms_post_w), reinterpret_cast<const void*>(rms_final_w),
        reinterpret_cast<const void*>(w_gate), reinterpret_cast<const void*>(w_up),
        reinterpret_cast<const void*>(w_down), reinterpret_cast<const void*>(w_vocab), (int32_t)arena_k.size(0),
        (int32_t)H, (int32_t)arena_k.size(3), (int32_t)arena_k.size(4), (int32_t)logits_out.size(1), (int32_t)I,
        (float)rms_eps, current_stream());
    check_rc(fcci_last_status(), "capture_decode_ext");
}

void rmsnorm(at::Tensor x, at::Tensor w, at::Tensor y, double eps) {
    TORCH_CHECK(x.is_cuda() && w.is_cuda() && y.is_cuda(), "all tensors must be CUDA");
    TORCH_CHECK(x.scalar_type() == at::kHalf && w.scalar_type() == at::kHalf && y.scalar_type() == at::kHalf,
                "x,w,y must be fp16");
    const int32_t H = (int32_t)x.size(-1);
    TORCH_CHECK(w.numel() == H && y.numel() == H, "shape mismatch");
    c10::cuda::CUDAGuard guard(x.device());
    rmsnorm_host(x.data_ptr(), w.data_ptr(), y.data_ptr(), H, (float)eps, current_stream());
    check_rc(fcci_last_status(), "rmsnorm");
}

void rmsnorm_ptr(at::Tensor x, uint64_t w_ptr, at::Tensor y, double eps) {
    TORCH_CHECK(x.is_cuda() && y.is_cuda(), "tensors must be CUDA");
    TORCH_CHECK(x.scalar_type() == at::kHalf && y.scalar_type() == at::kHalf, "x,y must be fp16");
    const int32_t H = (int32_t)x.size(-1);
    TORCH_CHECK(y.numel() == H, "shape mismatch");
    c10::cuda::CUDAGuard guard(x.device());
    rmsnorm_host(x.data_ptr(), reinterpret_cast<const void*>(w_ptr), y.data_ptr(), H, (float)eps, current_stream());
    check_rc(fcci_last_status(), "rmsnorm_ptr");
}

// out = W . a with a = RMSNorm(x) * rms_w (when rms_w is given) or x; mode "store",
// "residual" (out += W . a) or "swiglu" (W holds 2N rows: gate then up; out = SiLU(g) * u).
void gemv_fused(at::Tensor W, at::Tensor x, at::Tensor out, const std::string& mode,
                c10::optional<at::Tensor> rms_w, double eps) {
    TORCH_CHECK(W.is_cuda() && x.is_cuda() && out.is_cuda(), "all tensors must be CUDA");
    TORCH_CHECK(W.scalar_type() == at::kHalf && x.scalar_type() == at::kHalf && out.scalar_type() == at::kHalf,
                "W, x, out must be fp16");
    TORCH_CHECK(W.dim() == 2 && W.stride(1) == 1, "W must be a row-major [rows, K] matrix");
    TORCH_CHECK(x.is_contiguous() && out.is_contiguous(), "x and out must be contiguous");
    const int m = mode == "store" ? 0 : (mode == "residual" ? 1 : (mode == "swiglu" ? 2 : -1));
    TORCH_CHECK(m >= 0, "mode must be 'store', 'residual' or 'swiglu'");
    const int64_t N = out.numel(), K = x.numel();
    TORCH_CHECK(W.size(1) == K, "W columns must equal x length");
    TORCH_CHECK(W.size(0) == (m == 2 ? 2 * N : N), "W rows must be out length (2x for swiglu)");
    TORCH_CHECK(N < (1ll << 31) && K < (1ll << 31), "sizes exceed int32");
    fcci_gemv_desc d;
    std::memset(&d, 0, sizeof(d));
    d.W = W.data_ptr();
    d.ld_w = W.stride(0);
    d.N = (int32_t)N;
    d.K = (int32_t)K;
    d.x = x.data_ptr();
    if (rms_w.has_value() && rms_w->defined()) {
        TORCH_CHECK(rms_w->is_cuda() && rms_w->scalar_type() == at::kHalf && rms_w->numel() == K &&
                        rms_w->is_contiguous(),
                    "rms_w must be a contiguous fp16 [K] CUDA tensor");
        d.rms_w = rms_w->data_ptr();
    }
    d.eps = (float)eps;
    d.out = out.data_ptr();
    d.mode = m;
    c10::cuda::CUDAGuard guard(x.device());
    check_rc(fcci_gemv_fused(&d, current_stream()), "gemv_fused");
}

void swiglu(at::Tensor gate, at::Tensor up, at::Tensor act) {
    TORCH_CHECK(gate.is_cuda() && up.is_cuda() && act.is_cuda(), "all tensors must be CUDA");
    TORCH_CHECK(gate.scalar_type() == at::kHalf && up.scalar_type() == at::kHalf && act.scalar_type() == at::kHalf,
                "gate/up/act must be fp16");
    const int32_t I = (int32_t)gate.numel();
    TORCH_CHECK(up.numel() == I && act.numel() == I, "shape mismatch");
    c10::cuda::CUDAGuard guard(gate.device());
    swiglu_host(gate.data_ptr(), up.data_ptr(), act.data_ptr(), I, current_stream());
    check_rc(fcci_last_status(), "swiglu");
}

void gemv(const at::Tensor& x, at::Tensor& y, uint64_t w_ptr, int64_t rows, int64_t cols, bool fp32_out,
          const char* what) {
    TORCH_CHECK(x.is_cuda() && y.is_cuda(), "tensors must be CUDA");
    TORCH_CHECK(x.scalar_type() == at::kHalf, "fp16 required");
    TORCH_CHECK(y.scalar_type() == (fp32_out ? at::kFloat : at::kHalf), fp32_out ? "y fp16, logits fp32" : "fp16 required");
    c10::cuda::CUDAGuard guard(x.device());
    check_rc(fcci_gemv_rowmajor(reinterpret_cast<const void*>(w_ptr), x.data_ptr(), y.data_ptr(), (int32_t)rows,
                                (int32_t)cols, fp32_out ? 1 : 0, current_stream()),
             what);
}

void gate_up_gemm(at::Tensor x_norm, at::Tensor gate_out, at::Tensor up_out, uint64_t w_gate_ptr, uint64_t w_up_ptr,
                  int64_t H, int64_t I) {
    TORCH_CHECK(x_norm.dim() == 1 && x_norm.size(0) == H, "x_norm shape");
    TORCH_CHECK(gate_out.dim() == 1 && gate_out.size(0) == I, "gate_out shape");
    TORCH_CHECK(up_out.dim() == 1 && up_out.size(0) == I, "up_out shape");
    gemv(x_norm, gate_out, w_gate_ptr, I, H, false, "gate_up_gemm");
    gemv(x_norm, up_out, w_up_ptr, I, H, false, "gate_up_gemm");
}

void down_gemm(at::Tensor act, at::Tensor mlp_out, uint64_t w_down_ptr, int64_t I, int64_t H) {
    TORCH_CHECK(act.dim() == 1 && act.size(0) == I, "act shape");
    TORCH_CHECK(mlp_out.dim() == 1 && mlp_out.size(0) == H, "mlp_out shape");
    gemv(act, mlp_out, w_down_ptr, H, I, false, "down_gemm");
}

void logits_gemm_vocab(at::Tensor y, at::Tensor logits_out, uint64_t w_vocab_ptr, int64_t H, int64_t V) {
    TORCH_CHECK(y.dim() == 1 && y.size(0) == H, "y shape");
    TORCH_CHECK(logits_out.dim() == 1 && logits_out.size(0) == V, "logits shape");
    gemv(y, logits_out, w_vocab_ptr, V, H, true, "logits_gemm_vocab");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "Drop-in for the reference's capture_decode_step extension, with a B200 decode-attention step";
    m.def("capture_decode", &capture_decode,
          "Case4 custom capture/replay decode; with q/k_new/v_new/ctx_out: RoPE + append + attention for `layer`",
          py::arg("ctrl_input"), py::arg("arena_k"), py::arg("arena_v"), py::arg("seq_len_dev"), py::arg("pos_dev"),
          py::arg("logits_out"), py::arg("q") = py::none(), py::arg("k_new") = py::none(),
          py::arg("v_new") = py::none(), py::arg("ctx_out") = py::none(), py::arg("layer") = 0,
          py::arg("advance") = true, py::arg("workspace") = py::none(), py::arg("scale") = -1.0,
          py::arg("rope_theta") = 10000.0, py::arg("rotary_dim") = -1, py::arg("q_rot_out") = py::none());
    // 20 positional arguments as the reference module binds them (capture_decode_step.cpp:85-93), and 25 as the
    // reference's server passes them (case4_graph_generator_server_ipc.py:2261, 2291, 2405, 2526: L, H, max_len,
    // D and vocab before I and rms_eps, which this form checks against the tensors). Keyword arguments add the
    // attention step of one layer (q, k_new, v_new, ctx_out, layer, ...) or, with the per-layer weight lists of
    // weight_loader.load_and_pack (qkv_ptrs, o_ptrs, mlp_gate_ptrs, mlp_up_ptrs, mlp_down_ptrs, rms_in_ptrs,
    // rms_post_ptrs, emb_ptr) and qkv_s, the whole token step of every layer.
    auto ext20 = [](at::Tensor ctrl_input, at::Tensor arena_k, at::Tensor arena_v, at::Tensor seq_len_dev,
                    at::Tensor pos_dev, at::Tensor logits_out, at::Tensor x_norm_s, at::Tensor gate_out_s,
                    at::Tensor up_out_s, at::Tensor act_s, at::Tensor mlp_out_s, uint64_t rms_in_w,
                    uint64_t rms_post_w, uint64_t rms_final_w, uint64_t w_gate, uint64_t w_up, uint64_t w_down,
                    uint64_t w_vocab, int64_t I, double rms_eps, c10::optional<at::Tensor> q,
                    c10::optional<at::Tensor> k_new, c10::optional<at::Tensor> v_new,
                    c10::optional<at::Tensor> ctx_out, int64_t layer, c10::optional<at::Tensor> workspace,
                    double scale, double rope_theta, int64_t rotary_dim, c10::optional<at::Tensor> q_rot_out,
                    std::vector<uint64_t> qkv_ptrs, std::vector<uint64_t> o_ptrs,
                    std::vector<uint64_t> mlp_gate_ptrs, std::vector<uint64_t> mlp_up_ptrs,
                    std::vector<uint64_t> mlp_down_ptrs, std::vector<uint64_t> rms_in_ptrs,
                    std::vector<uint64_t> rms_post_ptrs, uint64_t emb_ptr, c10::optional<at::Tensor> qkv_s,
                    int64_t q_heads) {
        LayerWeights lw{qkv_ptrs, o_ptrs, mlp_gate_ptrs, mlp_up_ptrs, mlp_down_ptrs, rms_in_ptrs, rms_post_ptrs,
                        emb_ptr};
        capture_decode_ext(ctrl_input, arena_k, arena_v, seq_len_dev, pos_dev, logits_out, x_norm_s, gate_out_s,
                           up_out_s, act_s, mlp_out_s, rms_in_w, rms_post_w, rms_final_w, w_gate, w_up, w_down,
                           w_vocab, I, rms_eps, q, k_new, v_new, ctx_out, layer, workspace, scale, rope_theta,
                           rotary_dim, q_rot_out, lw, qkv_s, q_heads);
    };
    auto ext25 = [ext20](at::Tensor ctrl_input, at::Tensor arena_k, at::Tensor arena_v, at::Tensor seq_len_dev,
                         at::Tensor pos_dev, at::Tensor logits_out, at::Tensor x_norm_s, at::Tensor gate_out_s,
                         at::Tensor up_out_s, at::Tensor act_s, at::Tensor mlp_out_s, uint64_t rms_in_w,
                         uint64_t rms_post_w, uint64_t rms_final_w, uint64_t w_gate, uint64_t w_up, uint64_t w_down,
                         uint64_t w_vocab, int64_t L, int64_t H, int64_t max_len, int64_t D, int64_t vocab, int64_t I,
                         double rms_eps, c10::optional<at::Tensor> q, c10::optional<at::Tensor> k_new,
                         c10::optional<at::Tensor> v_new, c10::optional<at::Tensor> ctx_out, int64_t layer,
                         c10::optional<at::Tensor> workspace, double scale, double rope_theta, int64_t rotary_dim,
                         c10::optional<at::Tensor> q_rot_out, std::vector<uint64_t> qkv_ptrs,
                         std::vector<uint64_t> o_ptrs, std::vector<uint64_t> mlp_gate_ptrs,
                         std::vector<uint64_t> mlp_up_ptrs, std::vector<uint64_t> mlp_down_ptrs,
                         std::vector<uint64_t> rms_in_ptrs, std::vector<uint64_t> rms_post_ptrs, uint64_t emb_ptr,
                         c10::optional<at::Tensor> qkv_s, int64_t q_heads) {
        TORCH_CHECK(arena_k.dim() == 5, "arena must be [L, 1, H, max_len, D]");
        TORCH_CHECK(L == arena_k.size(0) && max_len == arena_k.size(3) && D == arena_k.size(4) &&
                        vocab == logits_out.size(1),
                    "capture_decode_ext: L, max_len, D and vocab must match the arena and logits_out");
        TORCH_CHECK(H == arena_k.size(2) || H == mlp_out_s.numel(),
                    "capture_decode_ext: H must be the arena's heads or the hidden size");
        ext20(ctrl_input, arena_k, arena_v, seq_len_dev, pos_dev, logits_out, x_norm_s, gate_out_s, up_out_s, act_s,
              mlp_out_s, rms_in_w, rms_post_w, rms_final_w, w_gate, w_up, w_down, w_vocab, I, rms_eps, q, k_new, v_new,
              ctx_out, layer, workspace, scale, rope_theta, rotary_dim, q_rot_out, qkv_ptrs, o_ptrs, mlp_gate_ptrs,
              mlp_up_ptrs, mlp_down_ptrs, rms_in_ptrs, rms_post_ptrs, emb_ptr, qkv_s, q_heads);
    };
    const char* ext_doc = "Case4 custom capture/replay decode (extended args)";
    m.def("capture_decode_ext", ext20, ext_doc, py::arg("ctrl_input"), py::arg("arena_k"), py::arg("arena_v"),
          py::arg("seq_len_dev"), py::arg("pos_dev"), py::arg("logits_out"), py::arg("x_norm_s"),
          py::arg("gate_out_s"), py::arg("up_out_s"), py::arg("act_s"), py::arg("mlp_out_s"), py::arg("rms_in_w"),
          py::arg("rms_post_w"), py::arg("rms_final_w"), py::arg("w_gate"), py::arg("w_up"), py::arg("w_down"),
          py::arg("w_vocab"), py::arg("I"), py::arg("rms_eps"), py::arg("q") = py::none(),
          py::arg("k_new") = py::none(), py::arg("v_new") = py::none(), py::arg("ctx_out") = py::none(),
          py::arg("layer") = 0, py::arg("workspace") = py::none(), py::arg("scale") = -1.0,
          py::arg("rope_theta") = 10000.0, py::arg("rotary_dim") = -1, py::arg("q_rot_out") = py::none(),
          py::kw_only(), py::arg("qkv_ptrs") = std::vector<uint64_t>(), py::arg("o_ptrs") = std::vector<uint64_t>(),
          py::arg("mlp_gate_ptrs") = std::vector<uint64_t>(), py::arg("mlp_up_ptrs") = std::vector<uint64_t>(),
          py::arg("mlp_down_ptrs") = std::vector<uint64_t>(), py::arg("rms_in_ptrs") = std::vector<uint64_t>(),
          py::arg("rms_post_ptrs") = std::vector<uint64_t>(), py::arg("emb_ptr") = 0,
          py::arg("qkv_s") = py::none(), py::arg("q_heads") = -1);
    m.def("capture_decode_ext", ext25, ext_doc, py::arg("ctrl_input"), py::arg("arena_k"), py::arg("arena_v"),
          py::arg("seq_len_dev"), py::arg("pos_dev"), py::arg("logits_out"), py::arg("x_norm_s"),
          py::arg("gate_out_s"), py::arg("up_out_s"), py::arg("act_s"), py::arg("mlp_out_s"), py::arg("rms_in_w"),
          py::arg("rms_post_w"), py::arg("rms_final_w"), py::arg("w_gate"), py::arg("w_up"), py::arg("w_down"),
          py::arg("w_vocab"), py::arg("L"), py::arg("H"), py::arg("max_len"), py::arg("D"), py::arg("vocab"),
          py::arg("I"), py::arg("rms_eps"), py::arg("q") = py::none(), py::arg("k_new") = py::none(),
          py::arg("v_new") = py::none(), py::arg("ctx_out") = py::none(), py::arg("layer") = 0,
          py::arg("workspace") = py::none(), py::arg("scale") = -1.0, py::arg("rope_theta") = 10000.0,
          py::arg("rotary_dim") = -1, py::arg("q_rot_out") = py::none(), py::kw_only(),
          py::arg("qkv_ptrs") = std::vector<uint64_t>(), py::arg("o_ptrs") = std::vector<uint64_t>(),
          py::arg("mlp_gate_ptrs") = std::vector<uint64_t>(), py::arg("mlp_up_ptrs") = std::vector<uint64_t>(),
          py::arg("mlp_down_ptrs") = std::vector<uint64_t>(), py::arg("rms_in_ptrs") = std::vector<uint64_t>(),
          py::arg("rms_post_ptrs") = std::vector<uint64_t>(), py::arg("emb_ptr") = 0,
          py::arg("qkv_s") = py::none(), py::arg("q_heads") = -1);
    m.def(
        "prepare_cublas", []() { prepare_cublas_handle(current_stream()); },
        "Prepare global cuBLAS handle on current stream (call before capture)");
    m.def("clear_workspace_cache", &clear_workspace_cache,
          "Drop the workspaces kept for attention steps called without one; needed only after a device timeout");
    m.def("rmsnorm", &rmsnorm, "Case4 fused RMSNorm (fp16)");
    m.def("rmsnorm_ptr", &rmsnorm_ptr, "Case4 fused RMSNorm with weight pointer (fp16)");
    m.def("swiglu", &swiglu, "Case4 SwiGLU (fp16)");
    m.def("gemv_fused", &gemv_fused,
          "Batch-1 projection out (=|+=) W . a, a = RMSNorm(x) * rms_w or x; mode store/residual/swiglu",
          py::arg("W"), py::arg("x"), py::arg("out"), py::arg("mode") = "store", py::arg("rms_w") = py::none(),
          py::arg("eps") = 1e-5);
    m.def("gate_up_gemm", &gate_up_gemm, "Case4 MLP gate/up GEMMs (fp16, fp32 accum)");
    m.def("down_gemm", &down_gemm, "Case4 MLP down GEMM (fp16, fp32 accum)");
    m.def("logits_gemm_vocab", &logits_gemm_vocab, "Case4 logits GEMM to vocab (fp16->fp32)");
}
