// fcci_llama_decode_step: one decode token of a Llama-2-shaped model (batch 1),
// every layer, as a fixed sequence of launches that a CUDA graph can hold.
//
// The reference's in-graph step, capture_decode_host_ext
// (custom_kernels/capture_decode_step_kernel.cu:137-274), stands in for this with
// its MLP on x = 0 for layer 0 only. This is the step it stands in for, in the order
// of the reference's standalone decode driver (scripts/direct_custom_decode_500.py:
// 208-296), per layer:
//   qkv  = W_qkv . RMSNorm(x) * rms_in                 (fused projection)
//   RoPE(q, k) at T, append (k, v) at T, attention over T + 1 keys
//                                                       (decode_attn_kernel; the last
//                                                        layer advances T)
//   x   += W_o . ctx                                    (fused residual)
//   act  = SiLU(W_gate . h) * (W_up . h), h = RMSNorm(x) * rms_post
//   x   += W_down . act
// then logits = W_vocab . RMSNorm(x) * rms_final in fp32. The token comes from the
// device (token[0]), T from the device (seq_len[0]): one graph serves every length.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>
#include <string.h>

#include "fcci_compat.h"
#include "fcci_decode.h"
#include "fcci_internal.h"

namespace fcci {

// x[0..H) = embed[token[0], 0..H) in 16-byte chunks; a token outside [0, vocab)
// gives a zero row (nothing is read out of range).
__global__ void __launch_bounds__(256) embed_row_kernel(const int64_t* __restrict__ token,
                                                        const __half* __restrict__ embed, int vocab, int H,
                                                        __half* __restrict__ x) {
    const int64_t t = token[0];
    const bool ok = t >= 0 && t < vocab;
    const uint4* src = reinterpret_cast<const uint4*>(embed + (ok ? t : 0) * (int64_t)H);
    uint4* dst = reinterpret_cast<uint4*>(x);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = ok ? src[c] : make_uint4(0u, 0u, 0u, 0u);
}

}  // namespace fcci

extern "C" int fcci_llama_decode_step(const fcci_llama_step_desc* d, cudaStream_t stream) {
    using namespace fcci;
    auto bad = [](const char* why) { return set_status(FCCI_EINVAL, why); };
    if (!d) return bad("fcci_llama_decode_step: descriptor is NULL");
    if (d->abi_version != FCCI_LLAMA_STEP_ABI_VERSION) return bad("fcci_llama_decode_step: abi_version mismatch");
    const int L = d->layers, H = d->hidden, Hq = d->q_heads, Hkv = d->kv_heads, D = d->head_dim;
    const int I = d->intermediate, V = d->vocab;
    if (L <= 0 || H <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || I <= 0 || V <= 0 || Hq % Hkv)
        return bad("fcci_llama_decode_step: sizes must be positive and q_heads a multiple of kv_heads");
    if ((H & 7) || (I & 7) || ((Hq * D) & 7)) return bad("fcci_llama_decode_step: hidden, intermediate, q_heads*head_dim must be multiples of 8");
    if (!d->token || !d->embed || !d->arena_k || !d->arena_v || !d->seq_len || !d->x || !d->qkv || !d->ctx ||
        !d->act || !d->logits || !d->rms_final || !d->workspace)
        return bad("fcci_llama_decode_step: a required pointer is NULL");
    if (!d->w_qkv || !d->w_o || !d->w_gate || !d->w_up || !d->w_down || !d->rms_in || !d->rms_post)
        return bad("fcci_llama_decode_step: per-layer weight arrays are required");
    for (int l = 0; l < L; ++l)
        if (!d->w_qkv[l] || !d->w_o[l] || !d->w_gate[l] || !d->w_up[l] || !d->w_down[l] || !d->rms_in[l] ||
            !d->rms_post[l])
            return bad("fcci_llama_decode_step: a per-layer weight pointer is NULL");
    if (d->max_len <= 0) return bad("fcci_llama_decode_step: max_len must be positive");

    embed_row_kernel<<<1, 256, 0, stream>>>(d->token, static_cast<const __half*>(d->embed), V, H,
                                            static_cast<__half*>(d->x));
    count_launch();
    int rc = set_cuda_status(cudaGetLastError());
    if (rc) return rc;

    const int qkv_rows = (Hq + 2 * Hkv) * D;
    __half* qkv = static_cast<__half*>(d->qkv);
    const int64_t layer_elems = (int64_t)Hkv * d->max_len * D;  // arena [L, 1, Hkv, max_len, D]
    for (int l = 0; l < L; ++l) {
        GemvArgs g;
        memset(&g, 0, sizeof(g));
        g.W = d->w_qkv[l];
        g.ld_w = H;
        g.N = qkv_rows;
        g.K = H;
        g.x = d->x;
        g.rms_w = d->rms_in[l];
        g.eps = d->rms_eps;
        g.out = qkv;
        g.mode = 0;
        if ((rc = gemv(&g, stream))) return rc;

        fcci_decode_desc a;
        memset(&a, 0, sizeof(a));
        a.abi_version = FCCI_DECODE_ABI_VERSION;
        a.B = 1;
        a.Hq = Hq;
        a.Hkv = Hkv;
        a.D = D;
        a.q = qkv;
        a.q_stride_b = (int64_t)Hq * D;
        a.q_stride_h = D;
        a.k_new = qkv + (int64_t)Hq * D;
        a.k_new_stride_b = (int64_t)Hkv * D;
        a.k_new_stride_h = D;
        a.v_new = qkv + (int64_t)(Hq + Hkv) * D;
        a.v_new_stride_b = (int64_t)Hkv * D;
        a.v_new_stride_h = D;
        a.k_cache = static_cast<__half*>(d->arena_k) + l * layer_elems;
        a.v_cache = static_cast<__half*>(d->arena_v) + l * layer_elems;
        a.k_stride_b = a.v_stride_b = layer_elems;
        a.k_stride_h = a.v_stride_h = (int64_t)d->max_len * D;
        a.k_stride_t = a.v_stride_t = D;
        a.capacity = d->max_len;
        a.seq_lens = d->seq_len;
        a.out = d->ctx;
        a.out_stride_b = (int64_t)Hq * D;
        a.out_stride_h = D;
        a.scale = (float)(1.0 / sqrt((double)D));  // as the pybind surfaces compute the default
        a.rope_theta = d->rope_theta;
        a.rotary_dim = d->rotary_dim < 0 ? D : d->rotary_dim;
        a.advance = l == L - 1;
        a.split = 1;
        a.workspace = d->workspace;
        a.workspace_bytes = d->workspace_bytes;
        // the only kernel before this one on the stream is the QKV projection, which
        // writes neither the lengths nor this layer's cached rows
        a.flags = FCCI_DECODE_PREFETCH_KV;
        if ((rc = decode_attention(&a, stream))) return rc;

        g.W = d->w_o[l];
        g.ld_w = (int64_t)Hq * D;
        g.N = H;
        g.K = Hq * D;
        g.x = d->ctx;
        g.rms_w = nullptr;
        g.out = d->x;
        g.mode = 1;
        if ((rc = gemv(&g, stream))) return rc;

        g.W = d->w_gate[l];
        g.W2 = d->w_up[l];
        g.ld_w = H;
        g.N = I;
        g.K = H;
        g.x = d->x;
        g.rms_w = d->rms_post[l];
        g.out = d->act;
        g.mode = 2;
        if ((rc = gemv(&g, stream))) return rc;

        g.W = d->w_down[l];
        g.W2 = nullptr;
        g.ld_w = I;
        g.N = H;
        g.K = I;
        g.x = d->act;
        g.rms_w = nullptr;
        g.out = d->x;
        g.mode = 1;
        if ((rc = gemv(&g, stream))) return rc;
    }
    GemvArgs g;
    memset(&g, 0, sizeof(g));
    g.W = d->lm_head ? d->lm_head : d->embed;
    g.ld_w = H;
    g.N = V;
    g.K = H;
    g.x = d->x;
    g.rms_w = d->rms_final;
    g.eps = d->rms_eps;
    g.out = d->logits;
    g.mode = 3;
    return gemv(&g, stream);
}
