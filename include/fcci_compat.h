/*
 * fcci_compat.h — the rest of the reference's `capture_decode_step` C ABI.
 *
 * These are the callers around the decode-attention path that the reference
 * exports from the same extension module; they are kept so this library's
 * `capture_decode_step` module is a complete drop-in. Each cites the reference
 * symbol it replaces (paths inside divakar-yadav/Fully_Custom_Cuda_Inference_Lamma2):
 *
 *   capture_decode_host_ext  custom_kernels/capture_decode_step_kernel.cu:137-274
 *   prepare_cublas_handle    custom_kernels/capture_decode_step_kernel.cu:132-134
 *   rmsnorm_host             custom_kernels/capture_decode_step_kernel.cu:276-292
 *   swiglu_host              custom_kernels/capture_decode_step_kernel.cu:294-308
 *   fcci_gemv_rowmajor       custom_kernels/capture_decode_step.cpp:176-310
 *                            (gate_up_gemm / down_gemm / logits_gemm_vocab: y = W x
 *                            with W row-major [rows, cols], fp16 in, fp32 accumulate)
 *
 * GEMMs go through cuBLAS with one handle per device created on first use (or by
 * prepare_cublas_handle before graph capture); the reference instead created and
 * destroyed a handle on every GEMV call (capture_decode_step.cpp:184-213).
 */
#ifndef FCCI_COMPAT_H
#define FCCI_COMPAT_H

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

void capture_decode_host_ext(const int64_t* ctrl_input, void* arena_k, void* arena_v, int32_t* seq_len_ptr,
                             const int32_t* position_ptr, float* logits_out, void* x_norm_scratch,
                             void* gate_out_scratch, void* up_out_scratch, void* act_scratch, void* mlp_out_scratch,
                             const void* rms_in_w, const void* rms_post_w, const void* rms_final_w,
                             const void* mlp_gate_w, const void* mlp_up_w, const void* mlp_down_w,
                             const void* lm_head_w, int32_t L, int32_t H, int32_t max_len, int32_t D, int32_t vocab,
                             int32_t I, float rms_eps, cudaStream_t stream);

void prepare_cublas_handle(cudaStream_t stream);

void rmsnorm_host(const void* x, const void* w, void* y, int32_t H, float eps, cudaStream_t stream);

void swiglu_host(const void* gate, const void* up, void* act, int32_t I, cudaStream_t stream);

/* y[rows] = W[rows, cols] (row-major fp16) . x[cols] (fp16); y is fp16 when
 * y_fp32 == 0, else fp32. Returns FCCI_OK or an FCCI_E* code. */
int fcci_gemv_rowmajor(const void* W, const void* x, void* y, int32_t rows, int32_t cols, int y_fp32,
                       cudaStream_t stream);

/*
 * Fused batch-1 projection of the decode step (no reference counterpart as one call;
 * it fuses, per layer of capture_decode_step_kernel.cu:137-274, the RMSNorm kernel
 * :276-292, the cuBLAS GEMV of capture_decode_step.cpp:176-310, the SwiGLU kernel
 * :294-308 and the residual add):
 *   a    = rms_w ? fp16(x * rsqrt(mean(x^2) + eps) * rms_w) : x          (x [K])
 *   mode 0 (store):     out[n]  = fp16(W[n] . a)                          (out [N])
 *   mode 1 (residual):  out[n]  = fp16(out[n] + fp16(W[n] . a))
 *   mode 2 (SwiGLU):    out[n]  = fp16(SiLU(g) * u), g = fp16(W[n] . a), u = fp16(W[N + n] . a)
 * W row-major fp16 with leading dimension ld_w (elements); K and ld_w multiples of 8;
 * W, x and rms_w 16-byte aligned; fp32 accumulation. In mode 1 `out` may not alias x.
 */
typedef struct fcci_gemv_desc {
    const void* W;
    int64_t ld_w;
    int32_t N, K;
    const void* x;
    const void* rms_w; /* NULL: no RMSNorm prologue */
    float eps;
    void* out;
    int32_t mode;
} fcci_gemv_desc;

int fcci_gemv_fused(const fcci_gemv_desc* desc, cudaStream_t stream);

/*
 * The whole decode step of a Llama-2-shaped model for one token (batch 1). The
 * reference's capture_decode_host_ext (custom_kernels/capture_decode_step_kernel.cu:
 * 137-274) stands in for it with a layer-0 MLP on x = 0; this is the step in the order
 * of the reference's decode driver (scripts/direct_custom_decode_500.py:208-296):
 *
 *   x = embed[token[0]]                        (a token outside [0, vocab) gives zeros)
 *   per layer l:
 *     qkv = W_qkv[l] . RMSNorm(x) * rms_in[l]  rows [q (Hq*D) | k (Hkv*D) | v (Hkv*D)]
 *     RoPE(q, k) at T = seq_len[0]; arena_k/v[l, 0, :, T, :] = k_rot, v;
 *     ctx = softmax(q k^T / sqrt(D)) v over keys 0..T      (GQA: head h reads h / (Hq/Hkv))
 *     x  += W_o[l] . ctx
 *     x  += W_down[l] . (SiLU(W_gate[l] . h) * (W_up[l] . h)),  h = RMSNorm(x) * rms_post[l]
 *   logits = lm_head . RMSNorm(x) * rms_final  (fp32; lm_head NULL = tied to embed)
 *   seq_len[0] = T + 1 (by the last layer's attention launch, after every read of T)
 *
 * Weights are row-major fp16 device matrices (the layout of the reference's
 * weight_loader.load_and_pack: qkv_ptrs [(Hq+2Hkv)*D, hidden], o_ptrs [hidden, Hq*D],
 * mlp_gate_ptrs / mlp_up_ptrs [I, hidden], mlp_down_ptrs [hidden, I]); the per-layer
 * arrays are host arrays of device pointers, read during the call (a captured graph
 * keeps the pointers of its capture). The arena is the reference's [layers, 1, Hkv,
 * max_len, D] fp16. Scratch: x [hidden], qkv [(Hq+2Hkv)*D], ctx [Hq*D], act [I] fp16;
 * workspace: fcci_decode_workspace_bytes(1, Hq, Hkv, D, device) bytes, zeroed once.
 * Nothing is allocated and the host is not synchronised: the call can be captured.
 */
#define FCCI_LLAMA_STEP_ABI_VERSION 1
typedef struct fcci_llama_step_desc {
    int32_t abi_version; /* FCCI_LLAMA_STEP_ABI_VERSION */
    int32_t layers, hidden, q_heads, kv_heads, head_dim, intermediate, vocab;
    float rms_eps, rope_theta;
    int32_t rotary_dim; /* -1: head_dim */
    const int64_t* token;
    const void* embed;
    const void* const* w_qkv;
    const void* const* w_o;
    const void* const* w_gate;
    const void* const* w_up;
    const void* const* w_down;
    const void* const* rms_in;
    const void* const* rms_post;
    const void* rms_final;
    const void* lm_head;
    void* arena_k;
    void* arena_v;
    int32_t max_len;
    int32_t* seq_len;
    void* x;
    void* qkv;
    void* ctx;
    void* act;
    float* logits;
    void* workspace;
    size_t workspace_bytes;
} fcci_llama_step_desc;

int fcci_llama_decode_step(const fcci_llama_step_desc* desc, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FCCI_COMPAT_H */
