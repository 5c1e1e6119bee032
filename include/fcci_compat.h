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

#ifdef __cplusplus
}
#endif

#endif /* FCCI_COMPAT_H */
