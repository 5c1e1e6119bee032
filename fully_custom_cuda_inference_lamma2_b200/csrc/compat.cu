// The non-attention parts of the reference's capture_decode_step extension:
// RMSNorm, SwiGLU, cuBLAS GEMVs and the `_ext` placeholder step. They are callers
// of the decode-attention path kept for module compatibility, not the hot path.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "fcci_compat.h"
#include "fcci_decode.h"
#include "fcci_internal.h"

namespace fcci {

// y = x * rsqrt(mean(x^2) + eps) * w for one fp16 vector (one CTA), as
// capture_decode_step_kernel.cu:10-40, with a shuffle reduction.
__global__ void rmsnorm_kernel(const __half* __restrict__ x, const __half* __restrict__ w, __half* __restrict__ y,
                               int H, float eps) {
    __shared__ float warp_sums[32];
    float local = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = __half2float(x[i]);
        local += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = local;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? warp_sums[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) warp_sums[0] = v;
    }
    __syncthreads();
    const float inv_rms = rsqrtf(warp_sums[0] / (float)(H > 1 ? H : 1) + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        // x and y may alias (the reference normalises x_norm in place)
        const float v = __half2float(x[i]);
        y[i] = __float2half(v * inv_rms * __half2float(w[i]));
    }
}

// act = SiLU(g) * u (capture_decode_step_kernel.cu:43-56)
__global__ void swiglu_kernel(const __half* __restrict__ gate, const __half* __restrict__ up, __half* __restrict__ act,
                              int I) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < I; i += blockDim.x * gridDim.x) {
        const float g = __half2float(gate[i]);
        const float u = __half2float(up[i]);
        act[i] = __float2half(g / (1.0f + expf(-g)) * u);
    }
}

__global__ void inc_seq_len_kernel(int32_t* seq_len) {
    if (threadIdx.x == 0 && blockIdx.x == 0) seq_len[0] += 1;
}

struct CublasSlot {
    std::mutex mu;
    cublasHandle_t handle = nullptr;
};

static CublasSlot& cublas_slot(int dev) {
    static CublasSlot slots[128];
    return slots[dev < 0 ? 0 : (dev & 127)];
}

// Runs fn(handle) with the device's handle bound to `stream`, serialised per device.
template <class F>
static int with_cublas(cudaStream_t stream, F fn) {
    int dev = 0;
    cudaGetDevice(&dev);
    CublasSlot& s = cublas_slot(dev);
    std::lock_guard<std::mutex> lk(s.mu);
    if (!s.handle && cublasCreate(&s.handle) != CUBLAS_STATUS_SUCCESS) {
        s.handle = nullptr;
        return set_status(FCCI_ECUDA, "cublasCreate failed");
    }
    if (cublasSetStream(s.handle, stream) != CUBLAS_STATUS_SUCCESS) return set_status(FCCI_ECUDA, "cublasSetStream failed");
    const cublasStatus_t st = fn(s.handle);
    if (st != CUBLAS_STATUS_SUCCESS) return set_status(FCCI_ECUDA, "cublasGemmEx failed");
    return set_status(FCCI_OK, nullptr);
}

}  // namespace fcci

extern "C" {

void prepare_cublas_handle(cudaStream_t stream) {
    fcci::with_cublas(stream, [](cublasHandle_t) { return CUBLAS_STATUS_SUCCESS; });
}

void rmsnorm_host(const void* x, const void* w, void* y, int32_t H, float eps, cudaStream_t stream) {
    if (!x || !w || !y || H <= 0) {
        fcci::set_status(FCCI_EINVAL, "rmsnorm_host: invalid argument");
        return;
    }
    fcci::rmsnorm_kernel<<<1, 256, 0, stream>>>(static_cast<const __half*>(x), static_cast<const __half*>(w),
                                                 static_cast<__half*>(y), H, eps);
    fcci::count_launch();
    fcci::set_cuda_status(cudaGetLastError());
}

void swiglu_host(const void* gate, const void* up, void* act, int32_t I, cudaStream_t stream) {
    if (!gate || !up || !act || I <= 0) {
        fcci::set_status(FCCI_EINVAL, "swiglu_host: invalid argument");
        return;
    }
    const int blocks = (I + 255) / 256;
    fcci::swiglu_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __half*>(gate), static_cast<const __half*>(up),
                                                     static_cast<__half*>(act), I);
    fcci::count_launch();
    fcci::set_cuda_status(cudaGetLastError());
}

int fcci_gemv_rowmajor(const void* W, const void* x, void* y, int32_t rows, int32_t cols, int y_fp32,
                       cudaStream_t stream) {
    if (!W || !x || !y || rows <= 0 || cols <= 0) return fcci::set_status(FCCI_EINVAL, "fcci_gemv_rowmajor: invalid");
    // column-major view: W^T is [cols, rows] with ld = cols; y = op(W^T)=T applied to x
    return fcci::with_cublas(stream, [&](cublasHandle_t h) {
        const float alpha = 1.f, beta = 0.f;
        return cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, rows, 1, cols, &alpha, W, CUDA_R_16F, cols, x, CUDA_R_16F,
                            cols, &beta, y, y_fp32 ? CUDA_R_32F : CUDA_R_16F, rows, CUBLAS_COMPUTE_32F,
                            CUBLAS_GEMM_DEFAULT);
    });
}

// The reference's `_ext` step runs its MLP on x = 0 for layer 0 only, with
// CUBLAS_OP_N on the row-major weights (capture_decode_step_kernel.cu:190-243);
// the same calls are issued here so results match it on the same inputs.
void capture_decode_host_ext(const int64_t* ctrl_input, void* arena_k, void* arena_v, int32_t* seq_len_ptr,
                             const int32_t* position_ptr, float* logits_out, void* x_norm_scratch,
                             void* gate_out_scratch, void* up_out_scratch, void* act_scratch, void* mlp_out_scratch,
                             const void* rms_in_w, const void* rms_post_w, const void* rms_final_w,
                             const void* mlp_gate_w, const void* mlp_up_w, const void* mlp_down_w,
                             const void* lm_head_w, int32_t L, int32_t H, int32_t max_len, int32_t D, int32_t vocab,
                             int32_t I, float rms_eps, cudaStream_t stream) {
    (void)ctrl_input;
    (void)arena_k;
    (void)arena_v;
    (void)position_ptr;
    (void)rms_post_w;
    (void)L;
    (void)max_len;
    (void)D;
    if (!seq_len_ptr || !logits_out || !x_norm_scratch || !gate_out_scratch || !up_out_scratch || !act_scratch ||
        !mlp_out_scratch || H <= 0 || vocab <= 0 || I < 0) {
        fcci::set_status(FCCI_EINVAL, "capture_decode_host_ext: invalid argument");
        return;
    }
    __half* x_norm = static_cast<__half*>(x_norm_scratch);
    __half* gate_o = static_cast<__half*>(gate_out_scratch);
    __half* up_o = static_cast<__half*>(up_out_scratch);
    __half* act_o = static_cast<__half*>(act_scratch);
    __half* mlp_o = static_cast<__half*>(mlp_out_scratch);
    cudaMemsetAsync(x_norm, 0, sizeof(__half) * H, stream);
    cudaMemsetAsync(gate_o, 0, sizeof(__half) * I, stream);
    cudaMemsetAsync(up_o, 0, sizeof(__half) * I, stream);
    cudaMemsetAsync(act_o, 0, sizeof(__half) * I, stream);
    cudaMemsetAsync(mlp_o, 0, sizeof(__half) * H, stream);
    cudaMemsetAsync(logits_out, 0, sizeof(float) * vocab, stream);
    int rc = FCCI_OK;
    if (rms_in_w) {
        fcci::rmsnorm_kernel<<<1, 256, 0, stream>>>(x_norm, static_cast<const __half*>(rms_in_w), x_norm, H, rms_eps);
        fcci::count_launch();
    }
    if (mlp_gate_w && mlp_up_w && mlp_down_w && I > 0) {
        rc = fcci::with_cublas(stream, [&](cublasHandle_t h) {
            const float alpha = 1.f, beta = 0.f;
            cublasStatus_t s = cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, I, 1, H, &alpha, mlp_gate_w, CUDA_R_16F, I,
                                            x_norm, CUDA_R_16F, H, &beta, gate_o, CUDA_R_16F, I, CUBLAS_COMPUTE_32F,
                                            CUBLAS_GEMM_DEFAULT);
            if (s != CUBLAS_STATUS_SUCCESS) return s;
            return cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, I, 1, H, &alpha, mlp_up_w, CUDA_R_16F, I, x_norm,
                                CUDA_R_16F, H, &beta, up_o, CUDA_R_16F, I, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
        });
        fcci::swiglu_kernel<<<(I + 255) / 256, 256, 0, stream>>>(gate_o, up_o, act_o, I);
        fcci::count_launch();
        if (!rc) {
            rc = fcci::with_cublas(stream, [&](cublasHandle_t h) {
                const float alpha = 1.f, beta = 0.f;
                return cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, H, 1, I, &alpha, mlp_down_w, CUDA_R_16F, H, act_o,
                                    CUDA_R_16F, I, &beta, mlp_o, CUDA_R_16F, H, CUBLAS_COMPUTE_32F,
                                    CUBLAS_GEMM_DEFAULT);
            });
        }
    }
    __half* y_final = mlp_o;
    if (rms_final_w) {
        fcci::rmsnorm_kernel<<<1, 256, 0, stream>>>(y_final, static_cast<const __half*>(rms_final_w), x_norm, H,
                                                     rms_eps);
        fcci::count_launch();
        y_final = x_norm;
    }
    if (lm_head_w && !rc) {
        rc = fcci::with_cublas(stream, [&](cublasHandle_t h) {
            const float alpha = 1.f, beta = 0.f;
            return cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, vocab, 1, H, &alpha, lm_head_w, CUDA_R_16F, vocab,
                                y_final, CUDA_R_16F, H, &beta, logits_out, CUDA_R_32F, vocab, CUBLAS_COMPUTE_32F,
                                CUBLAS_GEMM_DEFAULT);
        });
    }
    fcci::inc_seq_len_kernel<<<1, 1, 0, stream>>>(seq_len_ptr);
    fcci::count_launch();
    if (!rc) fcci::set_cuda_status(cudaGetLastError());
}

}  // extern "C"
