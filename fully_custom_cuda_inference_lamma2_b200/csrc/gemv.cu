// Batch-1 projections of the decode step, fused with their neighbours:
//   y = W a                    with a = RMSNorm(x) * w_rms (prologue) or a = x
//   out  = y                   (mode STORE)
//   out += y                   (mode RESIDUAL: the residual stream update)
//   out  = SiLU(y_g) * y_u     (mode SWIGLU: W holds the gate rows, then the up rows,
//                               or the up rows are a second matrix W2)
//   out  = y in fp32           (mode STORE_F32: the vocab projection's logits)
// They replace, per layer of the reference's in-graph step
// (custom_kernels/capture_decode_step_kernel.cu:137-274, capture_decode_step.cpp:176-310),
// the RMSNorm kernel, the cuBLAS GEMV, the SwiGLU kernel and the residual add as
// separate launches. The rounding of each fused stage is that of the separate
// kernels: the normalised vector is rounded to fp16 before the product, y is
// rounded to fp16 before the residual add or the SwiGLU.
//
// HBM-bound: every weight byte is read once per token (16-byte cache-streaming
// loads), a warp computes kRpw rows at a time with the vector held in shared
// memory; a persistent grid of one wave pays the prologue once per CTA.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fcci_compat.h"
#include "fcci_decode.h"
#include "fcci_internal.h"
#include "ptx.cuh"

namespace fcci {
namespace gv {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRpw = 2;  // output rows per warp per pass

// 16-byte chunks per row in flight per lane (the SwiGLU mode reads twice the rows)
template <int MODE>
struct Unroll {
    static constexpr int value = MODE == 2 ? 4 : 8;
};

enum Mode { kStore = 0, kResidual = 1, kSwiglu = 2, kStoreF32 = 3 };

__device__ __forceinline__ float dot8(uint4 w, uint4 a) {
    const __half2* wh = reinterpret_cast<const __half2*>(&w);
    const __half2* ah = reinterpret_cast<const __half2*>(&a);
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 wf = __half22float2(wh[q]);
        const float2 af = __half22float2(ah[q]);
        s = fmaf(wf.x, af.x, s);
        s = fmaf(wf.y, af.y, s);
    }
    return s;
}

template <int MODE, bool NORM>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const __half* __restrict__ W, const __half* __restrict__ W2,
                                                        int64_t ldw, int N, int K, const __half* __restrict__ x,
                                                        const __half* __restrict__ rms_w, float eps,
                                                        void* __restrict__ out_) {
    __half* out = static_cast<__half*>(out_);
    extern __shared__ __align__(16) uint8_t gv_sm[];
    uint4* a_s = reinterpret_cast<uint4*>(gv_sm);  // K / 8 chunks of the input vector
    __shared__ float red[kWarps];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nchunk = K >> 3;
    // a programmatic dependent of this launch (the decode-attention kernel) may start its
    // set-up now; it waits for this grid's completion before reading anything
    griddep_launch_dependents();

    // ---- prologue: the input vector (normalised when asked) into shared memory
    if (NORM) {
        float ss = 0.f;
        for (int c = tid; c < nchunk; c += kThreads) {
            const uint4 v = reinterpret_cast<const uint4*>(x)[c];
            const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = __half22float2(h[q]);
                ss = fmaf(f.x, f.x, ss);
                ss = fmaf(f.y, f.y, ss);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += red[w];
        const float inv = rsqrtf(tot / (float)K + eps);
        for (int c = tid; c < nchunk; c += kThreads) {
            const uint4 v = reinterpret_cast<const uint4*>(x)[c];
            const uint4 g = reinterpret_cast<const uint4*>(rms_w)[c];
            const __half* hv = reinterpret_cast<const __half*>(&v);
            const __half* hg = reinterpret_cast<const __half*>(&g);
            uint4 r;
            __half* hr = reinterpret_cast<__half*>(&r);
#pragma unroll
            for (int e = 0; e < 8; ++e) hr[e] = __float2half(__half2float(hv[e]) * inv * __half2float(hg[e]));
            a_s[c] = r;
        }
    } else {
        for (int c = tid; c < nchunk; c += kThreads) a_s[c] = reinterpret_cast<const uint4*>(x)[c];
    }
    __syncthreads();

    // ---- rows: a persistent grid; warp w of CTA b takes outputs
    //      [(b * kWarps + w) * kRpw, + kRpw), then strides by the whole grid
    constexpr int NR = MODE == kSwiglu ? 2 * kRpw : kRpw;  // weight rows read per warp
    constexpr int kUnroll = Unroll<MODE>::value;
    for (int n0 = (blockIdx.x * kWarps + warp) * kRpw; n0 < N; n0 += gridDim.x * kWarps * kRpw) {
    const __half* wr[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        // SWIGLU: rows 0..kRpw-1 are the gate rows n0+r, rows kRpw.. the up rows N+n0+r
        // (or rows n0+r of W2)
        const int o = r % kRpw;
        const bool up = MODE == kSwiglu && r >= kRpw;
        const int64_t row = (up && !W2) ? (int64_t)N + n0 + o : (int64_t)n0 + o;
        wr[r] = (n0 + o < N) ? (up && W2 ? W2 : W) + row * ldw : nullptr;
    }
    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.f;
    for (int c0 = lane; c0 < nchunk; c0 += 32 * kUnroll) {
        uint4 wv[kUnroll][NR];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < NR; ++r)
                wv[u][r] = (c < nchunk && wr[r]) ? __ldcs(reinterpret_cast<const uint4*>(wr[r]) + c)
                                                 : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int c = c0 + 32 * u;
            if (c < nchunk) {
                const uint4 av = a_s[c];
#pragma unroll
                for (int r = 0; r < NR; ++r) acc[r] += dot8(wv[u][r], av);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    // lane r writes output n0 + r (after the xor reduction every lane holds every sum)
    if (lane < kRpw && n0 + lane < N) {
        float yv = 0.f, uv = 0.f;
#pragma unroll
        for (int r = 0; r < kRpw; ++r)
            if (r == lane) {
                yv = acc[r];
                if (MODE == kSwiglu) uv = acc[kRpw + r];
            }
        const int n = n0 + lane;
        const __half y16 = __float2half(yv);
        if (MODE == kStoreF32) {
            static_cast<float*>(out_)[n] = yv;
        } else if (MODE == kStore) {
            out[n] = y16;
        } else if (MODE == kResidual) {
            out[n] = __float2half(__half2float(out[n]) + __half2float(y16));
        } else {
            const float g = __half2float(y16), up = __half2float(__float2half(uv));
            out[n] = __float2half(g / (1.0f + expf(-g)) * up);
        }
    }
    }
}

template <int MODE, bool NORM>
static int launch(const GemvArgs* d, cudaStream_t st) {
    const int rows_per_cta = kWarps * kRpw;
    const size_t smem = (size_t)d->K * 2;
    if (smem > 48 * 1024) {
        static cudaError_t e = cudaFuncSetAttribute(gemv_kernel<MODE, NORM>,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return set_cuda_status(e);
    }
    // one wave of resident CTAs, each paying the prologue once
    int dev = 0, occ = 0;
    cudaGetDevice(&dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_kernel<MODE, NORM>, kThreads, smem) != cudaSuccess ||
        occ < 1) {
        cudaGetLastError();
        occ = 1;
    }
    int grid = (d->N + rows_per_cta - 1) / rows_per_cta;
    const int wave = device_sm_count(dev) * occ;
    if (wave > 0 && grid > wave) grid = wave;
    gemv_kernel<MODE, NORM><<<grid, kThreads, smem, st>>>(
        static_cast<const __half*>(d->W), static_cast<const __half*>(d->W2), d->ld_w, d->N, d->K,
        static_cast<const __half*>(d->x), static_cast<const __half*>(d->rms_w), d->eps, d->out);
    count_launch();
    return set_cuda_status(cudaGetLastError());
}

}  // namespace gv

int gemv(const GemvArgs* d, cudaStream_t stream) {
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!d || !d->W || !d->x || !d->out) return set_status(FCCI_EINVAL, "fcci_gemv_fused: NULL argument");
    if (d->N <= 0 || d->K <= 0 || (d->K & 7) || d->ld_w < d->K || (d->ld_w & 7))
        return set_status(FCCI_EINVAL, "fcci_gemv_fused: K and ld_w must be positive multiples of 8, ld_w >= K");
    if ((int64_t)d->K * 2 > 227 * 1024) return set_status(FCCI_EUNSUPPORTED, "fcci_gemv_fused: K too large");
    if (!a16(d->W) || !a16(d->x) || (d->rms_w && !a16(d->rms_w)) || (d->W2 && !a16(d->W2)))
        return set_status(FCCI_EINVAL, "fcci_gemv_fused: W, W2, x and rms_w must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(d->out) & (d->mode == gv::kStoreF32 ? 3 : 1)))
        return set_status(FCCI_EINVAL, "fcci_gemv_fused: out misaligned");
    if (d->W2 && d->mode != gv::kSwiglu) return set_status(FCCI_EINVAL, "fcci_gemv_fused: W2 is for the SwiGLU mode");
    const bool norm = d->rms_w != nullptr;
    switch (d->mode * 2 + (norm ? 1 : 0)) {
        case 0: return gv::launch<gv::kStore, false>(d, stream);
        case 1: return gv::launch<gv::kStore, true>(d, stream);
        case 2: return gv::launch<gv::kResidual, false>(d, stream);
        case 3: return gv::launch<gv::kResidual, true>(d, stream);
        case 4: return gv::launch<gv::kSwiglu, false>(d, stream);
        case 5: return gv::launch<gv::kSwiglu, true>(d, stream);
        case 6: return gv::launch<gv::kStoreF32, false>(d, stream);
        case 7: return gv::launch<gv::kStoreF32, true>(d, stream);
        default: return set_status(FCCI_EINVAL, "fcci_gemv_fused: mode must be 0, 1, 2 or 3");
    }
}

}  // namespace fcci

extern "C" int fcci_gemv_fused(const fcci_gemv_desc* d, cudaStream_t stream) {
    if (!d) return fcci::set_status(FCCI_EINVAL, "fcci_gemv_fused: NULL argument");
    if (d->mode < 0 || d->mode > 2) return fcci::set_status(FCCI_EINVAL, "fcci_gemv_fused: mode must be 0, 1 or 2");
    fcci::GemvArgs a;
    a.W = d->W;
    a.W2 = nullptr;
    a.ld_w = d->ld_w;
    a.N = d->N;
    a.K = d->K;
    a.x = d->x;
    a.rms_w = d->rms_w;
    a.eps = d->eps;
    a.out = d->out;
    a.mode = d->mode;
    return fcci::gemv(&a, stream);
}
