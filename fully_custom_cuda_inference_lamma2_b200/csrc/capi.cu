// extern "C" surface of libfcci_decode.so: the reference's two launcher symbols
// (attn_varlen_host, capture_decode_host) and the new descriptor-based entry points.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "fcci_decode.h"
#include "fcci_internal.h"
#include "ptx.cuh"

namespace fcci {

static thread_local int t_status = FCCI_OK;
static thread_local char t_msg[256] = "";
static std::atomic<uint64_t> g_launches{0};

int set_status(int code, const char* msg) {
    t_status = code;
    if (code == FCCI_OK) t_msg[0] = '\0';
    else snprintf(t_msg, sizeof(t_msg), "%s", msg ? msg : "error");
    return code;
}

int set_cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return set_status(FCCI_OK, nullptr);
    t_status = FCCI_ECUDA;
    snprintf(t_msg, sizeof(t_msg), "CUDA error: %s", cudaGetErrorString(e));
    return FCCI_ECUDA;
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Placeholder decode step of capture_decode_step_kernel.cu:58-92, race-free on
// any grid: zero arena rows at T for every (layer, head), one-hot logits.
__global__ void placeholder_step_kernel(const int64_t* __restrict__ ctrl, __half* __restrict__ ak,
                                        __half* __restrict__ av, const int32_t* __restrict__ seq_len,
                                        float* __restrict__ logits, int L, int H, int max_len, int D, int vocab) {
    const int T = seq_len[0];
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (T >= 0 && T < max_len) {
        const int64_t n = (int64_t)L * H * D;
        for (int64_t i = i0; i < n; i += stride) {
            const int64_t row = i / D;  // l * H + h
            const int64_t d = i - row * D;
            const int64_t off = (row * max_len + T) * D + d;
            ak[off] = __float2half(0.0f);
            av[off] = __float2half(0.0f);
        }
    }
    const int64_t hot = ctrl[0] % (int64_t)vocab;  // C remainder, as the reference
    for (int64_t i = i0; i < vocab; i += stride) logits[i] = (i == hot) ? 1.0f : 0.0f;
}

__global__ void bump_seq_len_kernel(int32_t* seq_len) {
    if (threadIdx.x == 0 && blockIdx.x == 0) seq_len[0] += 1;
}

int launch_placeholder(const int64_t* ctrl, void* ak, void* av, int32_t* seq_len, float* logits, int L, int H,
                       int max_len, int D, int vocab, cudaStream_t stream) {
    if (!ctrl || !ak || !av || !seq_len || !logits || L < 0 || H < 0 || max_len < 0 || D < 0 || vocab <= 0)
        return set_status(FCCI_EINVAL, "capture_decode_host: invalid argument");
    const int64_t work = (int64_t)L * H * D > vocab ? (int64_t)L * H * D : vocab;
    int blocks = (int)((work + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    placeholder_step_kernel<<<blocks, 256, 0, stream>>>(ctrl, static_cast<__half*>(ak), static_cast<__half*>(av),
                                                         seq_len, logits, L, H, max_len, D, vocab);
    count_launch();
    bump_seq_len_kernel<<<1, 32, 0, stream>>>(seq_len);
    count_launch();
    return set_cuda_status(cudaGetLastError());
}

}  // namespace fcci

extern "C" {

int fcci_decode_attention(const fcci_decode_desc* desc, cudaStream_t stream) {
    return fcci::decode_attention(desc, stream);
}

int fcci_rope_append(const fcci_decode_desc* desc, cudaStream_t stream) { return fcci::rope_append(desc, stream); }

size_t fcci_decode_workspace_bytes(int32_t B, int32_t Hq, int32_t Hkv, int32_t D, int device) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || D <= 0) return 0;
    const int grid = fcci::max_grid(device);
    if (grid <= 0) return 0;
    return fcci::workspace_layout(B, Hq, Hkv, D, grid).total;
}

int fcci_decode_workspace_init(void* workspace, size_t bytes, cudaStream_t stream) {
    if (!workspace || bytes == 0) return fcci::set_status(FCCI_EINVAL, "fcci_decode_workspace_init: no workspace");
    return fcci::set_cuda_status(cudaMemsetAsync(workspace, 0, bytes, stream));
}

int fcci_decode_read_error(void* workspace, uint32_t* flags, int clear, cudaStream_t stream) {
    if (!workspace || !flags) return fcci::set_status(FCCI_EINVAL, "fcci_decode_read_error: null argument");
    cudaError_t e = cudaMemcpyAsync(flags, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(workspace, 0, sizeof(uint32_t), stream);
    return fcci::set_cuda_status(e);
}

int fcci_decode_set_tuning(int stages, int ctas_per_sm) {
    if (stages < 0 || stages > 8 || ctas_per_sm < 0 || ctas_per_sm > fcci::kMaxCtasPerSm)
        return fcci::set_status(FCCI_EINVAL, "fcci_decode_set_tuning: out of range");
    fcci::tuning().stages = stages;
    fcci::tuning().ctas_per_sm = ctas_per_sm;
    return fcci::set_status(FCCI_OK, nullptr);
}

int fcci_decode_set_cluster_tuning(int max_cluster, int solo_tiles, int min_tiles) {
    if (max_cluster < 0 || max_cluster > 16 || solo_tiles < -1 || min_tiles < 0)
        return fcci::set_status(FCCI_EINVAL, "fcci_decode_set_cluster_tuning: out of range");
    fcci::tuning().max_cluster = max_cluster;
    fcci::tuning().solo_tiles = solo_tiles;
    fcci::tuning().cluster_min_tiles = min_tiles;
    return fcci::set_status(FCCI_OK, nullptr);
}

int fcci_last_status(void) { return fcci::t_status; }

const char* fcci_last_error_string(void) { return fcci::t_msg; }

uint64_t fcci_launch_count(void) { return fcci::g_launches.load(std::memory_order_relaxed); }

void attn_varlen_host(const __half* q, const __half* k, const __half* v, int32_t H, int32_t T, int32_t D, float scale,
                      __half* ctx_out, cudaStream_t stream) {
    if (!q || !k || !v || !ctx_out || H <= 0 || T <= 0 || D <= 0) {
        fcci::set_status(FCCI_EINVAL, "attn_varlen_host: invalid argument");
        return;
    }
    fcci_decode_desc d;
    memset(&d, 0, sizeof(d));
    d.abi_version = FCCI_DECODE_ABI_VERSION;
    d.B = 1;
    d.Hq = H;
    d.Hkv = H;
    d.D = D;
    d.q = q;
    d.q_stride_b = (int64_t)H * D;
    d.q_stride_h = D;
    d.k_cache = const_cast<__half*>(k);
    d.k_stride_b = (int64_t)H * T * D;
    d.k_stride_h = (int64_t)T * D;
    d.k_stride_t = D;
    d.v_cache = const_cast<__half*>(v);
    d.v_stride_b = (int64_t)H * T * D;
    d.v_stride_h = (int64_t)T * D;
    d.v_stride_t = D;
    d.capacity = T;
    d.fixed_len = T;
    d.out = ctx_out;
    d.out_stride_b = (int64_t)H * D;
    d.out_stride_h = D;
    d.scale = scale;
    d.rotary_dim = 0;
    d.split = 0;
    fcci::decode_attention(&d, stream);
}

void capture_decode_host(const int64_t* ctrl_input, void* arena_k, void* arena_v, int32_t* seq_len_ptr,
                         const int32_t* position_ptr, float* logits_out, int32_t L, int32_t H, int32_t max_len,
                         int32_t D, int32_t vocab, cudaStream_t stream) {
    (void)position_ptr;
    fcci::launch_placeholder(ctrl_input, arena_k, arena_v, seq_len_ptr, logits_out, L, H, max_len, D, vocab, stream);
}

}  // extern "C"

// Self-test of the bounded wait every pipeline wait of the kernels goes through:
// one CTA waits on an mbarrier that nothing arrives on. The wait must give up after
// the limit and report it, the kernel must return, and the context stays usable.
namespace fcci {
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns, uint32_t* out) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const uint64_t t0 = global_timer_ns();
    const bool ok = mbar_wait_bounded(&bar, 0, &abort_flag, limit_ns);  // no arrival ever comes
    const uint64_t t1 = global_timer_ns();
    if (threadIdx.x == 0) {
        out[0] = ok ? 0u : FCCI_DEV_ERR_TIMEOUT;
        out[1] = (uint32_t)((t1 - t0) / 1000000ull);  // milliseconds waited
    }
}
}  // namespace fcci

extern "C" int fcci_selftest_bounded_wait(uint64_t limit_ns, uint32_t* result, cudaStream_t stream) {
    if (!result) return fcci::set_status(FCCI_EINVAL, "fcci_selftest_bounded_wait: result is NULL");
    if (limit_ns == 0 || limit_ns > 1000000000ull)
        return fcci::set_status(FCCI_EINVAL, "fcci_selftest_bounded_wait: limit must be in (0, 1 s]");
    uint32_t* d = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&d), 2 * sizeof(uint32_t), stream);
    if (e != cudaSuccess) return fcci::set_cuda_status(e);
    fcci::bounded_wait_probe_kernel<<<1, 32, 0, stream>>>(limit_ns, d);
    fcci::count_launch();
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(result, d, 2 * sizeof(uint32_t), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    cudaFreeAsync(d, stream);
    return fcci::set_cuda_status(e);
}
