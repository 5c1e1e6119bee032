// Helpers shared by the two pybind modules: tensor checks, descriptor filling
// and workspace handling on top of the C ABI in fcci_decode.h.
#pragma once
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <cmath>
#include <map>
#include <mutex>
#include <tuple>

#include "fcci_decode.h"

namespace fcci_py {

inline void check_rc(int rc, const char* where) {
    TORCH_CHECK(rc == FCCI_OK, where, " failed (fcci status ", rc, "): ", fcci_last_error_string());
}

inline cudaStream_t current_stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

inline void check_half_cuda(const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.scalar_type() == at::kHalf, name, " must be fp16");
}

inline void check_int32_cuda(const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.scalar_type() == at::kInt, name, " must be int32");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

// A K/V view the TMA descriptor can describe: head_dim contiguous, the other
// strides multiples of 8 elements (16 bytes), base 16-byte aligned.
inline bool tma_compatible(const at::Tensor& t) {
    if (t.stride(-1) != 1) return false;
    if ((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) != 0) return false;
    for (int64_t i = 0; i + 1 < t.dim(); ++i)
        if (t.size(i) > 1 && (t.stride(i) % 8 != 0 || t.stride(i) <= 0)) return false;
    return true;
}

// Returns t itself when usable, else a fresh aligned contiguous copy.
inline at::Tensor tma_ready(const at::Tensor& t) {
    if (tma_compatible(t)) return t;
    at::Tensor c = t.contiguous();
    if (!tma_compatible(c)) c = t.clone(at::MemoryFormat::Contiguous);
    return c;
}

inline fcci_decode_desc blank_desc() {
    fcci_decode_desc d;
    std::memset(&d, 0, sizeof(d));
    d.abi_version = FCCI_DECODE_ABI_VERSION;
    d.rope_theta = 10000.0f;
    return d;
}

inline at::Tensor make_workspace(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, const at::Device& dev) {
    const size_t bytes = fcci_decode_workspace_bytes((int32_t)B, (int32_t)Hq, (int32_t)Hkv, (int32_t)D, dev.index());
    TORCH_CHECK(bytes > 0, "fcci_decode_workspace_bytes: invalid shape");
    at::Tensor ws = at::empty({(int64_t)bytes}, at::TensorOptions().dtype(at::kByte).device(dev));
    check_rc(fcci_decode_workspace_init(ws.data_ptr(), bytes, current_stream()), "fcci_decode_workspace_init");
    return ws;
}

// Workspace for calls that were not given one (the reference-shaped `forward` and
// `capture_decode(..., q=...)`): one zeroed buffer per (device, stream, shape), made
// on first use and kept for the process, so that repeated calls neither allocate nor
// launch a memset. Calls on one stream run in order, which is what sharing a
// workspace needs; calls on another stream get their own. While the stream is being
// captured a fresh workspace is made instead (from the graph's memory pool, zeroed
// inside the graph), as a per-call allocation was before. The counters in a
// workspace return to zero after every call; a call that timed out on the device
// (FCCI_DEV_ERR_TIMEOUT) may leave them mid-count, and clear_workspace_cache() then
// drops every cached buffer so that the next calls start from fresh zeroed ones.
struct WorkspaceKey {
    int dev;
    uintptr_t stream;
    int64_t B, Hq, Hkv, D;
    bool operator<(const WorkspaceKey& o) const {
        return std::tie(dev, stream, B, Hq, Hkv, D) < std::tie(o.dev, o.stream, o.B, o.Hq, o.Hkv, o.D);
    }
};

inline std::mutex& workspace_cache_mutex() {
    static std::mutex mu;
    return mu;
}

inline std::map<WorkspaceKey, at::Tensor>& workspace_cache() {
    static auto* cache = new std::map<WorkspaceKey, at::Tensor>();  // lives until exit
    return *cache;
}

inline void clear_workspace_cache() {
    std::lock_guard<std::mutex> lk(workspace_cache_mutex());
    workspace_cache().clear();
}

inline at::Tensor cached_workspace(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, const at::Device& dev) {
    const cudaStream_t s = current_stream();
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    TORCH_CHECK(cudaStreamIsCapturing(s, &cap) == cudaSuccess, "cudaStreamIsCapturing failed");
    if (cap != cudaStreamCaptureStatusNone) return make_workspace(B, Hq, Hkv, D, dev);
    const WorkspaceKey key{(int)dev.index(), reinterpret_cast<uintptr_t>(s), B, Hq, Hkv, D};
    std::lock_guard<std::mutex> lk(workspace_cache_mutex());
    auto& cache = workspace_cache();
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    at::Tensor ws = make_workspace(B, Hq, Hkv, D, dev);
    if (cache.size() < 64) cache.emplace(key, ws);  // beyond 64 shapes: a workspace per call
    return ws;
}

inline void bind_workspace(fcci_decode_desc& d, const at::Tensor& ws) {
    TORCH_CHECK(ws.is_cuda() && ws.scalar_type() == at::kByte && ws.is_contiguous(),
                "workspace must be a contiguous uint8 CUDA tensor from make_workspace()");
    d.workspace = ws.data_ptr();
    d.workspace_bytes = (size_t)ws.numel();
}

// Query-like operand [n, H, D] or anything with numel n*H*D viewed as such; must be contiguous.
inline void check_rows(const at::Tensor& t, int64_t numel, const char* name) {
    check_half_cuda(t, name);
    TORCH_CHECK(t.numel() == numel, name, " has ", t.numel(), " elements, expected ", numel);
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

}  // namespace fcci_py
