// fcci_decode_attention_noalloc: the decode-attention step with its scratch in a
// fixed device array that this library owns, for callers that cannot allocate
// device memory themselves.
//
// Who needs it: a caller embedded in a host runtime that owns every byte of
// device memory (a serving framework with its own memory pool, or a plugin
// whose allocator is not reachable from its language's FFI) may not call
// cudaMalloc at all, and a caller on a latency-critical path may not afford
// one (cudaMalloc/cudaFree can synchronize the device). Such a caller still
// passes its own inputs and outputs; only the split-KV scratch (partial
// results, merge counters, error word) comes from here.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "fcci_decode.h"
#include "fcci_internal.h"

namespace fcci {

// Split-KV scratch of the allocation-free entry point. Every GPU that loads this
// library holds these FCCI_NOALLOC_SCRATCH_BYTES until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FCCI_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on device `dev` (the current device). In
// host code the array's name is only a stand-in for the symbol, so the address
// is looked up once per device with cudaGetSymbolAddress. A failed look-up is
// not remembered: a later call (for example one made outside stream capture)
// tries again. The look-up is refused while `stream` is capturing, because the
// first use of the symbol on a device may have to load the module there.
static int noalloc_scratch(int dev, cudaStream_t stream, void** out) {
    static std::mutex mu;
    static void* addr[128];
    if (dev < 0 || dev >= 128) return set_status(FCCI_EINVAL, "fcci_decode_attention_noalloc: device index");
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        cudaError_t e = cudaStreamIsCapturing(stream, &cap);
        if (e != cudaSuccess) return set_cuda_status(e);
        if (cap != cudaStreamCaptureStatusNone)
            return set_status(FCCI_EINVAL,
                              "fcci_decode_attention_noalloc: the first call on a device must come before any stream "
                              "capture (it looks up the built-in scratch's device address)");
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_cuda_status(e);
        }
        addr[dev] = p;
    }
    *out = addr[dev];
    return FCCI_OK;
}

}  // namespace fcci

extern "C" int fcci_decode_attention_noalloc(const fcci_decode_desc* desc, cudaStream_t stream) {
    if (!desc) return fcci::set_status(FCCI_EINVAL, "fcci_decode_attention_noalloc: descriptor is NULL");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fcci::set_cuda_status(e);
    const size_t need = fcci_decode_workspace_bytes(desc->B, desc->Hq, desc->Hkv, desc->D, dev);
    if (need == 0) return fcci::set_status(FCCI_EINVAL, "fcci_decode_attention_noalloc: invalid shape");
    if (need > FCCI_NOALLOC_SCRATCH_BYTES) {
        static thread_local char msg[200];
        snprintf(msg, sizeof(msg),
                 "fcci_decode_attention_noalloc: this shape needs %zu bytes of scratch; the built-in scratch holds %u "
                 "bytes (use fcci_decode_attention with a caller workspace)",
                 need, (unsigned)FCCI_NOALLOC_SCRATCH_BYTES);
        return fcci::set_status(FCCI_EWORKSPACE, msg);
    }
    void* scratch = nullptr;
    int rc = fcci::noalloc_scratch(dev, stream, &scratch);
    if (rc) return rc;
    // the array keeps the previous call's contents: the counters and the error
    // word must start at zero
    const fcci::WorkspaceLayout L =
        fcci::workspace_layout(desc->B, desc->Hq, desc->Hkv, desc->D, fcci::max_grid(dev));
    e = cudaMemsetAsync(scratch, 0, L.zero_bytes, stream);
    if (e != cudaSuccess) return fcci::set_cuda_status(e);
    // a version-1 descriptor ends before `flags`: copy only what the caller has
    fcci_decode_desc d;
    memset(&d, 0, sizeof(d));
    memcpy(&d, desc, desc->abi_version >= 2 ? sizeof(d) : offsetof(fcci_decode_desc, flags));
    d.workspace = scratch;
    d.workspace_bytes = FCCI_NOALLOC_SCRATCH_BYTES;
    return fcci_decode_attention(&d, stream);
}

extern "C" int fcci_decode_noalloc_read_error(uint32_t* flags, int clear, cudaStream_t stream) {
    if (!flags) return fcci::set_status(FCCI_EINVAL, "fcci_decode_noalloc_read_error: flags is NULL");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fcci::set_cuda_status(e);
    void* scratch = nullptr;
    int rc = fcci::noalloc_scratch(dev, stream, &scratch);
    if (rc) return rc;
    return fcci_decode_read_error(scratch, flags, clear, stream);
}
