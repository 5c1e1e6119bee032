// CUDA IPC buffers and the bounded flag wait of the ctx exchange (fcci_exchange.h).
// The stores and the flag raise themselves are part of the decode kernel
// (decode_attn.cu): its CTAs store the ctx slice to every peer's buffer, fence at
// system scope, and the last CTA raises this GPU's slot of every flag array.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "fcci_decode.h"
#include "fcci_exchange.h"
#include "fcci_internal.h"
#include "ptx.cuh"

namespace fcci {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread i < n waits until flags[i] has reached the epoch (wrap-safe comparison),
// giving up after limit_ns with the timeout bit set in *err. Launched as a
// programmatic dependent of the decode launch before it: it is resident before that
// launch ends and reads the epoch only after it (griddepcontrol.wait); the next
// launch may set up in its turn while this one waits (its reads of the exchanged
// ctx come after its own griddepcontrol.wait, i.e. after this kernel).
__global__ void exchange_wait_kernel(const uint32_t* flags, int n, const uint32_t* epoch, uint32_t* err,
                                     uint64_t limit_ns) {
    griddep_launch_dependents();
    griddep_wait();
    const uint32_t e = *epoch;
    if ((int)threadIdx.x < n) {
        const uint64_t t0 = global_timer_ns();
        while ((int32_t)(ld_acquire_sys(flags + threadIdx.x) - e) < 0) {
            if (global_timer_ns() - t0 > limit_ns) {
                atomicOr(err, FCCI_DEV_ERR_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
}

}  // namespace fcci

extern "C" {

int fcci_ipc_alloc(size_t bytes, void** dev_ptr, void* handle_out) {
    if (!dev_ptr || !handle_out || bytes == 0) return fcci::set_status(FCCI_EINVAL, "fcci_ipc_alloc: bad argument");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return fcci::set_cuda_status(e);
    }
    static_assert(sizeof(h) <= FCCI_IPC_HANDLE_BYTES, "IPC handle size");
    memset(handle_out, 0, FCCI_IPC_HANDLE_BYTES);
    memcpy(handle_out, &h, sizeof(h));
    *dev_ptr = p;
    return fcci::set_status(FCCI_OK, nullptr);
}

int fcci_ipc_open(const void* handle, void** dev_ptr) {
    if (!handle || !dev_ptr) return fcci::set_status(FCCI_EINVAL, "fcci_ipc_open: bad argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return fcci::set_cuda_status(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int fcci_ipc_close(void* dev_ptr) {
    if (!dev_ptr) return fcci::set_status(FCCI_EINVAL, "fcci_ipc_close: NULL");
    return fcci::set_cuda_status(cudaIpcCloseMemHandle(dev_ptr));
}

int fcci_ipc_free(void* dev_ptr) {
    if (!dev_ptr) return fcci::set_status(FCCI_EINVAL, "fcci_ipc_free: NULL");
    return fcci::set_cuda_status(cudaFree(dev_ptr));
}

int fcci_exchange_wait(const uint32_t* flags, int n, const uint32_t* epoch, uint32_t* err, uint64_t limit_ns,
                       cudaStream_t stream) {
    if (!flags || !epoch || !err || n < 1 || n > FCCI_MAX_PEERS + 1)
        return fcci::set_status(FCCI_EINVAL, "fcci_exchange_wait: bad argument");
    if (limit_ns == 0 || limit_ns > 10000000000ull)
        return fcci::set_status(FCCI_EINVAL, "fcci_exchange_wait: limit must be in (0, 10 s]");
    return fcci::launch_pdl(fcci::exchange_wait_kernel, dim3(1), dim3(32), 0, stream, flags, n, epoch, err,
                            limit_ns);
}

int fcci_decode_attention_exchange(const fcci_decode_desc* desc, const fcci_ctx_exchange* ex, cudaStream_t stream) {
    if (!ex) return fcci::set_status(FCCI_EINVAL, "fcci_decode_attention_exchange: exchange is NULL");
    if (ex->n_peers < 1 || ex->n_peers > FCCI_MAX_PEERS || ex->rank < 0 || ex->rank > ex->n_peers)
        return fcci::set_status(FCCI_EINVAL, "fcci_decode_attention_exchange: n_peers in 1..7, rank in 0..n_peers");
    if (!ex->flags || !ex->epoch) return fcci::set_status(FCCI_EINVAL, "fcci_decode_attention_exchange: flags/epoch");
    for (int i = 0; i < ex->n_peers; ++i)
        if (!ex->peer_out[i] || !ex->peer_flags[i] || (reinterpret_cast<uintptr_t>(ex->peer_out[i]) & 3))
            return fcci::set_status(FCCI_EINVAL,
                                    "fcci_decode_attention_exchange: peer buffers must be non-NULL, 4-byte aligned");
    return fcci::decode_attention(desc, stream, ex);
}

}  // extern "C"
