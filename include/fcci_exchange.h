/*
 * fcci_exchange.h — the ctx exchange of the kv-head partition across the GPUs of one
 * node, fused into the decode-attention launch (no reference counterpart: the
 * reference runs on one GPU, case4_graph_generator_server_ipc.py:155).
 *
 * With the kv heads sharded over N GPUs, GPU r computes ctx[:, heads of r, :] and an
 * unsharded output projection needs ctx[:, all heads, :] on every GPU. Instead of an
 * all-gather after the attention, the decode launch stores its slice straight into
 * every GPU's full-ctx buffer (plain stores to CUDA IPC mappings of the peers' memory,
 * over NVLink), and its last CTA then raises this GPU's slot of every GPU's flag array
 * to a per-call epoch (release, system scope). fcci_exchange_wait holds a stream until
 * every slot of the local flag array has reached the local epoch (acquire, system
 * scope; bounded: a wait that runs out sets FCCI_DEV_ERR_TIMEOUT and returns).
 *
 * Buffers shared this way come from fcci_ipc_alloc (zeroed cudaMalloc memory and its
 * IPC handle); a peer maps one with fcci_ipc_open. Flag arrays hold N uint32 slots;
 * the epoch is one uint32 in the GPU's own memory. Full-ctx buffers are used in pairs
 * (alternate layers), so that a GPU that has passed layer l's wait can store layer
 * l+1's slice while another still reads layer l's ctx.
 */
#ifndef FCCI_EXCHANGE_H
#define FCCI_EXCHANGE_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#include "fcci_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

#define FCCI_IPC_HANDLE_BYTES 64
#define FCCI_MAX_PEERS 7

/* Where a decode launch sends its ctx slice besides `out`, and how it signals. */
typedef struct fcci_ctx_exchange {
    int32_t n_peers;                        /* other GPUs, 1..FCCI_MAX_PEERS */
    int32_t rank;                           /* this GPU's slot in every flag array, 0..n_peers */
    void* peer_out[FCCI_MAX_PEERS];         /* this GPU's mapping of each peer's full-ctx buffer; the slice
                                               is stored at the same element offsets as in desc->out */
    uint32_t* peer_flags[FCCI_MAX_PEERS];   /* this GPU's mapping of each peer's flag array */
    uint32_t* flags;                        /* this GPU's own flag array (its own slot is raised too) */
    uint32_t* epoch;                        /* this GPU's epoch counter: raised by one per call */
} fcci_ctx_exchange;

/* fcci_decode_attention (same descriptor, workspace required) whose ctx slice also goes
 * to every peer's buffer, followed by the flag raise described above. */
int fcci_decode_attention_exchange(const fcci_decode_desc* desc, const fcci_ctx_exchange* ex, cudaStream_t stream);

/* `bytes` of zeroed device memory on the current device and its IPC handle
 * (FCCI_IPC_HANDLE_BYTES bytes written to handle_out). */
int fcci_ipc_alloc(size_t bytes, void** dev_ptr, void* handle_out);
/* Map a buffer of another process on this node (the current device must be able to
 * reach its GPU over NVLink / PCIe peer access). */
int fcci_ipc_open(const void* handle, void** dev_ptr);
int fcci_ipc_close(void* dev_ptr);
int fcci_ipc_free(void* dev_ptr);

/* Hold `stream` until flags[i] >= *epoch for every i < n (n <= FCCI_MAX_PEERS + 1).
 * One CTA; every wait bounded by limit_ns (0 < limit_ns <= 10 s). On timeout the
 * kernel ORs FCCI_DEV_ERR_TIMEOUT into *err and returns. */
int fcci_exchange_wait(const uint32_t* flags, int n, const uint32_t* epoch, uint32_t* err, uint64_t limit_ns,
                       cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FCCI_EXCHANGE_H */
