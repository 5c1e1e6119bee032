/*
 * fcci_prefill.h — C ABI of the B200 (sm_100a) causal varlen prefill path.
 *
 * One call processes a batch of prompts (or prompt chunks) for one layer:
 *   RoPE on q and k_new at positions T_b + i, append of (k_rot, v_new) into the
 *   same persistent KV arena the decode path reads, and causal attention of the
 *   new tokens over all T_b + n_b keys of their sequence. It replaces, in the
 *   reference (divakar-yadav/Fully_Custom_Cuda_Inference_Lamma2):
 *
 *   case4_graph_generator_server_ipc.py:1241-1262   kv_init: the HF model forward
 *        (LlamaAttention: rotate-half RoPE, causal softmax(q k^T * scale) v) and the
 *        copy of each layer's past_key_values into arena_k / arena_v[l, 0, :, :T, :],
 *        followed by seq_len_dev = T.
 *
 * Entry points:
 *   fcci_prefill_attention        the whole step (two or three kernel launches on
 *                                 `stream`: RoPE table check, RoPE + append + work
 *                                 list, tcgen05 attention)
 *   fcci_prefill_prepare / fcci_prefill_attend   its two halves
 *   fcci_prefill_workspace_bytes  size of the caller-owned workspace
 *   fcci_prefill_workspace_init   zero a fresh workspace (stream-ordered)
 *
 * Status codes, the device error word and fcci_last_status / fcci_last_error_string
 * are those of fcci_decode.h. The device error word of a prefill workspace is
 * read with fcci_prefill_read_error.
 */
#ifndef FCCI_PREFILL_H
#define FCCI_PREFILL_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#include "fcci_decode.h"

#ifdef __cplusplus
extern "C" {
#endif

#define FCCI_PREFILL_ABI_VERSION 1

/*
 * Shapes and layouts (fp16 unless stated; strides in elements; head_dim contiguous):
 *   new tokens        sequence b owns rows cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1 of
 *                     q [total_q, Hq, D], k_new / v_new [total_q, Hkv, D] and
 *                     out [total_q, Hq, D]; n_b = cu_seqlens_q[b+1] - cu_seqlens_q[b]
 *                     must not exceed max_seqlen_q
 *   arena             k_cache / v_cache with the decode descriptor's two layouts:
 *                     batched (cu_seqlens_kv == NULL): row (b, h, t) at
 *                       cache + b*stride_b + h*stride_h + t*stride_t, t < capacity;
 *                     packed: cache + h*stride_h + (cu_seqlens_kv[b] + t)*stride_t,
 *                       t < cu_seqlens_kv[b+1] - cu_seqlens_kv[b]
 *   T_b               seq_lens ? seq_lens[b] : fixed_len (device int32): tokens already
 *                     cached; 0 for a fresh prompt, > 0 for a later chunk
 *   RoPE              rotate-half on the first rotary_dim dims at position T_b + i
 *                     (inv_freq_i = rope_theta^(-i/(rotary_dim/2)), fp32, rounded to
 *                     fp16), rotary_dim a multiple of 16 (0 disables it)
 *   append            arena row T_b + i of sequence b := (k_rot, v_new) of new token i
 *   attention         out[row i of b, hq] = softmax_t(q_rot . k[b, hq/G, t] * scale) v,
 *                     over keys t <= T_b + i (causal), fp32 accumulation
 *   advance           when non-zero, seq_lens[b] += n_b after the step
 * head_dim D must be 128; Hq a multiple of Hkv.
 */
typedef struct fcci_prefill_desc {
    int32_t abi_version; /* FCCI_PREFILL_ABI_VERSION */
    int32_t B, Hq, Hkv, D;
    int32_t total_q;      /* rows of q / k_new / v_new / out (= cu_seqlens_q[B]) */
    int32_t max_seqlen_q; /* bound on n_b, used to size the work list */
    const int32_t* cu_seqlens_q;
    const void* q;
    int64_t q_stride_t, q_stride_h;
    const void* k_new;
    int64_t k_new_stride_t, k_new_stride_h;
    const void* v_new;
    int64_t v_new_stride_t, v_new_stride_h;
    void* k_cache;
    int64_t k_stride_b, k_stride_h, k_stride_t;
    void* v_cache;
    int64_t v_stride_b, v_stride_h, v_stride_t;
    int32_t capacity;
    const int32_t* cu_seqlens_kv;
    int32_t* seq_lens;
    int32_t fixed_len;
    void* out;
    int64_t out_stride_t, out_stride_h;
    float scale;
    float rope_theta;
    int32_t rotary_dim;
    int32_t advance;
    void* workspace;
    size_t workspace_bytes;
} fcci_prefill_desc;

int fcci_prefill_attention(const fcci_prefill_desc* desc, cudaStream_t stream);

/* The two halves of fcci_prefill_attention, for callers that schedule them
 * separately (same descriptor and workspace, prepare first, on one stream or with
 * the caller's own ordering): prepare = RoPE table check + RoPE/append of the new
 * tokens + work list; attend = the causal attention kernel. */
int fcci_prefill_prepare(const fcci_prefill_desc* desc, cudaStream_t stream);
int fcci_prefill_attend(const fcci_prefill_desc* desc, cudaStream_t stream);

/* Workspace bytes: rotated queries (total_q x Hq x D fp16), the RoPE cos/sin
 * table (capacity x rotary_dim/2 float2, rebuilt on device only when theta,
 * rotary_dim or capacity change), the work list and counters. */
size_t fcci_prefill_workspace_bytes(int32_t B, int32_t Hq, int32_t Hkv, int32_t D, int32_t total_q,
                                    int32_t max_seqlen_q, int32_t capacity, int32_t rotary_dim);
int fcci_prefill_workspace_init(void* workspace, size_t bytes, cudaStream_t stream);
int fcci_prefill_read_error(void* workspace, uint32_t* flags, int clear, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FCCI_PREFILL_H */
