/*
 * fcci_decode.h — C ABI of the B200 (sm_100a) varlen decode-attention path.
 *
 * The library (libfcci_decode.so) exports plain `extern "C"` entry points that take
 * raw device pointers, sizes and element strides. Nothing here depends on torch;
 * the pybind modules `attn_varlen` and `capture_decode_step` (same names as the
 * reference's extensions) are thin wrappers over these symbols.
 *
 * Entry points and the reference interface each one replaces (paths are inside
 * divakar-yadav/Fully_Custom_Cuda_Inference_Lamma2):
 *
 *   attn_varlen_host            custom_kernels/attn_varlen_kernel.cu:88-99
 *                               (same symbol, same argument list, same meaning;
 *                               launched on `stream`)
 *   capture_decode_host         custom_kernels/capture_decode_step_kernel.cu:101-121
 *                               (same symbol and arguments; placeholder step kept
 *                               bit-for-bit: zero K/V row at T, one-hot logits,
 *                               seq_len[0] = T + 1)
 *   fcci_decode_attention       new: the attention step the reference performs in
 *                               torch + attn_varlen inside its decode drivers
 *                               (scripts/direct_custom_decode_500.py:229-250,
 *                               scripts/debug_parity_seq8.py:182-195): RoPE on
 *                               q/k at position T, append of k/v at T into the
 *                               persistent arena, GQA split-KV attention over
 *                               T+1 keys, device-side seq_len advance. Batched,
 *                               varlen (cu_seqlens) and strided.
 *   fcci_rope_append            new: only the RoPE + append half of the above
 *                               (driver lines :233-240), for callers that run
 *                               attention elsewhere.
 *   fcci_decode_workspace_bytes / fcci_decode_workspace_init / fcci_decode_read_error
 *                               new: sizing, zeroing and error readback of the
 *                               caller-owned workspace (split-KV partials,
 *                               last-arriver counters, device error word).
 *
 * Data types: every tensor argument is IEEE fp16 unless stated. Element strides
 * are in units of elements (not bytes). The innermost dimension (head_dim) must be
 * contiguous.
 *
 * Error behaviour: functions returning int return FCCI_OK (0) or a positive
 * FCCI_E* code and never abort the process; a launch error is reported as
 * FCCI_ECUDA with the CUDA error string available from fcci_last_error_string().
 * attn_varlen_host and capture_decode_host return void like the reference; their
 * status is available from fcci_last_status(). Runtime range problems that only
 * the device can see (seq_len beyond the arena capacity) are recorded in the
 * workspace's device error word and read with fcci_decode_read_error(); the
 * kernels never trap.
 */
#ifndef FCCI_DECODE_H
#define FCCI_DECODE_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 2 adds the trailing `flags` field; descriptors of version 1 (no flags) are still accepted */
#define FCCI_DECODE_ABI_VERSION 2

/* status codes */
#define FCCI_OK 0
#define FCCI_EINVAL 1       /* bad pointer, size, stride or alignment */
#define FCCI_EUNSUPPORTED 2 /* head_dim / group size outside the compiled set */
#define FCCI_EWORKSPACE 3   /* workspace missing or too small */
#define FCCI_ECUDA 4        /* CUDA runtime error at launch */
#define FCCI_ETMAP 5        /* TMA descriptor could not be encoded */

/* device error word bits (fcci_decode_read_error) */
#define FCCI_DEV_ERR_CAPACITY 1u /* T (+1 when appending) exceeded a sequence's capacity */
#define FCCI_DEV_ERR_TIMEOUT 2u  /* a pipeline wait hit its time limit (kernel bailed out) */
#define FCCI_DEV_ERR_EARLY_READ 4u /* FCCI_DECODE_PREFETCH_KV: a length or sequence offset read before the
                                      programmatic-launch wait had changed by the end of the wait (a kernel
                                      still running wrote it); the step used the stale value */

/*
 * One decode-attention step over B sequences.
 *
 *   query q            [B, Hq, D]          q + b*q_stride_b + hq*q_stride_h + d
 *   new rows k_new/v_new [B, Hkv, D]       nullable together: when set, the step
 *                                          appends them at position T_b
 *   arena k_cache/v_cache                  row (b, h, t) at
 *        batched layout (cu_seqlens == NULL): cache + b*stride_b + h*stride_h + t*stride_t,
 *                                          t < capacity
 *        packed layout  (cu_seqlens != NULL): cache + h*stride_h + (cu_seqlens[b] + t)*stride_t,
 *                                          t < cu_seqlens[b+1]-cu_seqlens[b]; capacity is the
 *                                          total token extent of the packed arena
 *   T_b                = seq_lens ? seq_lens[b] : fixed_len   (device int32, read on device)
 *   keys attended L_b  = T_b + (k_new ? 1 : 0)
 *   RoPE               rotate-half on the first rotary_dim dims of q (and k_new) at
 *                      position T_b, inv_freq_i = rope_theta^(-i/(rotary_dim/2)),
 *                      fp32 math, rounded to fp16 (rotary_dim == 0 disables it)
 *   out                [B, Hq, D]          out + b*out_stride_b + hq*out_stride_h + d
 *                      out[b,hq] = softmax(q_rot[b,hq] . K[b, hq/G]^T * scale) V[b, hq/G]
 *   q_rot_out          nullable, [B, Hq, D] contiguous: the rotated fp16 query
 *   advance            when non-zero, seq_lens[b] += 1 once every CTA has read it
 *   workspace          caller-owned device buffer of fcci_decode_workspace_bytes()
 *                      bytes, zeroed once with fcci_decode_workspace_init(). May be
 *                      NULL only when advance == 0 and split == 0 (one CTA per
 *                      (sequence, kv head) pair, no partials).
 *   split              0: one CTA per (sequence, kv-head) pair; 1: persistent
 *                      stream-K split over all SMs with last-arriver combine, or,
 *                      with few pairs, one thread-block cluster per pair whose CTAs
 *                      merge their pieces through distributed shared memory.
 *   flags              (abi_version >= 2) bit set of FCCI_DECODE_* below.
 *
 * Calls that share a workspace must not overlap on the GPU.
 *
 * FCCI_DECODE_PREFETCH_KV: the kernel is launched as a programmatic dependent of
 * the kernel before it on the stream, and by default reads nothing until that
 * kernel has finished. With this flag it reads seq_lens, cu_seqlens and its first
 * pipeline stages of cached keys and values (rows below T_b) before that wait, so
 * those loads overlap the previous kernel's last CTAs; q, k_new and v_new are
 * still read after it. Set it only when no kernel that can still be running when
 * this one starts writes seq_lens, cu_seqlens or those arena rows: for example a
 * chain of decode steps over different layers' arenas where only the last one
 * advances seq_lens (and the next step starts with a copy or a non-dependent
 * launch), or a decode step right after the projection that produced q/k/v.
 *
 * FCCI_DECODE_CHECK_EARLY_READ (with FCCI_DECODE_PREFETCH_KV): the kernel also reads
 * the lengths and sequence offsets again after the wait and reports any that changed
 * since its early read as FCCI_DEV_ERR_EARLY_READ in the workspace's error word (the
 * step's results are then not to be used). A changed arena row is not detected. It
 * costs about half a microsecond per launch, so it is meant for validating a caller's
 * use of the early reads, not for every step.
 */
#define FCCI_DECODE_PREFETCH_KV 1u
#define FCCI_DECODE_CHECK_EARLY_READ 2u
typedef struct fcci_decode_desc {
    int32_t abi_version; /* FCCI_DECODE_ABI_VERSION */
    int32_t B, Hq, Hkv, D;
    const void* q;
    int64_t q_stride_b, q_stride_h;
    const void* k_new;
    int64_t k_new_stride_b, k_new_stride_h;
    const void* v_new;
    int64_t v_new_stride_b, v_new_stride_h;
    void* k_cache;
    int64_t k_stride_b, k_stride_h, k_stride_t;
    void* v_cache;
    int64_t v_stride_b, v_stride_h, v_stride_t;
    int32_t capacity;
    const int32_t* cu_seqlens;
    int32_t* seq_lens;
    int32_t fixed_len;
    void* out;
    int64_t out_stride_b, out_stride_h;
    void* q_rot_out;
    float scale;
    float rope_theta;
    int32_t rotary_dim;
    int32_t advance;
    int32_t split;
    void* workspace;
    size_t workspace_bytes;
    uint32_t flags; /* abi_version >= 2 */
} fcci_decode_desc;

int fcci_decode_attention(const fcci_decode_desc* desc, cudaStream_t stream);

/*
 * Allocation-free form of fcci_decode_attention. It has no counterpart in the
 * reference. It is for callers that may not call cudaMalloc: code hosted in a
 * runtime that owns all device memory (its own pool, or an allocator its FFI
 * cannot reach), or a latency-critical path that cannot pay for an allocation.
 * The caller still passes inputs and outputs; desc->workspace and
 * workspace_bytes are ignored. The split-KV scratch is a fixed array of
 * FCCI_NOALLOC_SCRATCH_BYTES (8 MiB) inside this library, resident on every GPU
 * that loads it until the process exits. Shapes needing more scratch than that
 * (see fcci_decode_workspace_bytes) are rejected with FCCI_EWORKSPACE and a
 * message. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call before
 * any stream capture: a first call on a capturing stream is refused with
 * FCCI_EINVAL, and a later call outside capture does the look-up. Each call
 * zeroes the array's counters and error word on `stream` first. All calls share
 * the one array: calls that overlap on the GPU (other streams, other threads)
 * race and must be serialised by the caller. Nothing here calls cudaMalloc,
 * cudaFree or an allocating library routine.
 */
#define FCCI_NOALLOC_SCRATCH_BYTES (8u << 20)
int fcci_decode_attention_noalloc(const fcci_decode_desc* desc, cudaStream_t stream);

/* Device error word of the built-in scratch (FCCI_DEV_ERR_* bits of the last
 * fcci_decode_attention_noalloc call on this device), as fcci_decode_read_error
 * reads a caller workspace: synchronises `stream`, clears the word when clear != 0.
 * Read it after a call and before the next one, which zeroes the word again.
 * No counterpart in the reference; allocates nothing. */
int fcci_decode_noalloc_read_error(uint32_t* flags, int clear, cudaStream_t stream);

/* RoPE(q, k_new) at T_b and append of (k_rot, v_new) at T_b; no attention.
 * Same descriptor; out/scale/workspace/split are ignored; q_rot_out receives
 * the rotated query when non-NULL; advance requires no workspace here (the
 * kernel is a single wave that bumps seq_lens after its own reads). */
int fcci_rope_append(const fcci_decode_desc* desc, cudaStream_t stream);

/* Workspace size for B sequences, Hq/Hkv heads and head_dim D on `device`. */
size_t fcci_decode_workspace_bytes(int32_t B, int32_t Hq, int32_t Hkv, int32_t D, int device);
/* Zero the counters and error word of a fresh workspace (stream-ordered). */
int fcci_decode_workspace_init(void* workspace, size_t bytes, cudaStream_t stream);
/* Copy the device error word to *flags (synchronises `stream`); clear it when clear != 0.
 * After FCCI_DEV_ERR_TIMEOUT the workspace's merge counters may be left mid-count:
 * run fcci_decode_workspace_init on it before its next use. */
int fcci_decode_read_error(void* workspace, uint32_t* flags, int clear, cudaStream_t stream);

/* Tuning hook for measurements: pipeline stages per CTA (2..8) and persistent
 * CTAs per SM (1..2) of the split mode; 0 selects the automatic choice. */
int fcci_decode_set_tuning(int stages, int ctas_per_sm);
/* Measurement hook for the split mode's cluster launch (one cluster per (sequence, kv
 * head) pair when there are at most half as many pairs as resident CTAs):
 *   max_cluster  largest cluster; 0 = automatic (16), 1 = no clusters
 *   solo_tiles   pairs of at most this many 64-key tiles are carried by one CTA of
 *                their cluster instead of being split; -1 = automatic
 *   min_tiles    with a batched arena, each CTA of a cluster owns at least this many
 *                tiles when a pair fills the arena's capacity; 0 = automatic */
int fcci_decode_set_cluster_tuning(int max_cluster, int solo_tiles, int min_tiles);

/* Status of the last call on this host thread, and its message. */
int fcci_last_status(void);
const char* fcci_last_error_string(void);

/* Number of kernel launches this library has issued (process-wide counter). */
uint64_t fcci_launch_count(void);

/* Self-test of failure detection (no reference counterpart): one CTA runs the bounded
 * mbarrier wait that every pipeline wait of these kernels uses, on a barrier nothing
 * arrives on, with limit_ns in (0, 1 s]. result[0] receives FCCI_DEV_ERR_TIMEOUT when
 * the wait gave up (the expected outcome), result[1] the milliseconds it waited.
 * Synchronises `stream`. Nothing faults or hangs: the kernel returns after the limit. */
int fcci_selftest_bounded_wait(uint64_t limit_ns, uint32_t* result, cudaStream_t stream);

/*
 * Reference symbol (custom_kernels/attn_varlen_kernel.cu:88-99).
 * q [H,D], k/v [H,T,D] contiguous, ctx_out [H,D]; attention of each head over
 * the first T keys with softmax scale `scale`. D must be 64, 128 or 256.
 */
void attn_varlen_host(const __half* q, const __half* k, const __half* v, int32_t H, int32_t T, int32_t D,
                      float scale, __half* ctx_out, cudaStream_t stream);

/*
 * Reference symbol (custom_kernels/capture_decode_step_kernel.cu:101-121).
 * Placeholder decode step, kept identical: with T = seq_len_ptr[0], zero
 * arena_k/arena_v[l, 0, h, T, :] for every layer l and head h, set
 * logits_out[0..vocab) = 0 except logits_out[ctrl_input[0] % vocab] = 1,
 * then seq_len_ptr[0] = T + 1. position_ptr is unused, as in the reference.
 */
void capture_decode_host(const int64_t* ctrl_input, void* arena_k, void* arena_v, int32_t* seq_len_ptr,
                         const int32_t* position_ptr, float* logits_out, int32_t L, int32_t H, int32_t max_len,
                         int32_t D, int32_t vocab, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FCCI_DECODE_H */
