// Causal varlen prefill for B200 (sm_100a): RoPE + KV-arena append + attention
// on the 5th-generation tensor cores (tcgen05 MMAs, accumulators in TMEM).
//
// Replaces the prefill of the reference server's kv_init
// (case4_graph_generator_server_ipc.py:1241-1262): the HF LlamaAttention forward
// over the prompt (rotate-half RoPE, causal softmax(q k^T * scale) v, fp32
// softmax) and the copy of each layer's past_key_values into the arena.
//
// One step = up to three launches on the caller's stream:
//   1. rope_table_kernel   cos/sin of every (position, frequency) pair, kept in the
//                          workspace and rebuilt only when theta, rotary_dim or
//                          the arena capacity change (a header records them)
//   2. prefill_prep_kernel RoPE of q (into the workspace) and k_new (into the
//                          arena at T_b + i), v_new into the arena, and - in its
//                          last CTA - the work list
//   3. prefill_attn_kernel persistent attention over the work list
//
// Attention work item = (sequence b, query head h, query pair p): the 256 new
// tokens [256p, 256p + 256) of b as two 128-row query tiles Q0, Q1 sharing every
// K/V tile they read. Items are listed sequence-major (longest sequence first),
// head, then pair from last to first, so CTAs running at the same time read the
// K/V tiles of a few heads and those stay in L2. CTAs take items from an atomic
// counter.
//
// Inside a CTA (384 threads):
//   warp 0      TMA producer: Q0/Q1 tiles, then K_j / V_j tiles (128 keys each)
//               through a two-stage (K) and a three-stage (V) ring
//   warp 1      TMEM owner and MMA issuer (one thread issues, the warp zeroes the
//               V rows past the end of a sequence before they are multiplied)
//   warps 4-7   softmax of Q0 rows, warps 8-11 softmax of Q1 rows: thread r owns
//               row r, so row max and row sum need no shuffles
// TMEM (512 columns): S0 | S1 | O0 | O1, 128 fp32 columns each. P_g (fp16) is
// written over the first 64 columns of S_g and read from there by the PV MMA.
//   S_g  = Q_g K_j^T       tcgen05.mma kind::f16, M=128 N=128, A and B K-major
//   O_g += P_g V_j         A = P_g from TMEM, B = V_j MN-major (head_dim contiguous)
// The row maximum is only moved when it grows by more than 2^8 (P then stays
// below 256, exact in fp16 range), so the O correction (TMEM load, scale,
// store) is rare after the first tiles.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "fcci_decode.h"
#include "fcci_internal.h"
#include "fcci_prefill.h"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace fcci {
namespace pf {

constexpr int D = 128;
constexpr int kThreads = 384;
constexpr int kTileRows = 128;
constexpr int kPairRows = 256;
constexpr int kTileBytes = kTileRows * D * 2;  // 32 KB: 128 rows x 128 fp16
constexpr int kHalfBytes = kTileBytes / 2;     // one 64-column block
// K tiles in flight: 2 (K_j + 1 is read one tile ahead of the PV of tile j). V tiles: 3. A
// V stage is released only when the PV MMAs of its tile complete, so with two stages
// V_{j+2} started loading about one tile period before the MMA warp needed it, and
// the MMA warp waited for it (an L2-latency stall on every tile).
constexpr int kVStages = 3;
constexpr int kTmemCols = 512;
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s: far beyond any healthy wait
constexpr uint64_t kDrainLimitNs = 500000000ull;
constexpr float kRescaleLog2 = 8.0f;
constexpr uint32_t kTableMagic = 0x52504531u;  // "RPE1"
constexpr int kMaxSortB = 1024;                 // sequences ranked by length up to this batch size
constexpr int kPrepThreads = 256;

// Column pairs of each 32-column slice of S whose exponentials run on the FMA
// pipe (bit i: columns 2i, 2i+1); the others use the SFU's ex2. Per key tile and
// SM the two query tiles need as many exponentials (2 x 16384, 2048 cycles at 16
// per cycle) as the MMAs need tensor cycles (2048). Measured on the prefill16
// workload, moving 4, 5 or 8 of 16 pairs to the FMA pipe made the attention
// launch 3, 3.5 and 7.6 % slower than the SFU alone (the softmax is bound by its
// per-row instruction chain, not by the SFU), so the default is 0.
#ifndef FCCI_PF_POLY_MASK
#define FCCI_PF_POLY_MASK 0x0u
#endif
constexpr uint32_t kPolyMask = FCCI_PF_POLY_MASK;
#ifndef FCCI_PF_REG_SPLIT
#define FCCI_PF_REG_SPLIT 1
#endif
constexpr int kRegsLow = 104, kRegsHigh = 200;

struct Params {
    const __half* q;
    int64_t q_st, q_sh;
    const __half* k_new;
    int64_t kn_st, kn_sh;
    const __half* v_new;
    int64_t vn_st, vn_sh;
    __half* k_cache;
    int64_t k_sb, k_sh, k_st;
    __half* v_cache;
    int64_t v_sb, v_sh, v_st;
    int32_t capacity;
    const int32_t* cu_q;
    const int32_t* cu_kv;
    int32_t* seq_lens;
    int32_t fixed_len;
    __half* out;
    int64_t o_st, o_sh;
    float scale_log2;
    float rope_theta;
    int32_t rotary_dim;
    int32_t advance;
    int32_t B, Hq, Hkv, G, total_q, max_q;
    int32_t table_pos;  // positions covered by the table (= capacity)
    // workspace
    uint32_t* err;
    uint32_t* item_cnt;
    uint32_t* exit_cnt;
    int32_t* n_items;
    uint32_t* table_hdr;  // magic, theta bits, rotary_dim, positions
    uint32_t* table_cnt;
    int4* items;
    __half* q_rot;
    float2* table;
};

struct WsLayout {
    size_t items, q_rot, table, total;
    int64_t max_items;
};

static WsLayout ws_layout(int B, int Hq, int total_q, int max_q, int capacity, int rotary_dim) {
    auto up = [](size_t x) { return (x + 1023) & ~size_t(1023); };
    WsLayout w;
    const int64_t pairs = (int64_t)B * ((max_q + kPairRows - 1) / kPairRows);
    w.max_items = pairs * Hq;
    // the table sits at a fixed offset: its header stays valid across calls whose
    // token counts differ
    w.table = 1024;
    w.items = w.table + up((size_t)capacity * (rotary_dim / 2) * sizeof(float2));
    w.q_rot = w.items + up((size_t)w.max_items * sizeof(int4));
    w.total = w.q_rot + up((size_t)total_q * Hq * D * 2);
    return w;
}

// ------------------------------------------------------------------ device helpers

struct SeqRange {
    int T, n, tok0, kvrow0, kvb;
    bool ok;
};

__device__ __forceinline__ SeqRange seq_range(const Params& p, int b) {
    SeqRange s;
    s.tok0 = p.cu_q[b];
    s.n = p.cu_q[b + 1] - s.tok0;
    s.T = p.seq_lens ? p.seq_lens[b] : p.fixed_len;
    int cap = p.capacity;
    bool ok = true;
    if (p.cu_kv) {
        const int lo = p.cu_kv[b], hi = p.cu_kv[b + 1];
        s.kvrow0 = lo;
        s.kvb = 0;
        cap = hi - lo;
        ok = lo >= 0 && hi >= lo && hi <= p.capacity;
    } else {
        s.kvrow0 = 0;
        s.kvb = b;
    }
    ok = ok && s.T >= 0 && s.n >= 0 && s.n <= p.max_q && s.tok0 >= 0 && s.tok0 + s.n <= p.total_q &&
         (long long)s.T + s.n <= cap;
    s.ok = ok;
    return s;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x for two values x <= 8 on the FMA pipe (no SFU). Cody-Waite range reduction:
// x = n + f with n = round(x), taken from the low bits of x + 1.5 * 2^23, and
// f = x - n in [-1/2, 1/2]; 2^f by a degree-3 polynomial whose coefficients were
// fitted with the Remez exchange algorithm to the minimax relative error on
// [-1/2, 1/2] (max 7.5e-5 in fp32 Horner form, below half an fp16 ulp: P is
// rounded to fp16 for the PV MMA); 2^n is added into the exponent field. x is
// clamped at -120 first so that the exponent cannot underflow (2^-120 rounds to
// 0 in fp16 like the true value; -inf from masked columns gives 2^-120 * ~1).
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: x + kRound rounds x to an integer
    constexpr float c0 = 0.99992806f, c1 = 0.69326097f, c2 = 0.24261113f, c3 = 0.05517167f;
    x.x = fmaxf(x.x, -120.f);
    x.y = fmaxf(x.y, -120.f);
    const float2 j = __fadd2_rn(x, make_float2(kRound, kRound));
    const float2 n = __fadd2_rn(j, make_float2(-kRound, -kRound));
    const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
    float2 p = __ffma2_rn(make_float2(c3, c3), f, make_float2(c2, c2));
    p = __ffma2_rn(p, f, make_float2(c1, c1));
    p = __ffma2_rn(p, f, make_float2(c0, c0));
    // the low 9 bits of j hold n (two's complement): shifted into the exponent
    // field they add n to the exponent of p in [2^-1/2, 2^1/2]
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(j.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(j.y) << 23)));
}

__device__ __forceinline__ void set_error(const Params& p, uint32_t bit) {
    if (p.err) atomicOr(p.err, bit);
}

// RoPE angle and cos/sin exactly as the decode path (and the reference driver,
// scripts/direct_custom_decode_500.py:96-104): inv = theta ** (-i / half),
// angle = pos * inv, fp32 throughout.
__device__ __forceinline__ float2 rope_cs(float theta, int i, int half, int pos) {
    const float e = __fdiv_rn(-(float)i, (float)half);
    const float inv = powf(theta, e);
    const float ang = __fmul_rn((float)pos, inv);
    return make_float2(cosf(ang), sinf(ang));
}

__device__ __forceinline__ float rope_one(float x, float partner, float2 cs, bool first_half) {
    return first_half ? __fsub_rn(__fmul_rn(x, cs.x), __fmul_rn(partner, cs.y))
                      : __fadd_rn(__fmul_rn(x, cs.x), __fmul_rn(partner, cs.y));
}

// ------------------------------------------------------------------ 1. RoPE table

__global__ void __launch_bounds__(256) rope_table_kernel(const Params p) {
    const int rhalf = p.rotary_dim / 2;
    const uint32_t* h = p.table_hdr;
    const bool valid = h[0] == kTableMagic && h[1] == __float_as_uint(p.rope_theta) &&
                       h[2] == (uint32_t)p.rotary_dim && h[3] >= (uint32_t)p.table_pos;
    if (valid) return;  // every CTA of this launch sees the same header: only the last writes it
    const int64_t total = (int64_t)p.table_pos * rhalf;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int pos = (int)(idx / rhalf), i = (int)(idx % rhalf);
        p.table[idx] = rope_cs(p.rope_theta, i, rhalf, pos);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t c = atomicAdd(p.table_cnt, 1u);
        if (c == gridDim.x - 1) {
            __threadfence();
            volatile uint32_t* vh = p.table_hdr;
            vh[1] = __float_as_uint(p.rope_theta);
            vh[2] = (uint32_t)p.rotary_dim;
            vh[3] = (uint32_t)p.table_pos;
            __threadfence();
            vh[0] = kTableMagic;
            *p.table_cnt = 0;
        }
    }
}

// ------------------------------------------------------------------ 2. prep

// Work list: items (b, h, pair) sequence-major with sequences ranked by T_b + n_b
// (longest first), then head, then pair from last to first. Also resets the
// attention kernel's counters. One CTA.
__device__ void build_work_list(const Params& p, int* sm) {
    const int tid = threadIdx.x;
    const int B = p.B;
    int* np = sm;              // [B] pairs of sequence b (0 when invalid)
    int* key = np + B;         // [B] ranking key
    int* order = key + B;      // [B] rank -> b
    int* off = order + B;      // [B+1] first item of rank r
    for (int b = tid; b < B; b += blockDim.x) {
        const SeqRange s = seq_range(p, b);
        np[b] = s.ok ? (s.n + kPairRows - 1) / kPairRows : 0;
        key[b] = s.ok ? s.T + s.n : -1;
        order[b] = b;
    }
    __syncthreads();
    if (B <= kMaxSortB) {
        for (int b = tid; b < B; b += blockDim.x) {
            const int kb = key[b];
            int r = 0;
            for (int o = 0; o < B; ++o) {
                const int ko = key[o];
                r += (ko > kb) || (ko == kb && o < b);
            }
            order[r] = b;
        }
        __syncthreads();
    }
    if (tid == 0) {
        int acc = 0;
        for (int r = 0; r < B; ++r) {
            off[r] = acc;
            acc += np[order[r]] * p.Hq;
        }
        off[B] = acc;
        *p.n_items = acc;
        *p.item_cnt = 0u;
        *p.exit_cnt = 0u;
    }
    __syncthreads();
    const int total = off[B];
    for (int v = tid; v < total; v += blockDim.x) {
        int lo = 0, hi = B - 1;  // last rank with off[r] <= v
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (off[mid] <= v) lo = mid; else hi = mid - 1;
        }
        const int b = order[lo];
        const int n = np[b];
        const int w = v - off[lo];
        const int h = w / n;
        const int pair = n - 1 - (w % n);
        p.items[v] = make_int4(b, h, pair, 0);
    }
}

// Last sequence b with cu_q[b] <= t.
__device__ __forceinline__ int seq_of_row(const int32_t* cu, int B, int t) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cu[mid] <= t) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// RoPE of 8 consecutive dims [d0, d0 + 8) of one head row; `partner` holds dims
// d0 +- rotary_dim/2. Dims at or beyond rotary_dim pass through.
__device__ __forceinline__ uint4 rope_chunk(uint4 own, uint4 partner, int d0, int rot, const float2* cs) {
    if (d0 >= rot) return own;
    const int rhalf = rot >> 1;
    const bool first = d0 < rhalf;
    const int i0 = first ? d0 : d0 - rhalf;
    const __half* x = reinterpret_cast<const __half*>(&own);
    const __half* y = reinterpret_cast<const __half*>(&partner);
    uint4 r;
    __half* o = reinterpret_cast<__half*>(&r);
#pragma unroll
    for (int e = 0; e < 8; ++e)
        o[e] = __float2half_rn(rope_one(__half2float(x[e]), __half2float(y[e]), cs[i0 + e], first));
    return r;
}

__global__ void __launch_bounds__(kPrepThreads) prefill_prep_kernel(const Params p) {
    extern __shared__ int prep_sm[];
    if (blockIdx.x == gridDim.x - 1) {
        build_work_list(p, prep_sm);
        return;
    }
    const int rot = p.rotary_dim, rhalf = rot >> 1;
    const int chunks = D / 8;  // 16-byte chunks per head row
    const int nq = p.Hq * chunks, nk = p.Hkv * chunks;
    for (int t = blockIdx.x; t < p.total_q; t += gridDim.x - 1) {
        const int b = seq_of_row(p.cu_q, p.B, t);
        const SeqRange s = seq_range(p, b);
        if (!s.ok) {
            if (threadIdx.x == 0) set_error(p, FCCI_DEV_ERR_CAPACITY);
            continue;
        }
        const int pos = s.T + (t - s.tok0);
        const float2* cs = p.table + (int64_t)pos * rhalf;
        const int64_t krow_b = p.cu_kv ? 0 : (int64_t)b * p.k_sb;
        const int64_t vrow_b = p.cu_kv ? 0 : (int64_t)b * p.v_sb;
        const int64_t kv_t = (int64_t)s.kvrow0 + pos;
        for (int task = threadIdx.x; task < nq + 2 * nk; task += blockDim.x) {
            if (task < nq) {
                const int h = task / chunks, c = task % chunks, d0 = c * 8;
                const __half* src = p.q + (int64_t)t * p.q_st + (int64_t)h * p.q_sh;
                const uint4 own = *reinterpret_cast<const uint4*>(src + d0);
                uint4 r = own;
                if (d0 < rot) {
                    const int pd = d0 < rhalf ? d0 + rhalf : d0 - rhalf;
                    r = rope_chunk(own, *reinterpret_cast<const uint4*>(src + pd), d0, rot, cs);
                }
                *reinterpret_cast<uint4*>(p.q_rot + ((int64_t)t * p.Hq + h) * D + d0) = r;
            } else if (task < nq + nk) {
                const int w = task - nq, h = w / chunks, c = w % chunks, d0 = c * 8;
                const __half* src = p.k_new + (int64_t)t * p.kn_st + (int64_t)h * p.kn_sh;
                const uint4 own = *reinterpret_cast<const uint4*>(src + d0);
                uint4 r = own;
                if (d0 < rot) {
                    const int pd = d0 < rhalf ? d0 + rhalf : d0 - rhalf;
                    r = rope_chunk(own, *reinterpret_cast<const uint4*>(src + pd), d0, rot, cs);
                }
                *reinterpret_cast<uint4*>(p.k_cache + krow_b + (int64_t)h * p.k_sh + kv_t * p.k_st + d0) = r;
            } else {
                const int w = task - nq - nk, h = w / chunks, c = w % chunks, d0 = c * 8;
                const __half* src = p.v_new + (int64_t)t * p.vn_st + (int64_t)h * p.vn_sh;
                *reinterpret_cast<uint4*>(p.v_cache + vrow_b + (int64_t)h * p.v_sh + kv_t * p.v_st + d0) =
                    *reinterpret_cast<const uint4*>(src + d0);
            }
        }
    }
}

// ------------------------------------------------------------------ 3. attention

struct Item {
    int b, h, pair, T, n, tok0, kvrow0, kvb;  // b < 0: no more work
};

__device__ __forceinline__ int rows_of(const Item& it, int g) {
    const int r = it.n - (kPairRows * it.pair + kTileRows * g);
    return r < 0 ? 0 : (r > kTileRows ? kTileRows : r);
}

// Key tiles a query tile reads: up to and including the one holding its last row's position.
__device__ __forceinline__ int ntiles_of(const Item& it, int g) {
    const int r = rows_of(it, g);
    return r > 0 ? (it.T + kPairRows * it.pair + kTileRows * g + r - 1) / kTileRows + 1 : 0;
}

struct Smem {
    // tiles (each 1024-byte aligned): Q0 Q1 | K0 K1 | V stages
    static constexpr int kQ = 0;
    static constexpr int kK = 2 * kTileBytes;
    static constexpr int kV = 4 * kTileBytes;
    static constexpr int kBars = (4 + kVStages) * kTileBytes;
    // barriers (uint64 each)
    static constexpr int kQFull = 0, kQEmpty = 2, kKFull = 4, kKEmpty = 6, kVFull = 8, kVEmpty = kVFull + kVStages,
                         kSFull = kVEmpty + kVStages, kPFull = kSFull + 2, kOFull = kPFull + 2, kItemFull = kOFull + 2,
                         kItemEmpty = kItemFull + 2, kDrain = kItemEmpty + 2, kNumBars = kDrain + 1;
    static_assert(kNumBars * 8 <= 256, "barrier area");
    static constexpr int kRing = kBars + 256;  // 2 x Item
    static constexpr int kMisc = kRing + 64;   // tmem base, abort flag, last-CTA flag
    static constexpr int kBytes = kMisc + 64;
    static constexpr int kAlloc = kBytes + 1024;  // slack for aligning the base
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    return mbar_wait_bounded(bar, parity, abort_flag, kWaitLimitNs);
}

// Every lane waits; the outcome is made warp-uniform so that a timeout seen by
// some lanes cannot split the warp before a .sync.aligned tcgen05 instruction.
__device__ __forceinline__ bool wait_bar_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, kWaitLimitNs));
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const Params p) {
    extern __shared__ uint8_t attn_raw[];
    uint8_t* sm = attn_raw + ((1024u - (smem_u32(attn_raw) & 1023u)) & 1023u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Smem::kBars);
    Item* ring = reinterpret_cast<Item*>(sm + Smem::kRing);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Smem::kMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + Smem::kMisc + 8);
    int* last_flag = reinterpret_cast<int*>(sm + Smem::kMisc + 16);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint64_t* q_full = bars + Smem::kQFull;
    uint64_t* q_empty = bars + Smem::kQEmpty;
    uint64_t* k_full = bars + Smem::kKFull;
    uint64_t* k_empty = bars + Smem::kKEmpty;
    uint64_t* v_full = bars + Smem::kVFull;
    uint64_t* v_empty = bars + Smem::kVEmpty;
    uint64_t* s_full = bars + Smem::kSFull;
    uint64_t* p_full = bars + Smem::kPFull;
    uint64_t* o_full = bars + Smem::kOFull;
    uint64_t* item_full = bars + Smem::kItemFull;
    uint64_t* item_empty = bars + Smem::kItemEmpty;
    uint64_t* drain = bars + Smem::kDrain;

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(q_full + i, 1);
            mbar_init(q_empty + i, 1);
            mbar_init(k_full + i, 1);
            mbar_init(k_empty + i, 1);
            mbar_init(s_full + i, 1);
            mbar_init(p_full + i, kTileRows);
            mbar_init(o_full + i, 1);
            mbar_init(item_full + i, 1);
            mbar_init(item_empty + i, 1 + 8);  // the MMA warp and the 8 softmax warps
        }
        for (int i = 0; i < kVStages; ++i) {
            mbar_init(v_full + i, 1);
            mbar_init(v_empty + i, 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        *last_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = *tmem_slot;
    const int n_items = *p.n_items;

    auto fail = [&](uint32_t bit) {
        *abort_flag = 1;
        set_error(p, bit);
    };

    // Register split per warpgroup, taken at the top of each warpgroup's branch so
    // that the compiler allocates each branch under its own limit: the producer /
    // MMA warpgroup (warps 0-3; warps 2-3 idle) drops to kRegsLow, the two softmax
    // warpgroups rise to kRegsHigh. 128 x kRegsLow + 256 x kRegsHigh must not
    // exceed the 384 x 168 registers the block is launched with, or the increase
    // would wait for registers that never come free.
    static_assert(128 * kRegsLow + 256 * kRegsHigh <= kThreads * 168, "register split above the launch's total");
    if (warp < 4) {
#if FCCI_PF_REG_SPLIT
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
#endif
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tmap(&map_q);
            prefetch_tmap(&map_k);
            prefetch_tmap(&map_v);
            const uint64_t pol_q = l2_policy_evict_first();
            int tctr = 0;
            int nq[2] = {0, 0};
            bool ok = true, kv_short = false;
            for (int it = 0; ok; ++it) {
                const int slot = it & 1;
                if (!wait_bar(item_empty + slot, ((it >> 1) & 1) ^ 1, abort_flag)) {
                    fail(FCCI_DEV_ERR_TIMEOUT);
                    break;
                }
                Item item;
                item.b = -1;
                while (true) {
                    const uint32_t v = atomicAdd(p.item_cnt, 1u);
                    if (v >= (uint32_t)n_items) break;
                    const int4 e = p.items[v];
                    const SeqRange s = seq_range(p, e.x);
                    if (!s.ok) {
                        set_error(p, FCCI_DEV_ERR_CAPACITY);
                        continue;
                    }
                    item = Item{e.x, e.y, e.z, s.T, s.n, s.tok0, s.kvrow0, s.kvb};
                    break;
                }
                ring[slot] = item;
                mbar_arrive(item_full + slot);
                if (item.b < 0) break;
                const int hk = item.h / p.G;
                for (int g = 0; g < 2 && ok; ++g) {
                    if (rows_of(item, g) == 0) continue;
                    if (!wait_bar(q_empty + g, (nq[g] & 1) ^ 1, abort_flag)) {
                        fail(FCCI_DEV_ERR_TIMEOUT);
                        ok = false;
                        break;
                    }
                    uint8_t* dst = sm + Smem::kQ + g * kTileBytes;
                    const int row = item.tok0 + kPairRows * item.pair + kTileRows * g;
                    mbar_arrive_expect_tx(q_full + g, kTileBytes);
                    tma_load_3d(dst, &map_q, 0, item.h, row, q_full + g, pol_q);
                    tma_load_3d(dst + kHalfBytes, &map_q, 64, item.h, row, q_full + g, pol_q);
                    ++nq[g];
                }
                const int nt = max(ntiles_of(item, 0), ntiles_of(item, 1));
                for (int j = 0; j < nt && ok; ++j, ++tctr) {
                    const int st = tctr & 1;
                    const uint32_t par = ((tctr >> 1) & 1) ^ 1;
                    const int row = item.kvrow0 + kTileRows * j;
                    if (!wait_bar(k_empty + st, par, abort_flag)) {
                        fail(FCCI_DEV_ERR_TIMEOUT);
                        ok = false;
                        break;
                    }
                    uint8_t* kd = sm + Smem::kK + st * kTileBytes;
                    mbar_arrive_expect_tx(k_full + st, kTileBytes);
                    tma_load_4d_plain(kd, &map_k, 0, row, hk, item.kvb, k_full + st);
                    tma_load_4d_plain(kd + kHalfBytes, &map_k, 64, row, hk, item.kvb, k_full + st);
                    const int vs = tctr % kVStages;
                    if (!wait_bar(v_empty + vs, ((tctr / kVStages) & 1) ^ 1, abort_flag)) {
                        fail(FCCI_DEV_ERR_TIMEOUT);
                        ok = false;
                        // the K tile just issued is drained below (its V tile was not)
                        ++tctr;
                        kv_short = true;
                        break;
                    }
                    uint8_t* vd = sm + Smem::kV + vs * kTileBytes;
                    mbar_arrive_expect_tx(v_full + vs, kTileBytes);
                    tma_load_4d_plain(vd, &map_v, 0, row, hk, item.kvb, v_full + vs);
                    tma_load_4d_plain(vd + kHalfBytes, &map_v, 64, row, hk, item.kvb, v_full + vs);
                }
            }
            if (*abort_flag) {
                // wait (bounded) for this thread's copies still in flight before the CTA exits
                volatile int never = 0;
                for (int g = 0; g < 2; ++g)
                    if (nq[g] > 0) mbar_wait_bounded(q_full + g, (nq[g] - 1) & 1, &never, kDrainLimitNs);
                for (int st = 0; st < 2; ++st) {
                    const int uses = (tctr - st + 1) / 2;  // K tiles issued on stage st
                    if (uses > 0) mbar_wait_bounded(k_full + st, (uses - 1) & 1, &never, kDrainLimitNs);
                }
                const int vtiles = kv_short ? tctr - 1 : tctr;  // V tiles issued
                for (int st = 0; st < kVStages; ++st) {
                    const int uses = (vtiles - st + kVStages - 1) / kVStages;
                    if (uses > 0) mbar_wait_bounded(v_full + st, (uses - 1) & 1, &never, kDrainLimitNs);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t id_qk = tc::idesc_f16_f32(128, 128, 0, 0);
        const uint32_t id_pv = tc::idesc_f16_f32(128, 128, 0, 1);
        const uint32_t sq = smem_u32(sm + Smem::kQ), sk = smem_u32(sm + Smem::kK), sv = smem_u32(sm + Smem::kV);
        // One descriptor per operand buffer per call; a byte offset b inside the
        // buffer adds b / 16 to the 14-bit start-address field in the low word (no
        // carry: shared-memory addresses stay below 256 KB), so each MMA costs the
        // issuing thread one 32-bit add per operand instead of a rebuilt descriptor.
        // The MMA warp shares its SM sub-partition with two softmax warps; fewer
        // instructions per MMA let it keep the tensor pipe fed.
        auto desc_off = [](uint64_t d, uint32_t bytes) -> uint64_t {
            return ((d >> 32) << 32) | (uint32_t)((uint32_t)d + (bytes >> 4));
        };
        auto issue_s = [&](int g, int st) {  // S_g = Q_g K^T
            const uint64_t qd = tc::smem_desc_sw128(sq + g * kTileBytes, 16, 1024);
            const uint64_t kd = tc::smem_desc_sw128(sk + st * kTileBytes, 16, 1024);
            const uint32_t dt = tbase + kTileRows * g;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
                tc::mma_ss(dt, desc_off(qd, off), desc_off(kd, off), id_qk, kk > 0);
            }
        };
        auto issue_pv = [&](int g, int st, bool acc) {  // O_g += P_g V
            const uint64_t vd = tc::smem_desc_sw128(sv + st * kTileBytes, kHalfBytes, 1024);
            const uint32_t dt = tbase + 256 + kTileRows * g, at = tbase + kTileRows * g;
#pragma unroll
            for (int kk = 0; kk < kTileRows / 16; ++kk)
                tc::mma_ts(dt, at + kk * 8, desc_off(vd, kk * 2048), id_pv, (acc || kk > 0) ? 1u : 0u);
        };
        int tctr = 0;
        int nq[2] = {0, 0}, np_[2] = {0, 0};
        bool ok = true;
        for (int it = 0; ok; ++it) {
            const int slot = it & 1;
            if (!wait_bar_warp(item_full + slot, (it >> 1) & 1, abort_flag)) {
                fail(FCCI_DEV_ERR_TIMEOUT);
                break;
            }
            const Item item = ring[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(item_empty + slot);
            if (item.b < 0) break;
            const int nt_g[2] = {ntiles_of(item, 0), ntiles_of(item, 1)};
            const int nt = max(nt_g[0], nt_g[1]);
            const int keys = item.T + item.n;
            // tile 0: S_g(0) for both query tiles
            {
                const int st = tctr & 1;
                if (!wait_bar_warp(k_full + st, (tctr >> 1) & 1, abort_flag)) {
                    fail(FCCI_DEV_ERR_TIMEOUT);
                    break;
                }
                for (int g = 0; g < 2 && ok; ++g) {
                    if (nt_g[g] == 0) continue;
                    if (!wait_bar_warp(q_full + g, nq[g] & 1, abort_flag)) {
                        fail(FCCI_DEV_ERR_TIMEOUT);
                        ok = false;
                        break;
                    }
                    ++nq[g];
                    if (lane == 0) {
                        issue_s(g, st);
                        tc::commit(s_full + g);
                        // the last MMA that reads Q_g: the producer may load the next
                        // item's Q_g once it completes
                        if (nt_g[g] == 1) tc::commit(q_empty + g);
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (lane == 0) tc::commit(k_empty + st);
                __syncwarp();
            }
            for (int j = 0; j < nt && ok; ++j) {
                const int t = tctr + j, vs = t % kVStages;
                if (!wait_bar_warp(v_full + vs, (t / kVStages) & 1, abort_flag)) {
                    fail(FCCI_DEV_ERR_TIMEOUT);
                    ok = false;
                    break;
                }
                if (j == nt - 1 && kTileRows * (j + 1) > keys) {
                    // keys past the end of the sequence: zero their V rows (arena
                    // rows beyond T_b + n_b may hold anything, and 0 * NaN = NaN)
                    uint8_t* vt = sm + Smem::kV + vs * kTileBytes;
                    const int r0 = keys - kTileRows * j;
                    for (int c = r0 * 16 + lane; c < kTileRows * 16; c += 32) {
                        const int r = c >> 4, half = (c >> 3) & 1, ch = c & 7;
                        *reinterpret_cast<uint4*>(vt + half * kHalfBytes + r * 128 + ch * 16) =
                            make_uint4(0u, 0u, 0u, 0u);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                }
                bool next_k = false;
                for (int g = 0; g < 2; ++g) {
                    if (j >= nt_g[g]) continue;
                    if (!wait_bar_warp(p_full + g, np_[g] & 1, abort_flag)) {
                        fail(FCCI_DEV_ERR_TIMEOUT);
                        ok = false;
                        break;
                    }
                    ++np_[g];
                    tc::fence_after_sync();
                    if (lane == 0) issue_pv(g, vs, j > 0);
                    __syncwarp();
                    if (j + 1 < nt_g[g]) {
                        if (!next_k) {
                            const int t1 = t + 1;
                            if (!wait_bar_warp(k_full + (t1 & 1), (t1 >> 1) & 1, abort_flag)) {
                                fail(FCCI_DEV_ERR_TIMEOUT);
                                ok = false;
                                break;
                            }
                            next_k = true;
                        }
                        if (lane == 0) {
                            issue_s(g, (t + 1) & 1);
                            tc::commit(s_full + g);
                            if (j + 2 == nt_g[g]) tc::commit(q_empty + g);  // last S_g of the item
                        }
                    } else if (lane == 0) {
                        tc::commit(o_full + g);
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (lane == 0) {
                    if (next_k) tc::commit(k_empty + ((t + 1) & 1));
                    tc::commit(v_empty + vs);
                }
                __syncwarp();
            }
            tctr += nt;
        }
        // every MMA this thread issued has completed before TMEM is released
        if (lane == 0) {
            tc::commit(drain);
            volatile int never = 0;
            mbar_wait_bounded(drain, 0, &never, kDrainLimitNs);
        }
        __syncwarp();
    }
    } else {
#if FCCI_PF_REG_SPLIT
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
#endif
        // ------------------------------------------------------------ softmax + epilogue
        const int g = (warp - 4) >> 2;
        const int r = tid - 128 * (1 + g);  // query row of this thread in tile g
        const uint32_t lane_base = (uint32_t)(warp & 3) * 32;
        const uint32_t s_addr = tc::taddr(tbase, lane_base, kTileRows * g);
        const uint32_t o_addr = tc::taddr(tbase, lane_base, 256 + kTileRows * g);
        const float sl2 = p.scale_log2;
        int ns = 0, no = 0;
        for (int it = 0;; ++it) {
            const int slot = it & 1;
            if (!wait_bar_warp(item_full + slot, (it >> 1) & 1, abort_flag)) {
                fail(FCCI_DEV_ERR_TIMEOUT);
                break;
            }
            const Item item = ring[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(item_empty + slot);
            if (item.b < 0) break;
            const int nt = ntiles_of(item, g);
            if (nt == 0) continue;
            const int rows = rows_of(item, g);
            const int qrow = kPairRows * item.pair + kTileRows * g + r;  // row among the new tokens
            const int klim = min(item.T + qrow + 1, item.T + item.n);   // keys [0, klim) are visible
            float m = -INFINITY, l = 0.f;
            bool ok = true;
            for (int j = 0; j < nt; ++j) {
                if (!wait_bar_warp(s_full + g, ns & 1, abort_flag)) {
                    fail(FCCI_DEV_ERR_TIMEOUT);
                    ok = false;
                    break;
                }
                ++ns;
                tc::fence_after_sync();
                uint32_t sr[4][32];
#pragma unroll
                for (int c = 0; c < 4; ++c) tc::ld32(s_addr + 32 * c, sr[c]);
                tc::wait_ld();
                const int vis = klim - kTileRows * j;  // visible columns of this tile
                if (vis < kTileRows) {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (32 * c + i >= vis) sr[c][i] = __float_as_uint(-INFINITY);
                }
                // row maximum: three-input max, two independent chains
                float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        mxa = fmax3(mxa, __uint_as_float(sr[c][i]), __uint_as_float(sr[c][i + 1]));
                        mxb = fmax3(mxb, __uint_as_float(sr[c][i + 2]), __uint_as_float(sr[c][i + 3]));
                    }
                float mx = fmaxf(mxa, mxb) * sl2;
                float alpha = 1.f;
                const bool resc = mx > m + kRescaleLog2;
                if (resc) {
                    alpha = ex2(m - mx);  // 0 when m = -inf
                    m = mx;
                    l *= alpha;
                }
                const float mu = (m == -INFINITY) ? 0.f : m;
                const float2 scl = make_float2(sl2, sl2), nmu = make_float2(-mu, -mu);
                float2 rsa = make_float2(0.f, 0.f), rsb = make_float2(0.f, 0.f);
                // P = 2^(s * scale * log2 e - m) as fp16 over the first 64 columns of S_g;
                // column pairs in kPolyMask on the FMA pipe, the rest on the SFU
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 x = __ffma2_rn(
                            make_float2(__uint_as_float(sr[q4][2 * i]), __uint_as_float(sr[q4][2 * i + 1])), scl, nmu);
                        const float2 e = ((kPolyMask >> i) & 1u) ? exp2_fma2(x) : make_float2(ex2(x.x), ex2(x.y));
                        if (i & 1)
                            rsb = __fadd2_rn(rsb, e);
                        else
                            rsa = __fadd2_rn(rsa, e);
                        pk[i] = pack_half2(e.x, e.y);
                    }
                    tc::st16(s_addr + 16 * q4, pk);
                }
                const float rs = (rsa.x + rsa.y) + (rsb.x + rsb.y);
                // rows whose maximum moved rescale O_g (idle: PV_g of the previous
                // tile completed before S_g of this one was signalled)
                if (j > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t orr[32];
                        tc::ld32(o_addr + 32 * c, orr);
                        tc::wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
                        tc::st32(o_addr + 32 * c, orr);
                    }
                }
                l += rs;
                tc::wait_st();
                tc::fence_before_sync();
                mbar_arrive(p_full + g);
            }
            if (!ok) break;
            if (!wait_bar_warp(o_full + g, no & 1, abort_flag)) {
                fail(FCCI_DEV_ERR_TIMEOUT);
                break;
            }
            ++no;
            tc::fence_after_sync();
            const float inv = 1.f / l;
            __half* dst = p.out + (int64_t)(item.tok0 + qrow) * p.o_st + (int64_t)item.h * p.o_sh;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t orr[32];
                tc::ld32(o_addr + 32 * c, orr);
                tc::wait_ld();
                if (r < rows) {
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint4 w;
                        w.x = pack_half2(__uint_as_float(orr[8 * v + 0]) * inv, __uint_as_float(orr[8 * v + 1]) * inv);
                        w.y = pack_half2(__uint_as_float(orr[8 * v + 2]) * inv, __uint_as_float(orr[8 * v + 3]) * inv);
                        w.z = pack_half2(__uint_as_float(orr[8 * v + 4]) * inv, __uint_as_float(orr[8 * v + 5]) * inv);
                        w.w = pack_half2(__uint_as_float(orr[8 * v + 6]) * inv, __uint_as_float(orr[8 * v + 7]) * inv);
                        *reinterpret_cast<uint4*>(dst + 32 * c + 8 * v) = w;
                    }
                }
            }
            tc::fence_before_sync();
        }
    }

    // ---------------------------------------------------------------- teardown
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, kTmemCols);
    }
    if (tid == 0) {
        __threadfence();
        const uint32_t c = atomicAdd(p.exit_cnt, 1u);
        *last_flag = (c == gridDim.x - 1) ? 1 : 0;
    }
    __syncthreads();
    if (*last_flag) {
        // every CTA has finished every item: seq_lens may move, counters reset
        __threadfence();
        if (p.advance && p.seq_lens) {
            for (int b = tid; b < p.B; b += blockDim.x) {
                const SeqRange s = seq_range(p, b);
                if (s.ok) p.seq_lens[b] = s.T + s.n;
            }
        }
        if (tid == 0) {
            *p.item_cnt = 0u;
            *p.exit_cnt = 0u;
        }
    }
}

// ------------------------------------------------------------------ host side

static bool aligned16(const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; }

static int fill(const fcci_prefill_desc* d, Params& p, WsLayout& L) {
    auto bad = [](int code, const char* why) { return set_status(code, why); };
    if (!d) return bad(FCCI_EINVAL, "fcci_prefill_attention: descriptor is NULL");
    if (d->abi_version != FCCI_PREFILL_ABI_VERSION) return bad(FCCI_EINVAL, "fcci_prefill_attention: abi_version mismatch");
    if (d->B <= 0 || d->Hq <= 0 || d->Hkv <= 0 || d->Hq % d->Hkv != 0)
        return bad(FCCI_EINVAL, "fcci_prefill_attention: B, Hq, Hkv must be positive and Hq a multiple of Hkv");
    if (d->D != D) return bad(FCCI_EUNSUPPORTED, "fcci_prefill_attention: head_dim must be 128");
    if (d->total_q < 0 || d->max_seqlen_q < 0) return bad(FCCI_EINVAL, "fcci_prefill_attention: negative token count");
    if (!d->cu_seqlens_q) return bad(FCCI_EINVAL, "fcci_prefill_attention: cu_seqlens_q is required");
    if (!d->q || !d->k_new || !d->v_new || !d->k_cache || !d->v_cache || !d->out)
        return bad(FCCI_EINVAL, "fcci_prefill_attention: q, k_new, v_new, k_cache, v_cache and out are required");
    if (d->capacity <= 0) return bad(FCCI_EINVAL, "fcci_prefill_attention: capacity must be positive");
    if (d->rotary_dim < 0 || d->rotary_dim > D || (d->rotary_dim % 16))
        return bad(FCCI_EUNSUPPORTED, "fcci_prefill_attention: rotary_dim must be a multiple of 16 within head_dim");
    if (!(d->scale > 0.f)) return bad(FCCI_EINVAL, "fcci_prefill_attention: scale must be positive");
    if (d->advance && !d->seq_lens) return bad(FCCI_EINVAL, "fcci_prefill_attention: advance needs seq_lens");
    if (!d->seq_lens && d->fixed_len < 0) return bad(FCCI_EINVAL, "fcci_prefill_attention: fixed_len must be non-negative");
    const void* ptrs[6] = {d->q, d->k_new, d->v_new, d->k_cache, d->v_cache, d->out};
    for (int i = 0; i < 6; ++i)
        if (!aligned16(ptrs[i])) return bad(FCCI_EINVAL, "fcci_prefill_attention: tensors must be 16-byte aligned");
    const int64_t st[14] = {d->q_stride_t,   d->q_stride_h,     d->k_new_stride_t, d->k_new_stride_h, d->v_new_stride_t,
                            d->v_new_stride_h, d->k_stride_b,   d->k_stride_h,     d->k_stride_t,     d->v_stride_b,
                            d->v_stride_h,   d->v_stride_t,     d->out_stride_t,   d->out_stride_h};
    for (int i = 0; i < 14; ++i)
        if (st[i] < 0 || (st[i] & 7))
            return bad(FCCI_EINVAL, "fcci_prefill_attention: strides must be non-negative multiples of 8 elements");
    if (d->k_stride_t == 0 || d->v_stride_t == 0) return bad(FCCI_EINVAL, "fcci_prefill_attention: arena token stride is zero");
    L = ws_layout(d->B, d->Hq, d->total_q, d->max_seqlen_q, d->capacity, d->rotary_dim);
    if (L.max_items > 0x7fffffff) return bad(FCCI_EINVAL, "fcci_prefill_attention: too many work items");
    if (!d->workspace || d->workspace_bytes < L.total)
        return bad(FCCI_EWORKSPACE, "fcci_prefill_attention: workspace missing or too small");
    memset(&p, 0, sizeof(p));
    p.q = static_cast<const __half*>(d->q);
    p.q_st = d->q_stride_t;
    p.q_sh = d->q_stride_h;
    p.k_new = static_cast<const __half*>(d->k_new);
    p.kn_st = d->k_new_stride_t;
    p.kn_sh = d->k_new_stride_h;
    p.v_new = static_cast<const __half*>(d->v_new);
    p.vn_st = d->v_new_stride_t;
    p.vn_sh = d->v_new_stride_h;
    p.k_cache = static_cast<__half*>(d->k_cache);
    p.k_sb = d->k_stride_b;
    p.k_sh = d->k_stride_h;
    p.k_st = d->k_stride_t;
    p.v_cache = static_cast<__half*>(d->v_cache);
    p.v_sb = d->v_stride_b;
    p.v_sh = d->v_stride_h;
    p.v_st = d->v_stride_t;
    p.capacity = d->capacity;
    p.cu_q = d->cu_seqlens_q;
    p.cu_kv = d->cu_seqlens_kv;
    p.seq_lens = d->seq_lens;
    p.fixed_len = d->fixed_len;
    p.out = static_cast<__half*>(d->out);
    p.o_st = d->out_stride_t;
    p.o_sh = d->out_stride_h;
    p.scale_log2 = d->scale * 1.4426950408889634f;
    p.rope_theta = d->rope_theta;
    p.rotary_dim = d->rotary_dim;
    p.advance = d->advance;
    p.B = d->B;
    p.Hq = d->Hq;
    p.Hkv = d->Hkv;
    p.G = d->Hq / d->Hkv;
    p.total_q = d->total_q;
    p.max_q = d->max_seqlen_q;
    p.table_pos = d->capacity;
    uint8_t* ws = static_cast<uint8_t*>(d->workspace);
    p.err = reinterpret_cast<uint32_t*>(ws + 0);
    p.item_cnt = reinterpret_cast<uint32_t*>(ws + 4);
    p.exit_cnt = reinterpret_cast<uint32_t*>(ws + 8);
    p.n_items = reinterpret_cast<int32_t*>(ws + 12);
    p.table_cnt = reinterpret_cast<uint32_t*>(ws + 16);
    p.table_hdr = reinterpret_cast<uint32_t*>(ws + 32);
    p.items = reinterpret_cast<int4*>(ws + L.items);
    p.q_rot = reinterpret_cast<__half*>(ws + L.q_rot);
    p.table = reinterpret_cast<float2*>(ws + L.table);
    return FCCI_OK;
}

// Validated launch state shared by the two halves of a step.
struct Launch {
    Params p;
    WsLayout L;
    int dev, sms;
};

static int setup(const fcci_prefill_desc* d, Launch& x) {
    int rc = fill(d, x.p, x.L);
    if (rc) return rc;
    if (cudaGetDevice(&x.dev) != cudaSuccess) return set_cuda_status(cudaGetLastError());
    x.sms = device_sm_count(x.dev);
    if (x.sms <= 0) return set_status(FCCI_ECUDA, "fcci_prefill_attention: no device");
    if (x.dev < 0 || x.dev >= 128) return set_status(FCCI_EINVAL, "fcci_prefill_attention: device index");
    static std::once_flag flags[128];
    static cudaError_t attr_err[128];
    static bool regs_short[128];
    const int dev = x.dev;
    std::call_once(flags[dev], [dev]() {
        attr_err[dev] =
            cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::kAlloc);
        if (attr_err[dev] == cudaSuccess)
            attr_err[dev] =
                cudaFuncSetAttribute(prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
#if FCCI_PF_REG_SPLIT
        // The softmax warpgroups' setmaxnreg.inc takes registers from the block's
        // launch allocation: if the kernel were built with fewer registers per
        // thread than the split assumes, the increase would wait forever. Refuse
        // to launch such a build.
        if (attr_err[dev] == cudaSuccess) {
            cudaFuncAttributes fa;
            attr_err[dev] = cudaFuncGetAttributes(&fa, prefill_attn_kernel);
            regs_short[dev] =
                attr_err[dev] == cudaSuccess && fa.numRegs * kThreads < 128 * kRegsLow + 256 * kRegsHigh;
        }
#endif
    });
    if (attr_err[dev] != cudaSuccess) return set_cuda_status(attr_err[dev]);
    if (regs_short[dev])
        return set_status(FCCI_EUNSUPPORTED,
                          "fcci_prefill_attention: kernel built with fewer registers than its warpgroup split needs");
    return FCCI_OK;
}

// RoPE table check, RoPE + append of the new tokens, work list.
int prefill_prepare(const fcci_prefill_desc* d, cudaStream_t stream) {
    Launch x;
    int rc = setup(d, x);
    if (rc) return rc;
    Params& p = x.p;
    if (p.total_q == 0) return FCCI_OK;
    const size_t prep_smem = (size_t)(4 * p.B + 1) * sizeof(int);
    if (prep_smem > 227 * 1024) return set_status(FCCI_EUNSUPPORTED, "fcci_prefill_attention: batch too large");
    if (p.rotary_dim > 0) {
        const int64_t entries = (int64_t)p.table_pos * (p.rotary_dim / 2);
        int grid = (int)((entries + 255) / 256);
        if (grid > x.sms * 8) grid = x.sms * 8;
        if (grid < 1) grid = 1;
        rope_table_kernel<<<grid, 256, 0, stream>>>(p);
        count_launch();
    }
    int grid = x.sms * 8;
    if (grid > p.total_q) grid = p.total_q;
    prefill_prep_kernel<<<grid + 1, kPrepThreads, prep_smem, stream>>>(p);
    count_launch();
    return set_cuda_status(cudaGetLastError());
}

// Causal attention over the work list written by prefill_prepare (same descriptor).
int prefill_attend(const fcci_prefill_desc* d, cudaStream_t stream) {
    Launch x;
    int rc = setup(d, x);
    if (rc) return rc;
    Params& p = x.p;
    if (p.total_q == 0) return FCCI_OK;
    // tensor maps: rotated queries [total_q, Hq, D] (workspace) and the arena
    CUtensorMap mq, mk, mv;
    {
        const uint64_t dims[3] = {(uint64_t)D, (uint64_t)p.Hq, (uint64_t)p.total_q};
        const int64_t sb[2] = {(int64_t)D * 2, (int64_t)p.Hq * D * 2};
        const uint32_t box[3] = {64, 1, (uint32_t)kTileRows};
        rc = encode_f16_sw128(&mq, p.q_rot, 3, dims, sb, box);
    }
    const int Bdim = p.cu_kv ? 1 : p.B;
    if (!rc) {
        const uint64_t dims[4] = {(uint64_t)D, (uint64_t)p.capacity, (uint64_t)p.Hkv, (uint64_t)Bdim};
        const int64_t sbk[3] = {p.k_st * 2, p.k_sh * 2, p.k_sb * 2};
        const int64_t sbv[3] = {p.v_st * 2, p.v_sh * 2, p.v_sb * 2};
        const uint32_t box[4] = {64, (uint32_t)kTileRows, 1, 1};
        rc = encode_f16_sw128(&mk, p.k_cache, 4, dims, sbk, box);
        if (!rc) rc = encode_f16_sw128(&mv, p.v_cache, 4, dims, sbv, box);
    }
    if (rc) return set_status(rc, "fcci_prefill_attention: cuTensorMapEncodeTiled rejected a layout");
    int grid = x.sms;
    if (x.L.max_items < grid) grid = (int)(x.L.max_items > 0 ? x.L.max_items : 1);
    prefill_attn_kernel<<<grid, kThreads, Smem::kAlloc, stream>>>(mq, mk, mv, p);
    count_launch();
    return set_cuda_status(cudaGetLastError());
}

}  // namespace pf
}  // namespace fcci

extern "C" int fcci_prefill_attention(const fcci_prefill_desc* desc, cudaStream_t stream) {
    int rc = fcci::pf::prefill_prepare(desc, stream);
    return rc ? rc : fcci::pf::prefill_attend(desc, stream);
}

extern "C" int fcci_prefill_prepare(const fcci_prefill_desc* desc, cudaStream_t stream) {
    return fcci::pf::prefill_prepare(desc, stream);
}

extern "C" int fcci_prefill_attend(const fcci_prefill_desc* desc, cudaStream_t stream) {
    return fcci::pf::prefill_attend(desc, stream);
}

extern "C" size_t fcci_prefill_workspace_bytes(int32_t B, int32_t Hq, int32_t Hkv, int32_t D, int32_t total_q,
                                               int32_t max_seqlen_q, int32_t capacity, int32_t rotary_dim) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || D != fcci::pf::D || total_q < 0 || max_seqlen_q < 0 || capacity <= 0 ||
        rotary_dim < 0 || rotary_dim > D)
        return 0;
    return fcci::pf::ws_layout(B, Hq, total_q, max_seqlen_q, capacity, rotary_dim).total;
}

extern "C" int fcci_prefill_workspace_init(void* workspace, size_t bytes, cudaStream_t stream) {
    if (!workspace || bytes < 1024) return fcci::set_status(FCCI_EWORKSPACE, "fcci_prefill_workspace_init: workspace too small");
    return fcci::set_cuda_status(cudaMemsetAsync(workspace, 0, 1024, stream));
}

extern "C" int fcci_prefill_read_error(void* workspace, uint32_t* flags, int clear, cudaStream_t stream) {
    if (!workspace || !flags) return fcci::set_status(FCCI_EINVAL, "fcci_prefill_read_error: NULL argument");
    cudaError_t e = cudaMemcpyAsync(flags, workspace, 4, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && clear) e = cudaMemsetAsync(workspace, 0, 4, stream);
    return fcci::set_cuda_status(e);
}
