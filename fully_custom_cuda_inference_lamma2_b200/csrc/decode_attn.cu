// Varlen split-KV decode attention for B200 (sm_100a), with RoPE, KV append and
// device-side seq_len bookkeeping fused into the same launch.
//
// Replaces, for one decode token per sequence:
//   - custom_kernels/attn_varlen_kernel.cu:9-86 (attention of one query per head)
//   - the torch RoPE / append / gather / repeat_interleave steps of the decode
//     drivers (scripts/direct_custom_decode_500.py:229-250)
//   - the seq_len bump of capture_decode_step_kernel.cu:95-99
//
// Work decomposition. A "pair" is (sequence b, kv head h); its L_b keys are cut
// into tiles of 64 keys. All tiles of all pairs form one line of N tiles. In
// split mode a persistent grid of C CTAs takes contiguous ranges
// [c*N/C, (c+1)*N/C) (stream-K), so every CTA streams the same number of tiles
// whatever the length mix. A pair lying inside one CTA's range is finished by
// that CTA; a pair cut by CTA boundaries leaves one partial (o, lse) per piece
// in slot (pair + cta) — unique because both cut sets are ordered — and the
// last piece to finish (atomic counter, never waited on) merges them. When there
// are few pairs (at most half as many as CTAs) the split grid is launched as
// thread-block clusters of k CTAs, one cluster per pair: with uniform tile counts
// each CTA of a cluster takes 1/k of its pair's tiles, keeps its (o, lse) piece
// in shared memory, and after a cluster barrier each CTA merges a slice of the
// outputs from all k pieces through distributed shared memory. No CTA ever waits
// on another CTA's global counter. In pair mode there is one CTA per pair and no
// workspace.
//
// Inside a CTA: warp 4 is the TMA producer (one thread), warps 0..3 consume.
// A stage holds the K and V tiles of 64 keys (2 x 64 x D fp16), loaded as
// 16-row x 64-col boxes with 128-byte swizzle through a 4-D tensor map
// (head_dim, token, kv head, sequence); only boxes holding valid keys are
// fetched. Consumer warp w owns keys [16w, 16w+16) of each tile:
//   S^T[key, head] = K Q^T     (mma m16n8k16: A = K rows via ldmatrix, B = the
//                               rotated queries of the GQA group, n = 8 heads)
//   online softmax per head column (quad shuffles), P^T -> B fragments with
//   movmatrix.trans,
//   O^T[dim, head] += V^T P^T  (A = V via ldmatrix.trans)
// so a group of 8 query heads fills the n=8 MMA tile exactly and every K/V byte
// is read from HBM once per group.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "fcci_decode.h"
#include "fcci_exchange.h"
#include "fcci_internal.h"
#include "ptx.cuh"

namespace fcci {

constexpr int kTileKeys = 64;
constexpr int kGroupKeys = 16;
constexpr int kConsumerWarps = 4;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kBoxBytes = kGroupKeys * 128;  // 16 rows x 64 fp16
constexpr int kHalfTileBytes = kTileKeys * 128;
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s: far beyond any healthy wait
constexpr int kMaxCluster = 16;  // CTAs per cluster of a cluster launch (non-portable above 8)
constexpr int kSoloTiles = 2;     // pairs of at most this many tiles are not split in a cluster launch
constexpr int kClusterMinTiles = 2;  // a cluster's CTAs each own at least this many tiles at full capacity
constexpr uint64_t kDrainLimitNs = 500000000ull;
constexpr int kConsumerBar = 1;

struct Params {
    const __half* q;
    int64_t q_sb, q_sh;
    const __half* k_new;
    int64_t kn_sb, kn_sh;
    const __half* v_new;
    int64_t vn_sb, vn_sh;
    __half* k_cache;
    int64_t k_sb, k_sh, k_st;
    __half* v_cache;
    int64_t v_sb, v_sh, v_st;
    int32_t capacity;
    const int32_t* cu_seqlens;
    int32_t* seq_lens;
    int32_t fixed_len;
    __half* out;
    int64_t o_sb, o_sh;
    __half* q_rot_out;
    float scale_log2;
    float rope_theta;
    int32_t rotary_dim;
    int32_t advance;
    int32_t append;
    int32_t split;
    int32_t prefetch_kv;  // FCCI_DECODE_PREFETCH_KV: lengths and the first stages before griddepcontrol.wait
    int32_t check_early;  // FCCI_DECODE_CHECK_EARLY_READ: launch the instantiation with the early-read guard
    int32_t cluster_k;    // CTAs per cluster of a split launch in clusters of one pair each; 0 otherwise
    int32_t solo_tiles;   // in such a launch, pairs of at most this many tiles stay on one CTA
    // ctx exchange (fcci_exchange.h): the slice also goes to n_peers peers' buffers at the
    // offsets it has in `out`; the last CTA raises slot xrank of every flag array
    int32_t n_peers, xrank;
    __half* peer_out[FCCI_MAX_PEERS];
    uint32_t* peer_flags[FCCI_MAX_PEERS];
    uint32_t* xflags;
    uint32_t* xepoch;
    int32_t B, Hq, Hkv, G;
    int32_t stages;
    uint32_t* err;
    uint32_t* done_cnt;
    uint32_t* pair_cnt;
    float* part_lse;
    float* part_o;
};

struct SeqInfo {
    int T;         // cached length before this step
    int L;         // keys attended (0 when the sequence is invalid)
    int tok_base;  // first token row of the sequence in the arena
    bool ok;
};

__device__ __forceinline__ SeqInfo seq_info(const Params& p, int b) {
    SeqInfo s;
    s.T = p.seq_lens ? p.seq_lens[b] : p.fixed_len;
    int cap = p.capacity;
    s.tok_base = 0;
    bool ok = true;
    if (p.cu_seqlens) {
        const int lo = p.cu_seqlens[b], hi = p.cu_seqlens[b + 1];
        s.tok_base = lo;
        cap = hi - lo;
        ok = lo >= 0 && hi >= lo && hi <= p.capacity;
    }
    s.L = s.T + p.append;
    ok = ok && s.T >= 0 && s.L <= cap;
    s.ok = ok;
    if (!ok) s.L = 0;
    return s;
}

__device__ __forceinline__ int tiles_of(int L) { return L > 0 ? (L + kTileKeys - 1) / kTileKeys : 1; }

// ctx element(s) at element offset `off` of `out`, and of every peer's buffer when the
// launch exchanges ctx (static peer indices: the parameter array stays in param space)
__device__ __forceinline__ void store_ctx2(const Params& p, int64_t off, __half2 v) {
    *reinterpret_cast<__half2*>(p.out + off) = v;
#pragma unroll
    for (int i = 0; i < FCCI_MAX_PEERS; ++i)
        if (i < p.n_peers) *reinterpret_cast<__half2*>(p.peer_out[i] + off) = v;
}

__device__ __forceinline__ void store_ctx1(const Params& p, int64_t off, __half v) {
    p.out[off] = v;
#pragma unroll
    for (int i = 0; i < FCCI_MAX_PEERS; ++i)
        if (i < p.n_peers) p.peer_out[i][off] = v;
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_release_sys(uint32_t* ptr, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

__device__ __forceinline__ void set_error(const Params& p, uint32_t bit) {
    if (p.err) atomicOr(p.err, bit);
}

// ceil((t+1)*C/N) - 1: the CTA whose range [c*N/C, (c+1)*N/C) contains tile t.
__device__ __forceinline__ int cta_of_tile(long long t, long long N, long long C) {
    return (int)(((t + 1) * C + N - 1) / N - 1);
}

// Accurate RoPE table entry i for position pos: the reference computes
// inv = theta ** (-i / half) and angle = pos * inv in fp32, then cos/sin in fp32
// (scripts/direct_custom_decode_500.py:96-100).
__device__ __forceinline__ float rope_angle(float theta, int i, int half, int pos) {
    const float e = __fdiv_rn(-(float)i, (float)half);
    const float inv = powf(theta, e);
    return __fmul_rn((float)pos, inv);
}

__device__ __forceinline__ float2 rope_cs_entry(float theta, int i, int half, int pos) {
    const float ang = rope_angle(theta, i, half, pos);
    return make_float2(cosf(ang), sinf(ang));
}

// One rotate-half element, rounded exactly as the reference's separate torch ops:
// x1' = x1*cos - x2*sin, x2' = x2*cos + x1*sin (direct_custom_decode_500.py:103-104).
__device__ __forceinline__ float rope_elem(float x, float partner, float2 cs, bool first_half) {
    return first_half ? __fsub_rn(__fmul_rn(x, cs.x), __fmul_rn(partner, cs.y))
                      : __fadd_rn(__fmul_rn(x, cs.x), __fmul_rn(partner, cs.y));
}

// Below this many tiles per CTA, uniform-length problems get pair-aligned CTA ranges.
constexpr int kAlignBelow = 4;
// Uniform-length pairs of at most this many tiles take one CTA each in split mode.
constexpr int kPairTiles = 8;

// Most CTAs that can hold pieces of one pair: the split grid never exceeds this.
constexpr int kMaxPieces = 320;

template <int D, int NB>
struct Layout {
    static constexpr int G8 = 8 * NB;
    static constexpr int KT = 128 * D;  // bytes of one 64-key tile of K (or V)
    static constexpr int RP = D + 4;    // fp32 pitch of the cross-warp reduction rows
    static constexpr int QP = D + 8;    // fp16 pitch of the rotated-query rows
    // cross-warp reduction rows; reused for the per-piece weights of a pair merge
    static constexpr int RED = kConsumerWarps * G8 * RP > kMaxPieces * G8 ? kConsumerWarps * G8 * RP : kMaxPieces * G8;
    static __host__ __device__ constexpr size_t stage_bytes() { return 2 * (size_t)KT; }
    static __host__ __device__ constexpr size_t fixed_bytes(int stages) {
        return (size_t)stages * stage_bytes() + sizeof(float) * RED +
               sizeof(float) * kConsumerWarps * G8 * 2 + sizeof(float) * G8 * (D + 1) + sizeof(__half) * G8 * QP +
               sizeof(float2) * (D / 2) +
               sizeof(uint64_t) * 2 * stages + sizeof(int) * 8;
    }
    static __host__ size_t smem_bytes(int stages, int B, bool split) {
        return 1024 + fixed_bytes(stages) + (split ? sizeof(int) * (B + 1) + sizeof(int) * 3 * B : 0);
    }
};

// CHECK: the opt-in guard of the early-read contract (FCCI_DECODE_CHECK_EARLY_READ) is
// compiled in; the default instantiation carries none of its code.
template <int D, int NB, bool CHECK>
__global__ void __launch_bounds__(kThreads) decode_attn_kernel(const __grid_constant__ CUtensorMap tmK,
                                                               const __grid_constant__ CUtensorMap tmV,
                                                               const __grid_constant__ CUtensorMap tmK64,
                                                               const __grid_constant__ CUtensorMap tmV64,
                                                               const Params p) {
    using LY = Layout<D, NB>;
    constexpr int G8 = LY::G8;
    constexpr int KT = LY::KT;
    constexpr int RP = LY::RP;
    constexpr int QP = LY::QP;
    constexpr int HALVES = D / 64;
    constexpr int KSTEPS = D / 16;
    constexpr int E = D / 32;  // elements of a row per lane

    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    uint8_t* stages = sm;
    float* red_acc = reinterpret_cast<float*>(stages + (size_t)S * LY::stage_bytes());
    float* red_ml = red_acc + LY::RED;
    float* xo = red_ml + kConsumerWarps * G8 * 2;  // this CTA's normalised piece o [G8, D] (cluster merge)
    float* xl = xo + G8 * D;                       // and its log2-sum-exp [G8]
    __half* qrot = reinterpret_cast<__half*>(xl + G8);
    float2* rope_cs = reinterpret_cast<float2*>(qrot + G8 * QP);
    uint64_t* full = reinterpret_cast<uint64_t*>(rope_cs + D / 2);
    uint64_t* empty = full + S;
    int* misc = reinterpret_cast<int*>(empty + S);
    int* tile_base = misc + 8;        // [B+1] prefix of tiles per sequence (x Hkv), split mode
    int* seqT = tile_base + p.B + 1;  // [B] T_b, split mode
    int* seqL = seqT + p.B;           // [B] keys attended (0 when invalid)
    int* seqBase = seqL + p.B;        // [B] first arena row of the sequence
    volatile int* abort_flag = misc;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int B = p.B, Hkv = p.Hkv, G = p.G;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        misc[0] = 0;
        misc[1] = 0;
        fence_mbar_init();
    }
    if (tid == kConsumerThreads) {
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        prefetch_tmap(&tmK64);
        prefetch_tmap(&tmV64);
    }
    // the next launch may start its own set-up now. Everything below reads what
    // earlier kernels wrote (lengths, queries, new rows, the arena), so wait first;
    // with prefetch_kv the caller guarantees that no kernel still running writes the
    // lengths or the cached rows, and only the reads of q / k_new / v_new (consumers)
    // and the producer's loads after its first S stages wait
    griddep_launch_dependents();
    if (!p.prefetch_kv) griddep_wait();

    // ---- tile line: per-sequence tile counts and their prefix (split mode)
    bool uniform = false;
    if (p.split) {
        int* scratch = reinterpret_cast<int*>(red_acc);  // free until the first segment ends
        const int chunk = (B + kThreads - 1) / kThreads;
        const int lo = tid * chunk, hi = min(B, lo + chunk);
        int local = 0;
        for (int b = lo; b < hi; ++b) {
            const SeqInfo si = seq_info(p, b);
            if (!si.ok && blockIdx.x == 0) set_error(p, FCCI_DEV_ERR_CAPACITY);
            seqT[b] = si.T;
            seqL[b] = si.L;
            seqBase[b] = si.tok_base;
            const int c = tiles_of(si.L) * Hkv;
            tile_base[b + 1] = c;
            local += c;
            if (b == 0) misc[2] = c;  // sequence 0's tile count, for the uniformity test below
        }
        // exclusive prefix of the per-thread sums: shuffle scan per warp, then the
        // 5 warp totals
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += n;
        }
        if (lane == 31) scratch[warp] = incl;
        if (tid == 0) tile_base[0] = 0;
        __syncthreads();
        int run = incl - local;
        for (int w = 0; w < warp; ++w) run += scratch[w];
        for (int b = lo; b < hi; ++b) {
            run += tile_base[b + 1];
            tile_base[b + 1] = run;
        }
        // do all sequences have the same tile count? (misc[2] was written before the
        // barrier above)
        bool same = true;
        for (int b = lo; b < hi; ++b)
            if (tiles_of(seqL[b]) * Hkv != misc[2]) same = false;
        uniform = __syncthreads_and(same) != 0;
    } else if (tid == 0) {
        const SeqInfo si = seq_info(p, blockIdx.x / Hkv);
        if (!si.ok && (blockIdx.x % Hkv) == 0) set_error(p, FCCI_DEV_ERR_CAPACITY);
        misc[3] = si.T;  // the early read the guard below compares with
        misc[4] = si.tok_base;
    }
    __syncthreads();

    // ---- this CTA's tile range
    long long t_begin = 0, t_end = 0, N = 0;
    int b0 = 0, h0 = 0, j0 = 0;
    long long C = gridDim.x;  // CTAs that take tiles: never more than there are tiles
    const int ck = p.cluster_k;  // CTAs per cluster (cluster launch), else 0
    bool cmode = false;          // one cluster per pair, the pair's tiles split over k_eff of its CTAs
    int k_eff = 1;
    if (p.split) {
        N = tile_base[B];
        C = N < (long long)gridDim.x ? N : (long long)gridDim.x;
        // small uniform problems: use C = pairs * k CTAs with k dividing the tiles of a
        // pair, so that every range lies inside one pair (a range straddling two pairs
        // pays a second segment set-up and piece store, which dominate short ranges)
        // and when pairs are short, or many enough to fill half the grid, one CTA per
        // pair: no pieces and no merge, which cost more than the lost parallelism
        const long long P = (long long)B * Hkv;
        if (ck > 1 && uniform && P * ck == (long long)gridDim.x) {
            // cluster launch, uniform tile counts: cluster c serves pair c; CTA r of it takes
            // the r-th of k_eff equal parts of the pair's tiles (k_eff <= tiles, so none is
            // empty); CTAs r >= k_eff only join the cluster barriers
            cmode = true;
            const long long tp = N / P;
            k_eff = (int)(tp < ck ? tp : ck);
            if (tp <= p.solo_tiles) k_eff = 1;
            const long long pr = blockIdx.x / ck;
            const int r = (int)(blockIdx.x % ck);
            C = P * k_eff;
            if (r < k_eff) {
                t_begin = pr * tp + r * tp / k_eff;
                t_end = pr * tp + (r + 1) * tp / k_eff;
            }
        } else if (uniform && P <= (long long)gridDim.x) {
            const long long tp = N / P;
            if (tp <= kPairTiles || (2 * P >= (long long)gridDim.x && tp <= 4 * kPairTiles)) {
                C = P;
            } else if (N < (long long)kAlignBelow * gridDim.x) {
                long long k = (long long)gridDim.x / P;
                if (k > tp) k = tp;
                while (k > 1 && tp % k) --k;
                C = P * k;
            } else if (20 * P * ((long long)gridDim.x / P) >= 17 * (long long)gridDim.x) {
                // C = P * k puts CTA p*k exactly at the start of pair p (N = P * tp), so no
                // range straddles two pairs; taken when it keeps >= 85 % of the grid busy
                // (measured faster than full-grid stream-K down to that fraction)
                C = P * ((long long)gridDim.x / P);
            }
        }
        if (!cmode && (long long)blockIdx.x < C) {
            t_begin = (long long)blockIdx.x * N / C;
            t_end = ((long long)blockIdx.x + 1) * N / C;
        }
        if (t_begin < t_end) {
            int lo = 0, hi = B - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (tile_base[mid] <= t_begin) lo = mid;
                else hi = mid - 1;
            }
            b0 = lo;
            const int tiles = (tile_base[b0 + 1] - tile_base[b0]) / Hkv;
            const int rem = (int)(t_begin - tile_base[b0]);
            h0 = rem / tiles;
            j0 = rem - h0 * tiles;
        }
    } else {
        b0 = blockIdx.x / Hkv;
        h0 = blockIdx.x - b0 * Hkv;
        j0 = 0;
        t_begin = 0;
        t_end = tiles_of(seq_info(p, b0).L);
    }
    const int ntiles = (int)(t_end - t_begin);

    if (warp == kConsumerWarps) {
        // ============================================================ producer
        if (lane == 0 && ntiles > 0) {
            const uint64_t pol = l2_policy_evict_first();
            int b = b0, h = h0, j = j0;
            SeqInfo si = p.split ? SeqInfo{seqT[b], seqL[b], seqBase[b], true} : seq_info(p, b);
            int tiles = tiles_of(si.L);
            int issued = 0;
            for (int it = 0; it < ntiles; ++it) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (it == S && p.prefetch_kv) griddep_wait();
                if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag, kWaitLimitNs)) {
                    *abort_flag = 1;
                    set_error(p, FCCI_DEV_ERR_TIMEOUT);
                    break;
                }
                const int nv = min(kTileKeys, si.L - kTileKeys * j);
                const int ngr = nv > 0 ? (nv + kGroupKeys - 1) / kGroupKeys : 0;
                mbar_arrive_expect_tx(&full[s], (uint32_t)(ngr * 64 * D));
                uint8_t* kdst = stages + (size_t)s * LY::stage_bytes();
                uint8_t* vdst = kdst + KT;
                const int row0 = si.tok_base + kTileKeys * j;
                const int c3 = p.cu_seqlens ? 0 : b;
                if (nv == kTileKeys) {
                    // a full tile: one 64-row box per 64-column half (the same swizzled
                    // layout as four 16-row boxes, in a quarter of the TMA instructions)
#pragma unroll
                    for (int hf = 0; hf < HALVES; ++hf) {
                        tma_load_4d(kdst + hf * kHalfTileBytes, &tmK64, hf * 64, row0, h, c3, &full[s], pol);
                        tma_load_4d(vdst + hf * kHalfTileBytes, &tmV64, hf * 64, row0, h, c3, &full[s], pol);
                    }
                } else {
                    // the last tile of a pair: only the 16-row boxes holding valid keys
                    for (int g = 0; g < ngr; ++g) {
#pragma unroll
                        for (int hf = 0; hf < HALVES; ++hf) {
                            tma_load_4d(kdst + hf * kHalfTileBytes + g * kBoxBytes, &tmK, hf * 64,
                                        row0 + kGroupKeys * g, h, c3, &full[s], pol);
                            tma_load_4d(vdst + hf * kHalfTileBytes + g * kBoxBytes, &tmV, hf * 64,
                                        row0 + kGroupKeys * g, h, c3, &full[s], pol);
                        }
                    }
                }
                ++issued;
                if (++j == tiles) {
                    j = 0;
                    if (++h == Hkv) {
                        h = 0;
                        if (++b < B) {
                            si = p.split ? SeqInfo{seqT[b], seqL[b], seqBase[b], true} : seq_info(p, b);
                            tiles = tiles_of(si.L);
                        }
                    }
                }
            }
            if (*abort_flag) {
                // let copies still in flight land before the CTA can exit
                for (int it = max(0, issued - S); it < issued; ++it) {
                    volatile int never = 0;
                    mbar_wait_bounded(&full[it % S], (uint32_t)(it / S) & 1u, &never, kDrainLimitNs);
                }
            }
        }
    } else {
        // ============================================================ consumers
        const int w = warp;
        const int ctid = tid;  // 0..127
        const int g = lane >> 2, t4 = lane & 3;
        const int mi = lane >> 3;
        const uint32_t swz = (uint32_t)(lane & 7);
        const int rot = p.rotary_dim;
        const int rhalf = rot >> 1;

        float m[NB][2], l[NB][2], acc[NB][KSTEPS][4];
        uint32_t qf[NB][KSTEPS][2];
        int cached_pos = -1;

        int b = b0, h = h0, j = j0;
        SeqInfo si = p.split ? SeqInfo{seqT[b], seqL[b], seqBase[b], true} : seq_info(p, b);
        int tiles = tiles_of(si.L);
        bool seg_start = true;
        int guard_t = 0, guard_base = 0;
        if (p.prefetch_kv) {
            // the RoPE table of the first segment's position depends only on the lengths,
            // which may be read early: build it before waiting for the previous launch
            if (rot > 0 && ntiles > 0) {
                for (int i = ctid; i < 2 * rhalf; i += kConsumerThreads) {
                    const int k = i < rhalf ? i : i - rhalf;
                    const float ang = rope_angle(p.rope_theta, k, rhalf, si.T);
                    if (i < rhalf) rope_cs[k].x = cosf(ang);
                    else rope_cs[k].y = sinf(ang);
                }
                cached_pos = si.T;
                named_bar_sync(kConsumerBar, kConsumerThreads);
            }
            griddep_wait();
            // guard of the early-read contract (opt-in): read the lengths (and sequence
            // offsets) again now that the previous kernel has finished; they are compared
            // with the early values at the end of the kernel
            if (!CHECK) {
            } else if (p.split) {
                if (ctid < B) {
                    guard_t = p.seq_lens ? p.seq_lens[ctid] : p.fixed_len;
                    guard_base = p.cu_seqlens ? p.cu_seqlens[ctid] : 0;
                }
            } else if (ctid == 0) {
                const SeqInfo now = seq_info(p, blockIdx.x / Hkv);
                guard_t = now.T;
                guard_base = now.tok_base;
            }
        }

        for (int it = 0; it < ntiles; ++it) {
            if (seg_start) {
                seg_start = false;
                // ---- rotated queries of the group (shared by the 4 warps): issue the
                //      query loads first (one L2 round trip), then the RoPE table
                const bool write_qrot = (p.q_rot_out != nullptr) && (j == 0);
                const __half* qb = p.q + (int64_t)b * p.q_sb;
                constexpr int NQ = G8 * D / kConsumerThreads;  // element e -> (head, dim)
                __half qx[NQ], qp[NQ];
#pragma unroll
                for (int k = 0; k < NQ; ++k) {
                    const int e = ctid + k * kConsumerThreads;
                    const int hh = e / D;
                    const int d = e - hh * D;
                    qx[k] = qp[k] = __float2half_rn(0.f);
                    if (hh < G) {
                        const __half* qr = qb + (int64_t)(h * G + hh) * p.q_sh;
                        qx[k] = qr[d];
                        if (d < rot) qp[k] = qr[d < rhalf ? d + rhalf : d - rhalf];
                    }
                }
                if (rot > 0 && si.T != cached_pos) {
                    for (int i = ctid; i < 2 * rhalf; i += kConsumerThreads) {
                        const int k = i < rhalf ? i : i - rhalf;
                        const float ang = rope_angle(p.rope_theta, k, rhalf, si.T);
                        if (i < rhalf) rope_cs[k].x = cosf(ang);
                        else rope_cs[k].y = sinf(ang);
                    }
                    cached_pos = si.T;
                    named_bar_sync(kConsumerBar, kConsumerThreads);
                }
#pragma unroll
                for (int k = 0; k < NQ; ++k) {
                    const int e = ctid + k * kConsumerThreads;
                    const int hh = e / D;
                    const int d = e - hh * D;
                    __half val = qx[k];
                    if (hh < G && d < rot) {
                        const bool first = d < rhalf;
                        val = __float2half_rn(
                            rope_elem(__half2float(qx[k]), __half2float(qp[k]), rope_cs[first ? d : d - rhalf], first));
                    }
                    if (write_qrot && hh < G) p.q_rot_out[((int64_t)b * p.Hq + h * G + hh) * D + d] = val;
                    qrot[hh * QP + d] = val;
                }
                named_bar_sync(kConsumerBar, kConsumerThreads);
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
                    for (int kk = 0; kk < KSTEPS; ++kk) {
                        const __half* qrow = qrot + (nb * 8 + g) * QP + 16 * kk + 2 * t4;
                        qf[nb][kk][0] = *reinterpret_cast<const uint32_t*>(qrow);
                        qf[nb][kk][1] = *reinterpret_cast<const uint32_t*>(qrow + 8);
                    }
                    m[nb][0] = m[nb][1] = -INFINITY;
                    l[nb][0] = l[nb][1] = 0.f;
#pragma unroll
                    for (int mb = 0; mb < KSTEPS; ++mb) acc[nb][mb][0] = acc[nb][mb][1] = acc[nb][mb][2] = acc[nb][mb][3] = 0.f;
                }
            }

            const int s = it % S;
            const bool ready = mbar_wait_bounded(&full[s], (uint32_t)(it / S) & 1u, abort_flag, kWaitLimitNs);
            if (!ready && !*abort_flag) {
                *abort_flag = 1;
                set_error(p, FCCI_DEV_ERR_TIMEOUT);
            }
            const int key0 = kTileKeys * j + kGroupKeys * w;
            const int nvw = max(0, min(kGroupKeys, si.L - key0));
            if (ready && nvw > 0) {
                uint8_t* kt = stages + (size_t)s * LY::stage_bytes();
                uint8_t* vt = kt + KT;
                const int row_base = kGroupKeys * w;
                bool wrote = false;
                // ---- append: rotated k_new and v_new become key T of this pair
                if (p.append && si.T >= key0 && si.T < key0 + kGroupKeys) {
                    const int r = si.T - kTileKeys * j;
                    const int d0 = lane * E;
                    const __half* kn = p.k_new + (int64_t)b * p.kn_sb + (int64_t)h * p.kn_sh;
                    const __half* vn = p.v_new + (int64_t)b * p.vn_sb + (int64_t)h * p.vn_sh;
                    __align__(16) __half kr[E];
                    __align__(16) __half vr[E];
#pragma unroll
                    for (int e = 0; e < E; ++e) {
                        const int d = d0 + e;
                        if (d < rot) {
                            const bool first = d < rhalf;
                            const int i = first ? d : d - rhalf;
                            const float x = __half2float(kn[d]);
                            const float xp = __half2float(kn[first ? d + rhalf : d - rhalf]);
                            kr[e] = __float2half_rn(rope_elem(x, xp, rope_cs[i], first));
                        } else {
                            kr[e] = kn[d];
                        }
                        vr[e] = vn[d];
                    }
                    const int64_t bofs_k = p.cu_seqlens ? 0 : (int64_t)b * p.k_sb;
                    const int64_t bofs_v = p.cu_seqlens ? 0 : (int64_t)b * p.v_sb;
                    __half* kdst = p.k_cache + bofs_k + (int64_t)h * p.k_sh + (int64_t)(si.tok_base + si.T) * p.k_st + d0;
                    __half* vdst = p.v_cache + bofs_v + (int64_t)h * p.v_sh + (int64_t)(si.tok_base + si.T) * p.v_st + d0;
                    const uint32_t so = (uint32_t)((d0 >> 6) * kHalfTileBytes + r * 128 +
                                                   ((((d0 & 63) >> 3) ^ (r & 7)) << 4) + (d0 & 7) * 2);
                    if constexpr (E == 2) {
                        *reinterpret_cast<uint32_t*>(kdst) = *reinterpret_cast<uint32_t*>(kr);
                        *reinterpret_cast<uint32_t*>(vdst) = *reinterpret_cast<uint32_t*>(vr);
                        *reinterpret_cast<uint32_t*>(kt + so) = *reinterpret_cast<uint32_t*>(kr);
                        *reinterpret_cast<uint32_t*>(vt + so) = *reinterpret_cast<uint32_t*>(vr);
                    } else if constexpr (E == 4) {
                        *reinterpret_cast<uint2*>(kdst) = *reinterpret_cast<uint2*>(kr);
                        *reinterpret_cast<uint2*>(vdst) = *reinterpret_cast<uint2*>(vr);
                        *reinterpret_cast<uint2*>(kt + so) = *reinterpret_cast<uint2*>(kr);
                        *reinterpret_cast<uint2*>(vt + so) = *reinterpret_cast<uint2*>(vr);
                    } else {
                        *reinterpret_cast<uint4*>(kdst) = *reinterpret_cast<uint4*>(kr);
                        *reinterpret_cast<uint4*>(vdst) = *reinterpret_cast<uint4*>(vr);
                        *reinterpret_cast<uint4*>(kt + so) = *reinterpret_cast<uint4*>(kr);
                        *reinterpret_cast<uint4*>(vt + so) = *reinterpret_cast<uint4*>(vr);
                    }
                    wrote = true;
                }
                // ---- keys past the end: zero their V rows so 0 * garbage cannot make NaN
                if (nvw < kGroupKeys) {
                    const int nz = kGroupKeys - nvw;
                    for (int c = lane; c < nz * HALVES * 8; c += 32) {
                        const int r = row_base + nvw + c / (HALVES * 8);
                        const int rem = c % (HALVES * 8);
                        *reinterpret_cast<uint4*>(vt + (rem >> 3) * kHalfTileBytes + r * 128 + (rem & 7) * 16) =
                            make_uint4(0u, 0u, 0u, 0u);
                    }
                    wrote = true;
                }
                if (wrote) __syncwarp();

                // ---- S^T = K Q^T over the 16 keys of this warp
                const uint32_t kbase = smem_u32(kt);
                const uint32_t vbase = smem_u32(vt);
                const int rowA = row_base + (lane & 7) + ((mi & 1) << 3);
                float s0[NB][4], s1[NB][4];
#pragma unroll
                for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                    for (int c = 0; c < 4; ++c) s0[nb][c] = s1[nb][c] = 0.f;
#pragma unroll
                for (int kk = 0; kk < KSTEPS; ++kk) {
                    const int chunk = 2 * kk + (mi >> 1);
                    const uint32_t addr =
                        kbase + (chunk >> 3) * kHalfTileBytes + rowA * 128 + ((((uint32_t)chunk & 7u) ^ swz) << 4);
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(addr, a0, a1, a2, a3);
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb) {
                        if (kk & 1) mma_16816(s1[nb], a0, a1, a2, a3, qf[nb][kk][0], qf[nb][kk][1]);
                        else mma_16816(s0[nb], a0, a1, a2, a3, qf[nb][kk][0], qf[nb][kk][1]);
                    }
                }
                // ---- online softmax per head column (log2 domain)
                const bool v0 = g < nvw;
                const bool v8 = (g + 8) < nvw;
                uint32_t pb0[NB], pb1[NB];
                float alpha[NB][2];
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    const float x0 = v0 ? (s0[nb][0] + s1[nb][0]) * p.scale_log2 : -INFINITY;
                    const float x1 = v0 ? (s0[nb][1] + s1[nb][1]) * p.scale_log2 : -INFINITY;
                    const float x2 = v8 ? (s0[nb][2] + s1[nb][2]) * p.scale_log2 : -INFINITY;
                    const float x3 = v8 ? (s0[nb][3] + s1[nb][3]) * p.scale_log2 : -INFINITY;
                    float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 4));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 4));
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 8));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 8));
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 16));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 16));
                    const float mn0 = fmaxf(m[nb][0], mx0);
                    const float mn1 = fmaxf(m[nb][1], mx1);
                    alpha[nb][0] = ex2(m[nb][0] - mn0);
                    alpha[nb][1] = ex2(m[nb][1] - mn1);
                    const float p0 = ex2(x0 - mn0), p1 = ex2(x1 - mn1);
                    const float p2 = ex2(x2 - mn0), p3 = ex2(x3 - mn1);
                    l[nb][0] = l[nb][0] * alpha[nb][0] + (p0 + p2);
                    l[nb][1] = l[nb][1] * alpha[nb][1] + (p1 + p3);
                    m[nb][0] = mn0;
                    m[nb][1] = mn1;
                    pb0[nb] = movmatrix_t(pack_half2(p0, p1));
                    pb1[nb] = movmatrix_t(pack_half2(p2, p3));
                }
                // ---- O^T += V^T P^T
                const int rowV = row_base + (lane & 7) + ((mi >> 1) << 3);
#pragma unroll
                for (int mb = 0; mb < KSTEPS; ++mb) {
                    const int chunk = 2 * mb + (mi & 1);
                    const uint32_t addr =
                        vbase + (chunk >> 3) * kHalfTileBytes + rowV * 128 + ((((uint32_t)chunk & 7u) ^ swz) << 4);
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_t(addr, a0, a1, a2, a3);
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb) {
                        acc[nb][mb][0] *= alpha[nb][0];
                        acc[nb][mb][1] *= alpha[nb][1];
                        acc[nb][mb][2] *= alpha[nb][0];
                        acc[nb][mb][3] *= alpha[nb][1];
                        mma_16816(acc[nb][mb], a0, a1, a2, a3, pb0[nb], pb1[nb]);
                    }
                }
                if (wrote) fence_proxy_async_smem();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);

            const bool seg_end = (j == tiles - 1) || (it == ntiles - 1);
            if (seg_end) {
                // ---- merge the 4 warps' states through shared memory
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    float l0 = l[nb][0], l1 = l[nb][1];
                    l0 += __shfl_xor_sync(0xffffffffu, l0, 4);
                    l1 += __shfl_xor_sync(0xffffffffu, l1, 4);
                    l0 += __shfl_xor_sync(0xffffffffu, l0, 8);
                    l1 += __shfl_xor_sync(0xffffffffu, l1, 8);
                    l0 += __shfl_xor_sync(0xffffffffu, l0, 16);
                    l1 += __shfl_xor_sync(0xffffffffu, l1, 16);
                    const int hA = nb * 8 + 2 * t4;
                    if (g == 0) {
                        red_ml[(w * G8 + hA) * 2 + 0] = m[nb][0];
                        red_ml[(w * G8 + hA) * 2 + 1] = l0;
                        red_ml[(w * G8 + hA + 1) * 2 + 0] = m[nb][1];
                        red_ml[(w * G8 + hA + 1) * 2 + 1] = l1;
                    }
                    float* ra = red_acc + (w * G8 + hA) * RP;
#pragma unroll
                    for (int mb = 0; mb < KSTEPS; ++mb) {
                        const int d = 16 * mb + g;
                        ra[d] = acc[nb][mb][0];
                        ra[RP + d] = acc[nb][mb][1];
                        ra[d + 8] = acc[nb][mb][2];
                        ra[RP + d + 8] = acc[nb][mb][3];
                    }
                }
                named_bar_sync(kConsumerBar, kConsumerThreads);

                const int pidx = b * Hkv + h;
                bool whole = true;
                int c0 = 0, c1 = 0;
                if (cmode) {
                    // the piece stays in this CTA's shared memory for the cluster merge
                    whole = (k_eff == 1);
                } else if (p.split) {
                    const long long pfirst = tile_base[b] + (long long)h * tiles;
                    c0 = cta_of_tile(pfirst, N, C);
                    c1 = cta_of_tile(pfirst + tiles - 1, N, C);
                    whole = (c0 == c1);
                }
                const int slot = pidx + blockIdx.x;
                for (int e = ctid * 2; e < G * D; e += 2 * kConsumerThreads) {
                    const int hh = e / D;
                    const int d = e - hh * D;
                    float M = -INFINITY;
#pragma unroll
                    for (int ww = 0; ww < kConsumerWarps; ++ww) M = fmaxf(M, red_ml[(ww * G8 + hh) * 2]);
                    float Ls = 0.f, o0 = 0.f, o1 = 0.f;
                    if (M != -INFINITY) {
#pragma unroll
                        for (int ww = 0; ww < kConsumerWarps; ++ww) {
                            const float sc = ex2(red_ml[(ww * G8 + hh) * 2] - M);
                            Ls += red_ml[(ww * G8 + hh) * 2 + 1] * sc;
                            o0 += red_acc[(ww * G8 + hh) * RP + d] * sc;
                            o1 += red_acc[(ww * G8 + hh) * RP + d + 1] * sc;
                        }
                    }
                    const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
                    if (whole) {
                        store_ctx2(p, (int64_t)b * p.o_sb + (int64_t)(h * G + hh) * p.o_sh + d,
                                   __floats2half2_rn(o0 * inv, o1 * inv));
                    } else if (cmode) {
                        *reinterpret_cast<float2*>(xo + hh * D + d) = make_float2(o0 * inv, o1 * inv);
                        if (d == 0) xl[hh] = Ls > 0.f ? M + __log2f(Ls) : -INFINITY;
                    } else {
                        *reinterpret_cast<float2*>(p.part_o + ((size_t)slot * G + hh) * D + d) =
                            make_float2(o0 * inv, o1 * inv);
                        if (d == 0) p.part_lse[(size_t)slot * G + hh] = Ls > 0.f ? M + __log2f(Ls) : -INFINITY;
                    }
                }
                named_bar_sync(kConsumerBar, kConsumerThreads);
                if (!whole && !cmode) {
                    // ---- the last piece of a cut pair merges every piece's (o, lse).
                    //      The barrier above orders this CTA's piece stores before thread
                    //      0's fence and counter increment (release); the last arriver
                    //      fences again (acquire) before anyone reads the pieces.
                    if (ctid == 0) {
                        __threadfence();
                        const unsigned old = atomicAdd(&p.pair_cnt[pidx], 1u);
                        misc[1] = (old == (unsigned)(c1 - c0)) ? 1 : 0;
                        if (misc[1]) __threadfence();
                    }
                    named_bar_sync(kConsumerBar, kConsumerThreads);
                    if (misc[1]) {
                        // each thread merges its own elements over all pieces with a running
                        // log-sum-exp; loads of PB pieces are in flight at once
                        const int nparts = c1 - c0 + 1;
                        const float* pl = p.part_lse + (size_t)(pidx + c0) * G;
                        const float* po = p.part_o + (size_t)(pidx + c0) * G * D;
                        constexpr int NE = G8 * D / (2 * kConsumerThreads);  // float2 per thread
                        constexpr int PB = NE >= 8 ? 2 : 16 / (2 * NE);     // pieces per batch
                        float Mx[NE], Wt[NE];
                        float2 Ov[NE];
#pragma unroll
                        for (int k = 0; k < NE; ++k) {
                            Mx[k] = -INFINITY;
                            Wt[k] = 0.f;
                            Ov[k] = make_float2(0.f, 0.f);
                        }
                        for (int c = 0; c < nparts; c += PB) {
                            float lv[PB][NE];
                            float2 ov[PB][NE];
#pragma unroll
                            for (int u = 0; u < PB; ++u)
#pragma unroll
                                for (int k = 0; k < NE; ++k) {
                                    const int e = 2 * (ctid + k * kConsumerThreads);
                                    const bool ok = c + u < nparts && e < G * D;
                                    lv[u][k] = ok ? __ldcg(pl + (size_t)(c + u) * G + e / D) : -INFINITY;
                                    ov[u][k] = ok ? __ldcg(reinterpret_cast<const float2*>(po + (size_t)(c + u) * G * D + e))
                                                  : make_float2(0.f, 0.f);
                                }
#pragma unroll
                            for (int u = 0; u < PB; ++u)
#pragma unroll
                                for (int k = 0; k < NE; ++k) {
                                    const float lse = lv[u][k];
                                    if (lse != -INFINITY) {
                                        const float mn = fmaxf(Mx[k], lse);
                                        const float a = ex2(Mx[k] - mn), w = ex2(lse - mn);
                                        Wt[k] = Wt[k] * a + w;
                                        Ov[k].x = Ov[k].x * a + w * ov[u][k].x;
                                        Ov[k].y = Ov[k].y * a + w * ov[u][k].y;
                                        Mx[k] = mn;
                                    }
                                }
                        }
#pragma unroll
                        for (int k = 0; k < NE; ++k) {
                            const int e = 2 * (ctid + k * kConsumerThreads);
                            if (e < G * D) {
                                const int hh = e / D;
                                const int d = e - hh * D;
                                const float inv = Wt[k] > 0.f ? 1.f / Wt[k] : 0.f;
                                store_ctx2(p, (int64_t)b * p.o_sb + (int64_t)(h * G + hh) * p.o_sh + d,
                                           __floats2half2_rn(Ov[k].x * inv, Ov[k].y * inv));
                            }
                        }
                        if (ctid == 0) atomicExch(&p.pair_cnt[pidx], 0u);
                    }
                }
                seg_start = true;
            }

            if (++j == tiles) {
                j = 0;
                if (++h == Hkv) {
                    h = 0;
                    if (++b < B) {
                        si = p.split ? SeqInfo{seqT[b], seqL[b], seqBase[b], true} : seq_info(p, b);
                        tiles = tiles_of(si.L);
                    }
                }
            }
        }
        if (CHECK && p.prefetch_kv) {
            // a value that changed since this CTA read it early means a kernel that was
            // still running wrote it, and the step used a stale value
            bool stale = false;
            if (p.split) {
                if (ctid < B) stale = guard_t != seqT[ctid] || guard_base != seqBase[ctid];
                for (int bb = ctid + kConsumerThreads; bb < B; bb += kConsumerThreads) {
                    const int t_now = p.seq_lens ? p.seq_lens[bb] : p.fixed_len;
                    const int base_now = p.cu_seqlens ? p.cu_seqlens[bb] : 0;
                    stale = stale || t_now != seqT[bb] || base_now != seqBase[bb];
                }
            } else if (ctid == 0) {
                stale = guard_t != misc[3] || guard_base != misc[4];
            }
            if (stale) set_error(p, FCCI_DEV_ERR_EARLY_READ);
        }
    }

    __syncthreads();
    if (ck > 1) {
        // ---- cluster merge. Every CTA of the cluster executes both barriers, whatever its
        //      range (idle CTAs and the non-uniform fallback included), so none waits for a
        //      CTA that does not come. After the first, every piece is visible in its CTA's
        //      shared memory; CTA r merges the r-th slice of the pair's G x D outputs over the
        //      k_eff pieces, in piece order with a running log-sum-exp, reading them through
        //      distributed shared memory. The second keeps every CTA (and so its shared memory)
        //      alive until the others have read it.
        cluster_sync_all();
        const int r = (int)(blockIdx.x % ck);
        if (cmode && k_eff > 1 && r < k_eff && warp < kConsumerWarps) {
            const int pr = (int)(blockIdx.x / ck);
            const int mb = pr / Hkv, mh = pr - mb * Hkv;
            const int64_t obm = (int64_t)mb * p.o_sb + (int64_t)(mh * G) * p.o_sh;
            const int E = G * D;
            const int lo = (int)((long long)r * E / k_eff), hi = (int)((long long)(r + 1) * E / k_eff);
            const uint32_t xo_s = smem_u32(xo), xl_s = smem_u32(xl);
            for (int e = lo + tid; e < hi; e += kConsumerThreads) {
                const int hh = e / D;
                const int d = e - hh * D;
                float lv[kMaxCluster], ov[kMaxCluster];
#pragma unroll
                for (int c = 0; c < kMaxCluster; ++c) {
                    if (c < k_eff) {
                        lv[c] = ld_cluster_f32(cluster_map(xl_s + 4u * hh, (uint32_t)c));
                        ov[c] = ld_cluster_f32(cluster_map(xo_s + 4u * e, (uint32_t)c));
                    }
                }
                float Mx = -INFINITY, Wt = 0.f, Ov = 0.f;
#pragma unroll
                for (int c = 0; c < kMaxCluster; ++c) {
                    if (c < k_eff && lv[c] != -INFINITY) {
                        const float mn = fmaxf(Mx, lv[c]);
                        const float a = ex2(Mx - mn), wgt = ex2(lv[c] - mn);
                        Wt = Wt * a + wgt;
                        Ov = Ov * a + wgt * ov[c];
                        Mx = mn;
                    }
                }
                const float inv = Wt > 0.f ? 1.f / Wt : 0.f;
                store_ctx1(p, obm + (int64_t)hh * p.o_sh + d, __float2half_rn(Ov * inv));
            }
        }
        cluster_sync_all();
    }
    // ---- ctx exchange: every thread's stores to the peers become visible system-wide
    //      before its CTA counts in below
    if (p.n_peers > 0) {
        fence_acq_rel_sys();
        __syncthreads();
    }
    // ---- the last CTA: device-side seq_len advance (once every CTA has read the
    //      lengths) and the exchange's flag raise (once every CTA has stored its ctx)
    if (p.advance || p.n_peers > 0) {
        if (tid == 0) {
            __threadfence();
            const unsigned old = atomicAdd(p.done_cnt, 1u);
            misc[1] = (old == gridDim.x - 1) ? 1 : 0;
        }
        __syncthreads();
        if (misc[1]) {
            __threadfence();
            if (p.advance) {
                for (int b = tid; b < B; b += kThreads) {
                    const SeqInfo si = seq_info(p, b);
                    if (si.ok) p.seq_lens[b] = si.T + 1;
                }
            }
            if (tid == 0) {
                if (p.n_peers > 0) {
                    const uint32_t e = *p.xepoch + 1u;
                    *p.xepoch = e;
                    fence_acq_rel_sys();
#pragma unroll
                    for (int i = 0; i < FCCI_MAX_PEERS; ++i)
                        if (i < p.n_peers) st_release_sys(p.peer_flags[i] + p.xrank, e);
                    st_release_sys(p.xflags + p.xrank, e);
                }
                atomicExch(p.done_cnt, 0u);
            }
        }
    }
}

// RoPE(q, k_new) at T_b and append of (k_rot, v_new); one CTA per sequence.
template <int D>
__global__ void __launch_bounds__(128) rope_append_kernel(const Params p) {
    constexpr int E = D / 32;
    __shared__ float2 cs[D / 2];
    const int b = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const SeqInfo si = seq_info(p, b);
    const int rot = p.rotary_dim, rhalf = rot >> 1;
    if (!si.ok) {
        if (tid == 0) set_error(p, FCCI_DEV_ERR_CAPACITY);
        return;
    }
    for (int i = tid; i < rhalf; i += blockDim.x) cs[i] = rope_cs_entry(p.rope_theta, i, rhalf, si.T);
    __syncthreads();
    for (int h = warp; h < p.Hkv; h += blockDim.x / 32) {
        const __half* kn = p.k_new + (int64_t)b * p.kn_sb + (int64_t)h * p.kn_sh;
        const __half* vn = p.v_new + (int64_t)b * p.vn_sb + (int64_t)h * p.vn_sh;
        const int64_t bofs_k = p.cu_seqlens ? 0 : (int64_t)b * p.k_sb;
        const int64_t bofs_v = p.cu_seqlens ? 0 : (int64_t)b * p.v_sb;
        __half* kd = p.k_cache + bofs_k + (int64_t)h * p.k_sh + (int64_t)(si.tok_base + si.T) * p.k_st;
        __half* vd = p.v_cache + bofs_v + (int64_t)h * p.v_sh + (int64_t)(si.tok_base + si.T) * p.v_st;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int d = lane * E + e;
            __half r;
            if (d < rot) {
                const bool first = d < rhalf;
                const int i = first ? d : d - rhalf;
                r = __float2half_rn(rope_elem(__half2float(kn[d]), __half2float(kn[first ? d + rhalf : d - rhalf]),
                                              cs[i], first));
            } else {
                r = kn[d];
            }
            kd[d] = r;
            vd[d] = vn[d];
        }
        if (p.q_rot_out) {
            for (int hh = 0; hh < p.G; ++hh) {
                const int hq = h * p.G + hh;
                const __half* qr = p.q + (int64_t)b * p.q_sb + (int64_t)hq * p.q_sh;
                __half* qo = p.q_rot_out + ((int64_t)b * p.Hq + hq) * D;
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int d = lane * E + e;
                    if (d < rot) {
                        const bool first = d < rhalf;
                        const int i = first ? d : d - rhalf;
                        qo[d] = __float2half_rn(rope_elem(__half2float(qr[d]),
                                                          __half2float(qr[first ? d + rhalf : d - rhalf]), cs[i], first));
                    } else {
                        qo[d] = qr[d];
                    }
                }
            }
        }
    }
    __syncthreads();
    if (p.advance && tid == 0) p.seq_lens[b] = si.T + 1;
}

// ------------------------------------------------------------------ host side

static Tuning g_tuning;  // 0 = automatic

Tuning& tuning() { return g_tuning; }

int device_sm_count(int dev) {
    static std::mutex mu;
    static int cache[128] = {0};
    if (dev < 0 || dev >= 128) return 0;
    std::lock_guard<std::mutex> lk(mu);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        cache[dev] = n;
    }
    return cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }();
    return fn;
}

// fp16 tensor map with 128-byte swizzle. dims[0] is the contiguous dimension;
// stride_bytes[i] is the byte stride of dims[i + 1]. A stride of an extent-1
// dimension is never used by a load; it is replaced by the packed value so the
// encoder's alignment checks pass.
int encode_f16_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const int64_t* stride_bytes,
                     const uint32_t* box) {
    auto fn = encode_fn();
    if (!fn || rank < 1 || rank > 5) return FCCI_ETMAP;
    cuuint64_t d[5], st[4];
    cuuint32_t bx[5], estr[5];
    int64_t prev = 2;  // bytes per element: the stride of dimension 0
    for (int i = 0; i < rank; ++i) {
        d[i] = (cuuint64_t)dims[i];
        bx[i] = box[i];
        estr[i] = 1;
        if (i > 0) {
            int64_t sb = stride_bytes[i - 1];
            if (dims[i] == 1) sb = ((prev * (int64_t)dims[i - 1] + 15) / 16) * 16;
            st[i - 1] = (cuuint64_t)sb;
            prev = sb;
        }
    }
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base), d, st, bx, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FCCI_OK : FCCI_ETMAP;
}

// 4-D map (head_dim, token, kv head, sequence) over an fp16 arena; 64-column boxes of
// box_rows keys. Strides in elements.
static int encode_kv_map(CUtensorMap* map, const void* base, int D, int64_t tokens, int Hkv, int Bdim, int64_t st,
                         int64_t sh, int64_t sb, int box_rows = kGroupKeys) {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)tokens, (uint64_t)Hkv, (uint64_t)Bdim};
    const int64_t sbytes[3] = {st * 2, sh * 2, sb * 2};
    const uint32_t box[4] = {64, (uint32_t)box_rows, 1, 1};
    return encode_f16_sw128(map, base, 4, dims, sbytes, box);
}

WorkspaceLayout workspace_layout(int B, int Hq, int Hkv, int D, int grid) {
    WorkspaceLayout w;
    const int G = Hq / (Hkv > 0 ? Hkv : 1);
    const size_t P = (size_t)B * Hkv;
    const size_t slots = P + (size_t)grid;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    w.err = 0;
    w.done = 4;
    w.pair_cnt = 256;
    w.part_lse = w.pair_cnt + up(P * 4);
    w.part_o = w.part_lse + up(slots * G * 4);
    w.total = w.part_o + up(slots * G * (size_t)D * 4);
    w.zero_bytes = w.part_lse;  // header + counters
    return w;
}

int max_grid(int dev) { return device_sm_count(dev) * kMaxCtasPerSm; }

// Can `clusters` clusters of k CTAs of this kernel (with `smem` bytes of dynamic shared
// memory each) be resident on device `dev` at once? Answered by the occupancy API and
// remembered per (device, k, shared memory).
template <int D, int NB, bool CHECK>
static bool clusters_fit(int k, long long clusters, size_t smem, int dev, bool non_portable_ok) {
    if (k > 8 && !non_portable_ok) return false;
    static std::mutex mu;
    static std::map<std::tuple<int, int, size_t>, int> cache;  // one per instantiation
    const auto key = std::make_tuple(dev, k, smem);
    int n = -1;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) n = it->second;
    }
    if (n < 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(k * (clusters > 0 ? clusters : 1)));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute a[1];
        a[0].id = cudaLaunchAttributeClusterDimension;
        a[0].val.clusterDim.x = (unsigned)k;
        a[0].val.clusterDim.y = 1;
        a[0].val.clusterDim.z = 1;
        cfg.attrs = a;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, decode_attn_kernel<D, NB, CHECK>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        std::lock_guard<std::mutex> lk(mu);
        cache[key] = n;
    }
    return (long long)n >= clusters;
}

template <int D, int NB, bool CHECK>
static int launch_decode_t(Params prm, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mk64,
                           const CUtensorMap& mv64, int grid, cudaStream_t st,
                           int dev) {
    using LY = Layout<D, NB>;
    static std::once_flag flags[128];
    static cudaError_t attr_err[128];
    static bool non_portable[128];
    if (dev < 0 || dev >= 128) return FCCI_EINVAL;
    std::call_once(flags[dev], [&]() {
        attr_err[dev] = cudaFuncSetAttribute(decode_attn_kernel<D, NB, CHECK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024);
        // clusters of more than 8 CTAs need this opt-in; without it they are not used
        non_portable[dev] =
            cudaFuncSetAttribute(decode_attn_kernel<D, NB, CHECK>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
            cudaSuccess;
        if (!non_portable[dev]) cudaGetLastError();
    });
    if (attr_err[dev] != cudaSuccess) return set_cuda_status(attr_err[dev]);
    const size_t smem = LY::smem_bytes(prm.stages, prm.B, prm.split != 0);
    if (prm.split) {
        // a persistent grid larger than what fits at once would run in waves: cap it
        // by the resident CTAs per SM of this instantiation (its registers can allow
        // fewer than the shared-memory estimate of the launch shape)
        static std::mutex mu;
        static size_t occ_smem[128];
        static int occ_val[128];
        int occ = 0;
        {
            std::lock_guard<std::mutex> lk(mu);
            if (occ_val[dev] > 0 && occ_smem[dev] == smem) occ = occ_val[dev];
        }
        if (occ == 0) {
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_attn_kernel<D, NB, CHECK>, kThreads, smem) !=
                cudaSuccess) {
                cudaGetLastError();
                occ = 0;
            }
            std::lock_guard<std::mutex> lk(mu);
            occ_smem[dev] = smem;
            occ_val[dev] = occ;
        }
        if (occ >= 1 && grid > device_sm_count(dev) * occ) grid = device_sm_count(dev) * occ;
        // few (sequence, kv head) pairs: one cluster of k CTAs per pair, k as large as the
        // resident grid allows (every cluster resident at once, so no second wave)
        prm.cluster_k = 0;
        const long long P = (long long)prm.B * prm.Hkv;
        const int maxk = g_tuning.max_cluster > 0 ? g_tuning.max_cluster : kMaxCluster;
        // a batched arena bounds every pair's tiles by its capacity: no cluster needs
        // more CTAs than that (the packed layout gives no per-sequence bound here)
        const long long cap_tiles = prm.cu_seqlens ? (long long)kMaxCluster : ((long long)prm.capacity + kTileKeys - 1) / kTileKeys;
        const long long min_tiles = g_tuning.cluster_min_tiles > 0 ? g_tuning.cluster_min_tiles : kClusterMinTiles;
        if (maxk >= 2 && 2 * P <= (long long)grid && cap_tiles >= 2) {
            long long k = (long long)grid / P;
            if (k > maxk) k = maxk;
            if (k > cap_tiles / min_tiles) k = cap_tiles / min_tiles;
            while (k >= 2 && !clusters_fit<D, NB, CHECK>((int)k, P, smem, dev, non_portable[dev])) --k;
            if (k >= 2) {
                prm.cluster_k = (int)k;
                prm.solo_tiles = g_tuning.solo_tiles >= 0 ? g_tuning.solo_tiles : kSoloTiles;
                grid = (int)(P * k);
            }
        }
    }
    return launch_pdl_cluster(decode_attn_kernel<D, NB, CHECK>, dim3(grid), dim3(kThreads), smem, st, prm.cluster_k, mk, mv,
                              mk64, mv64, prm);
}

// Launch shape: persistent CTAs per SM and pipeline stages per CTA. Two CTAs
// per SM hide the consumers' per-tile latency (8 consumer warps per SM), so they
// are preferred whenever two stages fit in half of the SM's shared memory.
struct Shape {
    int stages, ctas_per_sm;
};

static Shape pick_shape(int D, int NB, int B, bool split) {
    auto bytes = [&](int s) -> size_t {
        switch (D * 10 + NB) {
            case 641: return Layout<64, 1>::smem_bytes(s, B, split);
            case 642: return Layout<64, 2>::smem_bytes(s, B, split);
            case 1281: return Layout<128, 1>::smem_bytes(s, B, split);
            case 1282: return Layout<128, 2>::smem_bytes(s, B, split);
            case 2561: return Layout<256, 1>::smem_bytes(s, B, split);
            default: return (size_t)1 << 40;
        }
    };
    const size_t sm_bytes = 228 * 1024, per_cta_reserved = 1024, cta_max = 227 * 1024;
    const int want_stages = g_tuning.stages > 0 ? g_tuning.stages : 4;
    for (int ctas = (g_tuning.ctas_per_sm > 0 ? g_tuning.ctas_per_sm : kMaxCtasPerSm); ctas >= 1; --ctas) {
        size_t budget = sm_bytes / ctas - per_cta_reserved;
        if (budget > cta_max) budget = cta_max;
        int s = want_stages;
        while (s >= 2 && bytes(s) > budget) --s;
        if (s >= 2) return {s, ctas};
        if (g_tuning.ctas_per_sm > 0) break;
    }
    return {0, 0};
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Validates a descriptor; on failure records the reason (fcci_last_error_string)
// and returns its FCCI_E* code.
static int fill_params(const fcci_decode_desc* d, Params& p, bool attention) {
    auto bad = [](int code, const char* why) { return set_status(code, why); };
    if (!d) return bad(FCCI_EINVAL, "descriptor is NULL");
    if (d->abi_version != 1 && d->abi_version != FCCI_DECODE_ABI_VERSION)
        return bad(FCCI_EINVAL, "abi_version mismatch");
    const uint32_t flags = d->abi_version >= 2 ? d->flags : 0u;
    if (flags & ~(FCCI_DECODE_PREFETCH_KV | FCCI_DECODE_CHECK_EARLY_READ)) return bad(FCCI_EINVAL, "unknown bits in flags");
    if (d->B <= 0 || d->Hq <= 0 || d->Hkv <= 0 || d->Hq % d->Hkv != 0)
        return bad(FCCI_EINVAL, "B, Hq, Hkv must be positive and Hq a multiple of Hkv");
    if (d->D != 64 && d->D != 128 && d->D != 256) return bad(FCCI_EUNSUPPORTED, "unsupported head_dim (64, 128 or 256)");
    if (!d->q || !d->k_cache || !d->v_cache) return bad(FCCI_EINVAL, "q, k_cache and v_cache are required");
    if (attention && !d->out) return bad(FCCI_EINVAL, "out is required");
    if ((d->k_new == nullptr) != (d->v_new == nullptr)) return bad(FCCI_EINVAL, "k_new and v_new go together");
    if (!attention && !d->k_new) return bad(FCCI_EINVAL, "k_new/v_new are required");
    if (d->capacity <= 0) return bad(FCCI_EINVAL, "capacity must be positive");
    if (d->rotary_dim < 0 || d->rotary_dim > d->D || (d->rotary_dim & 1))
        return bad(FCCI_EINVAL, "rotary_dim must be even and within head_dim");
    if (d->advance && !d->seq_lens) return bad(FCCI_EINVAL, "advance needs seq_lens");
    if (!d->seq_lens && d->fixed_len < 0) return bad(FCCI_EINVAL, "fixed_len must be non-negative");
    if (attention) {
        if (!aligned16(d->k_cache) || !aligned16(d->v_cache)) return bad(FCCI_EINVAL, "arena base not 16-byte aligned");
        const int64_t ks[6] = {d->k_stride_t, d->k_stride_h, d->k_stride_b, d->v_stride_t, d->v_stride_h, d->v_stride_b};
        for (int i = 0; i < 6; ++i)
            if (ks[i] < 0 || (ks[i] & 7)) return bad(FCCI_EINVAL, "arena strides must be non-negative multiples of 8");
        if (d->k_stride_t == 0 || d->v_stride_t == 0) return bad(FCCI_EINVAL, "arena token stride is zero");
        if ((reinterpret_cast<uintptr_t>(d->out) & 3) || (d->out_stride_h & 1) || (d->out_stride_b & 1))
            return bad(FCCI_EINVAL, "out must be 4-byte aligned with even strides");
    }
    const int E = d->D / 32;
    if (d->k_new) {
        // append path stores E contiguous halves per lane
        const uintptr_t a = (uintptr_t)2 * E - 1;
        if (((uintptr_t)d->k_cache & a) || ((uintptr_t)d->v_cache & a) || (d->k_stride_t * 2 & (int64_t)a) ||
            (d->k_stride_h * 2 & (int64_t)a) || (d->k_stride_b * 2 & (int64_t)a) || (d->v_stride_t * 2 & (int64_t)a) ||
            (d->v_stride_h * 2 & (int64_t)a) || (d->v_stride_b * 2 & (int64_t)a))
            return bad(FCCI_EINVAL, "arena rows misaligned for the append");
    }
    memset(&p, 0, sizeof(p));
    p.q = static_cast<const __half*>(d->q);
    p.q_sb = d->q_stride_b;
    p.q_sh = d->q_stride_h;
    p.k_new = static_cast<const __half*>(d->k_new);
    p.kn_sb = d->k_new_stride_b;
    p.kn_sh = d->k_new_stride_h;
    p.v_new = static_cast<const __half*>(d->v_new);
    p.vn_sb = d->v_new_stride_b;
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
    p.cu_seqlens = d->cu_seqlens;
    p.seq_lens = d->seq_lens;
    p.fixed_len = d->fixed_len;
    p.out = static_cast<__half*>(d->out);
    p.o_sb = d->out_stride_b;
    p.o_sh = d->out_stride_h;
    p.q_rot_out = static_cast<__half*>(d->q_rot_out);
    p.scale_log2 = d->scale * 1.4426950408889634f;
    p.rope_theta = d->rope_theta;
    p.rotary_dim = d->rotary_dim;
    p.advance = d->advance;
    p.append = d->k_new ? 1 : 0;
    p.split = d->split ? 1 : 0;
    p.prefetch_kv = (flags & FCCI_DECODE_PREFETCH_KV) ? 1 : 0;
    p.check_early = (flags & FCCI_DECODE_CHECK_EARLY_READ) ? 1 : 0;
    p.B = d->B;
    p.Hq = d->Hq;
    p.Hkv = d->Hkv;
    p.G = d->Hq / d->Hkv;
    return FCCI_OK;
}

static void bind_workspace(Params& p, void* ws, const WorkspaceLayout& L) {
    uint8_t* base = static_cast<uint8_t*>(ws);
    p.err = reinterpret_cast<uint32_t*>(base + L.err);
    p.done_cnt = reinterpret_cast<uint32_t*>(base + L.done);
    p.pair_cnt = reinterpret_cast<uint32_t*>(base + L.pair_cnt);
    p.part_lse = reinterpret_cast<float*>(base + L.part_lse);
    p.part_o = reinterpret_cast<float*>(base + L.part_o);
}

int decode_attention(const fcci_decode_desc* d, cudaStream_t stream, const fcci_ctx_exchange* ex) {
    Params p;
    int rc = fill_params(d, p, true);
    if (rc) return rc;
    if (ex) {
        p.n_peers = ex->n_peers;
        p.xrank = ex->rank;
        for (int i = 0; i < ex->n_peers; ++i) {
            p.peer_out[i] = static_cast<__half*>(ex->peer_out[i]);
            p.peer_flags[i] = ex->peer_flags[i];
        }
        p.xflags = ex->flags;
        p.xepoch = ex->epoch;
    }
    const int G = p.G;
    const int NB = G <= 8 ? 1 : (G <= 16 ? 2 : 0);
    if (NB == 0 || (d->D == 256 && NB == 2))
        return set_status(FCCI_EUNSUPPORTED, "fcci_decode_attention: query group size unsupported");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_status(cudaGetLastError());
    const int sms = device_sm_count(dev);
    if (sms <= 0) return set_status(FCCI_ECUDA, "fcci_decode_attention: no device");
    const bool split = p.split != 0;
    const int64_t pairs = (int64_t)p.B * p.Hkv;
    const Shape shape = pick_shape(d->D, NB, p.B, split);
    if (shape.stages == 0) return set_status(FCCI_EUNSUPPORTED, "fcci_decode_attention: batch too large for shared memory");
    p.stages = shape.stages;
    int grid;
    if (split) {
        grid = sms * shape.ctas_per_sm;
        if (grid > kMaxPieces) grid = kMaxPieces;
    } else {
        if (pairs > 0x7fffffff) return set_status(FCCI_EINVAL, "fcci_decode_attention: too many pairs");
        grid = (int)pairs;
    }
    const bool need_ws = split || p.advance || p.n_peers > 0;
    if (need_ws) {
        const WorkspaceLayout L = workspace_layout(p.B, p.Hq, p.Hkv, d->D, sms * kMaxCtasPerSm);
        if (!d->workspace || d->workspace_bytes < L.total)
            return set_status(FCCI_EWORKSPACE, "fcci_decode_attention: workspace missing or too small");
        bind_workspace(p, d->workspace, L);
    } else if (d->workspace) {
        const WorkspaceLayout L = workspace_layout(p.B, p.Hq, p.Hkv, d->D, sms * kMaxCtasPerSm);
        if (d->workspace_bytes >= L.total) bind_workspace(p, d->workspace, L);
    }

    CUtensorMap mk, mv;
    const int Bdim = p.cu_seqlens ? 1 : p.B;
    CUtensorMap mk64, mv64;
    rc = encode_kv_map(&mk, p.k_cache, d->D, p.capacity, p.Hkv, Bdim, p.k_st, p.k_sh, p.k_sb);
    if (!rc) rc = encode_kv_map(&mv, p.v_cache, d->D, p.capacity, p.Hkv, Bdim, p.v_st, p.v_sh, p.v_sb);
    if (!rc) rc = encode_kv_map(&mk64, p.k_cache, d->D, p.capacity, p.Hkv, Bdim, p.k_st, p.k_sh, p.k_sb, kTileKeys);
    if (!rc) rc = encode_kv_map(&mv64, p.v_cache, d->D, p.capacity, p.Hkv, Bdim, p.v_st, p.v_sh, p.v_sb, kTileKeys);
    if (rc) return set_status(rc, "fcci_decode_attention: cuTensorMapEncodeTiled rejected the arena layout");

    const bool check = p.check_early && p.prefetch_kv;
    switch (d->D * 10 + NB) {
        case 641: return check ? launch_decode_t<64, 1, true>(p, mk, mv, mk64, mv64, grid, stream, dev)
                               : launch_decode_t<64, 1, false>(p, mk, mv, mk64, mv64, grid, stream, dev);
        case 642: return check ? launch_decode_t<64, 2, true>(p, mk, mv, mk64, mv64, grid, stream, dev)
                               : launch_decode_t<64, 2, false>(p, mk, mv, mk64, mv64, grid, stream, dev);
        case 1281: return check ? launch_decode_t<128, 1, true>(p, mk, mv, mk64, mv64, grid, stream, dev)
                                : launch_decode_t<128, 1, false>(p, mk, mv, mk64, mv64, grid, stream, dev);
        case 1282: return check ? launch_decode_t<128, 2, true>(p, mk, mv, mk64, mv64, grid, stream, dev)
                                : launch_decode_t<128, 2, false>(p, mk, mv, mk64, mv64, grid, stream, dev);
        case 2561: return check ? launch_decode_t<256, 1, true>(p, mk, mv, mk64, mv64, grid, stream, dev)
                                : launch_decode_t<256, 1, false>(p, mk, mv, mk64, mv64, grid, stream, dev);
        default: return set_status(FCCI_EUNSUPPORTED, "fcci_decode_attention: unsupported head_dim");
    }
}

int rope_append(const fcci_decode_desc* d, cudaStream_t stream) {
    Params p;
    int rc = fill_params(d, p, false);
    if (rc) return rc;
    if (d->workspace) {
        int dev = 0;
        cudaGetDevice(&dev);
        const WorkspaceLayout L = workspace_layout(p.B, p.Hq, p.Hkv, d->D, max_grid(dev));
        if (d->workspace_bytes >= L.total) bind_workspace(p, d->workspace, L);
    }
    switch (d->D) {
        case 64: rope_append_kernel<64><<<p.B, 128, 0, stream>>>(p); break;
        case 128: rope_append_kernel<128><<<p.B, 128, 0, stream>>>(p); break;
        case 256: rope_append_kernel<256><<<p.B, 128, 0, stream>>>(p); break;
        default: return set_status(FCCI_EUNSUPPORTED, "fcci_rope_append: unsupported head_dim");
    }
    count_launch();
    return set_cuda_status(cudaGetLastError());
}

}  // namespace fcci
