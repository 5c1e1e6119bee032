// Python module `attn_varlen`: the reference's surface (forward, from
// custom_kernels/attn_varlen.cpp:16-49) plus allocation-free and batched entry
// points, all launching the sm_100a kernels of libfcci_decode.so on the current
// CUDA stream.
#include <pybind11/stl.h>

#include <string>
#include <vector>

#include "binding_common.h"
#include "fcci_exchange.h"
#include "fcci_prefill.h"

using namespace fcci_py;

namespace {

// Shared body of forward / forward_out: attention of every head over the first
// seq_len keys of k/v (honouring their real strides).
void run_forward(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in, int64_t seq_len,
                 double scale, at::Tensor& out, const c10::optional<at::Tensor>& workspace, bool may_allocate) {
    const int64_t H = q_in.size(0), D = q_in.size(1);
    at::Tensor q = q_in.stride(1) == 1 ? q_in : q_in.contiguous();
    at::Tensor k = tma_ready(k_in);
    at::Tensor v = tma_ready(v_in);
    fcci_decode_desc d = blank_desc();
    d.B = 1;
    d.Hq = (int32_t)H;
    d.Hkv = (int32_t)H;
    d.D = (int32_t)D;
    d.q = q.data_ptr();
    d.q_stride_b = H * q.stride(0);
    d.q_stride_h = q.stride(0);
    d.k_cache = k.data_ptr();
    d.k_stride_b = k.size(0) * k.stride(0);
    d.k_stride_h = k.stride(0);
    d.k_stride_t = k.stride(1);
    d.v_cache = v.data_ptr();
    d.v_stride_b = v.size(0) * v.stride(0);
    d.v_stride_h = v.stride(0);
    d.v_stride_t = v.stride(1);
    d.capacity = (int32_t)k.size(1);
    d.fixed_len = (int32_t)seq_len;
    d.out = out.data_ptr();
    d.out_stride_b = H * out.stride(0);
    d.out_stride_h = out.stride(0);
    d.scale = (float)scale;
    d.rotary_dim = 0;
    at::Tensor ws;
    if (workspace.has_value() && workspace->defined()) {
        ws = *workspace;
    } else if (may_allocate && seq_len > 256) {
        ws = cached_workspace(1, H, H, D, q.device());
    }
    if (ws.defined()) {
        bind_workspace(d, ws);
        d.split = 1;
    }
    check_rc(fcci_decode_attention(&d, current_stream()), "attn_varlen.forward");
}

void check_forward_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t seq_len) {
    // same preconditions and messages as attn_varlen.cpp:23-30
    TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "q,k,v must be CUDA");
    TORCH_CHECK(q.dtype() == at::kHalf && k.dtype() == at::kHalf && v.dtype() == at::kHalf, "q,k,v must be fp16");
    TORCH_CHECK(q.dim() == 2 && k.dim() == 3 && v.dim() == 3, "shapes: q[H,D], k[H,T,D], v[H,T,D]");
    const int64_t H = q.size(0), D = q.size(1);
    TORCH_CHECK(k.size(0) == H && v.size(0) == H, "head mismatch");
    TORCH_CHECK(k.size(2) == D && v.size(2) == D, "head_dim mismatch");
    TORCH_CHECK(seq_len >= 1 && seq_len <= k.size(1), "invalid seq_len");
    TORCH_CHECK(v.size(1) >= seq_len, "invalid seq_len");
    TORCH_CHECK(D == 64 || D == 128 || D == 256, "head_dim must be 64, 128 or 256 (got ", D, ")");
}

at::Tensor forward(at::Tensor q, at::Tensor k, at::Tensor v, int64_t seq_len, double scale) {
    check_forward_args(q, k, v, seq_len);
    c10::cuda::CUDAGuard guard(q.device());
    at::Tensor ctx = at::empty({q.size(0), q.size(1)}, q.options());
    run_forward(q, k, v, seq_len, scale, ctx, c10::nullopt, true);
    return ctx;
}

void forward_out(at::Tensor q, at::Tensor k, at::Tensor v, int64_t seq_len, double scale, at::Tensor out,
                 c10::optional<at::Tensor> workspace) {
    check_forward_args(q, k, v, seq_len);
    check_half_cuda(out, "out");
    TORCH_CHECK(out.dim() == 2 && out.size(0) == q.size(0) && out.size(1) == q.size(1), "out must be [H, D]");
    TORCH_CHECK(out.stride(1) == 1, "out must have a contiguous last dimension");
    c10::cuda::CUDAGuard guard(q.device());
    run_forward(q, k, v, seq_len, scale, out, workspace, false);
}

// Batched / varlen decode step over a persistent arena.
void decode(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor out, c10::optional<at::Tensor> k_new,
            c10::optional<at::Tensor> v_new, c10::optional<at::Tensor> seq_lens, c10::optional<at::Tensor> cu_seqlens,
            int64_t fixed_len, double scale, double rope_theta, int64_t rotary_dim, bool advance,
            c10::optional<at::Tensor> workspace, c10::optional<at::Tensor> q_rot_out, bool split, bool prefetch_kv,
            bool check_early_read,
            const std::vector<uint64_t>& peer_out, const std::vector<uint64_t>& peer_flags, uint64_t exch_flags,
            uint64_t exch_epoch, int64_t exch_rank) {
    check_half_cuda(q, "q");
    check_half_cuda(k_cache, "k_cache");
    check_half_cuda(v_cache, "v_cache");
    check_half_cuda(out, "out");
    TORCH_CHECK(q.dim() == 3, "q must be [B, Hq, D]");
    TORCH_CHECK(q.stride(2) == 1, "q must have a contiguous last dimension");
    const int64_t B = q.size(0), Hq = q.size(1), D = q.size(2);
    const bool packed = cu_seqlens.has_value() && cu_seqlens->defined();
    int64_t Hkv, cap;
    if (packed) {
        TORCH_CHECK(k_cache.dim() == 3 && v_cache.dim() == 3, "packed arena must be [Hkv, total_tokens, D]");
        Hkv = k_cache.size(0);
        cap = k_cache.size(1);
        check_int32_cuda(*cu_seqlens, "cu_seqlens");
        TORCH_CHECK(cu_seqlens->numel() == B + 1, "cu_seqlens must have B+1 entries");
    } else {
        TORCH_CHECK(k_cache.dim() == 4 && v_cache.dim() == 4, "arena must be [B, Hkv, capacity, D]");
        TORCH_CHECK(k_cache.size(0) == B, "arena batch mismatch");
        Hkv = k_cache.size(1);
        cap = k_cache.size(2);
    }
    TORCH_CHECK(v_cache.sizes() == k_cache.sizes(), "k_cache and v_cache shapes differ");
    TORCH_CHECK(k_cache.size(-1) == D, "head_dim mismatch");
    TORCH_CHECK(Hkv > 0 && Hq % Hkv == 0, "Hq must be a multiple of Hkv");
    TORCH_CHECK(tma_compatible(k_cache) && tma_compatible(v_cache),
                "arena must have a contiguous head_dim, 16-byte aligned base and strides");
    TORCH_CHECK(out.dim() == 3 && out.size(0) == B && out.size(1) == Hq && out.size(2) == D && out.stride(2) == 1,
                "out must be [B, Hq, D] with a contiguous last dimension");
    const bool has_new = k_new.has_value() && k_new->defined();
    TORCH_CHECK(has_new == (v_new.has_value() && v_new->defined()), "k_new and v_new go together");
    c10::cuda::CUDAGuard guard(q.device());
    fcci_decode_desc d = blank_desc();
    d.B = (int32_t)B;
    d.Hq = (int32_t)Hq;
    d.Hkv = (int32_t)Hkv;
    d.D = (int32_t)D;
    d.q = q.data_ptr();
    d.q_stride_b = q.stride(0);
    d.q_stride_h = q.stride(1);
    if (has_new) {
        check_half_cuda(*k_new, "k_new");
        check_half_cuda(*v_new, "v_new");
        TORCH_CHECK(k_new->dim() == 3 && k_new->size(0) == B && k_new->size(1) == Hkv && k_new->size(2) == D &&
                        k_new->stride(2) == 1,
                    "k_new must be [B, Hkv, D]");
        TORCH_CHECK(v_new->sizes() == k_new->sizes() && v_new->stride(2) == 1, "v_new must be [B, Hkv, D]");
        d.k_new = k_new->data_ptr();
        d.k_new_stride_b = k_new->stride(0);
        d.k_new_stride_h = k_new->stride(1);
        d.v_new = v_new->data_ptr();
        d.v_new_stride_b = v_new->stride(0);
        d.v_new_stride_h = v_new->stride(1);
    }
    d.k_cache = k_cache.data_ptr();
    d.v_cache = v_cache.data_ptr();
    if (packed) {
        d.k_stride_b = 0;
        d.k_stride_h = k_cache.stride(0);
        d.k_stride_t = k_cache.stride(1);
        d.v_stride_b = 0;
        d.v_stride_h = v_cache.stride(0);
        d.v_stride_t = v_cache.stride(1);
        d.cu_seqlens = cu_seqlens->data_ptr<int32_t>();
    } else {
        d.k_stride_b = k_cache.stride(0);
        d.k_stride_h = k_cache.stride(1);
        d.k_stride_t = k_cache.stride(2);
        d.v_stride_b = v_cache.stride(0);
        d.v_stride_h = v_cache.stride(1);
        d.v_stride_t = v_cache.stride(2);
    }
    TORCH_CHECK(cap < (int64_t)1 << 31, "arena too long");
    d.capacity = (int32_t)cap;
    if (seq_lens.has_value() && seq_lens->defined()) {
        check_int32_cuda(*seq_lens, "seq_lens");
        TORCH_CHECK(seq_lens->numel() == B, "seq_lens must have B entries");
        d.seq_lens = seq_lens->data_ptr<int32_t>();
    } else {
        TORCH_CHECK(fixed_len >= 0, "give seq_lens or a non-negative fixed_len");
        TORCH_CHECK(!advance, "advance needs seq_lens");
        d.fixed_len = (int32_t)fixed_len;
    }
    d.out = out.data_ptr();
    d.out_stride_b = out.stride(0);
    d.out_stride_h = out.stride(1);
    if (q_rot_out.has_value() && q_rot_out->defined()) {
        check_rows(*q_rot_out, B * Hq * D, "q_rot_out");
        d.q_rot_out = q_rot_out->data_ptr();
    }
    d.scale = scale > 0 ? (float)scale : (float)(1.0 / std::sqrt((double)D));
    d.rope_theta = (float)rope_theta;
    d.rotary_dim = (int32_t)(rotary_dim < 0 ? (has_new ? D : 0) : rotary_dim);
    d.advance = advance ? 1 : 0;
    at::Tensor ws;
    if (workspace.has_value() && workspace->defined()) ws = *workspace;
    else if (split || advance || exch_rank >= 0) ws = cached_workspace(B, Hq, Hkv, D, q.device());
    if (ws.defined()) bind_workspace(d, ws);
    d.split = split ? 1 : 0;
    d.flags = (prefetch_kv ? FCCI_DECODE_PREFETCH_KV : 0u) | (check_early_read ? FCCI_DECODE_CHECK_EARLY_READ : 0u);
    if (exch_rank >= 0) {
        // ctx exchange: `out` is this rank's slice of its full-ctx buffer; the peers'
        // mappings receive the same slice at the same offsets
        TORCH_CHECK(!peer_out.empty() && peer_out.size() == peer_flags.size() && peer_out.size() <= FCCI_MAX_PEERS,
                    "peer_out and peer_flags: one entry per peer (1..7)");
        TORCH_CHECK(exch_flags != 0 && exch_epoch != 0, "exch_flags and exch_epoch are required");
        TORCH_CHECK(ws.defined(), "the exchange needs a workspace");
        fcci_ctx_exchange ex;
        std::memset(&ex, 0, sizeof(ex));
        ex.n_peers = (int32_t)peer_out.size();
        ex.rank = (int32_t)exch_rank;
        for (size_t i = 0; i < peer_out.size(); ++i) {
            ex.peer_out[i] = reinterpret_cast<void*>(peer_out[i]);
            ex.peer_flags[i] = reinterpret_cast<uint32_t*>(peer_flags[i]);
        }
        ex.flags = reinterpret_cast<uint32_t*>(exch_flags);
        ex.epoch = reinterpret_cast<uint32_t*>(exch_epoch);
        check_rc(fcci_decode_attention_exchange(&d, &ex, current_stream()), "attn_varlen.decode (exchange)");
        return;
    }
    check_rc(fcci_decode_attention(&d, current_stream()), "attn_varlen.decode");
}

void rope_append(at::Tensor q, at::Tensor k_new, at::Tensor v_new, at::Tensor k_cache, at::Tensor v_cache,
                 at::Tensor seq_lens, c10::optional<at::Tensor> cu_seqlens, double rope_theta, int64_t rotary_dim,
                 bool advance, c10::optional<at::Tensor> q_rot_out) {
    check_half_cuda(q, "q");
    check_half_cuda(k_new, "k_new");
    check_half_cuda(v_new, "v_new");
    check_half_cuda(k_cache, "k_cache");
    check_half_cuda(v_cache, "v_cache");
    check_int32_cuda(seq_lens, "seq_lens");
    TORCH_CHECK(q.dim() == 3 && q.stride(2) == 1, "q must be [B, Hq, D]");
    const int64_t B = q.size(0), Hq = q.size(1), D = q.size(2);
    const bool packed = cu_seqlens.has_value() && cu_seqlens->defined();
    const int64_t Hkv = packed ? k_cache.size(0) : k_cache.size(1);
    TORCH_CHECK(k_cache.dim() == (packed ? 3 : 4) && v_cache.sizes() == k_cache.sizes(), "arena shape");
    TORCH_CHECK(k_cache.stride(-1) == 1 && v_cache.stride(-1) == 1, "arena head_dim must be contiguous");
    TORCH_CHECK(k_new.dim() == 3 && k_new.size(0) == B && k_new.size(1) == Hkv && k_new.size(2) == D &&
                    k_new.stride(2) == 1 && v_new.sizes() == k_new.sizes() && v_new.stride(2) == 1,
                "k_new/v_new must be [B, Hkv, D]");
    TORCH_CHECK(seq_lens.numel() == B, "seq_lens must have B entries");
    c10::cuda::CUDAGuard guard(q.device());
    fcci_decode_desc d = blank_desc();
    d.B = (int32_t)B;
    d.Hq = (int32_t)Hq;
    d.Hkv = (int32_t)Hkv;
    d.D = (int32_t)D;
    d.q = q.data_ptr();
    d.q_stride_b = q.stride(0);
    d.q_stride_h = q.stride(1);
    d.k_new = k_new.data_ptr();
    d.k_new_stride_b = k_new.stride(0);
    d.k_new_stride_h = k_new.stride(1);
    d.v_new = v_new.data_ptr();
    d.v_new_stride_b = v_new.stride(0);
    d.v_new_stride_h = v_new.stride(1);
    d.k_cache = k_cache.data_ptr();
    d.v_cache = v_cache.data_ptr();
    if (packed) {
        check_int32_cuda(*cu_seqlens, "cu_seqlens");
        d.cu_seqlens = cu_seqlens->data_ptr<int32_t>();
        d.k_stride_h = k_cache.stride(0);
        d.k_stride_t = k_cache.stride(1);
        d.v_stride_h = v_cache.stride(0);
        d.v_stride_t = v_cache.stride(1);
        d.capacity = (int32_t)k_cache.size(1);
    } else {
        d.k_stride_b = k_cache.stride(0);
        d.k_stride_h = k_cache.stride(1);
        d.k_stride_t = k_cache.stride(2);
        d.v_stride_b = v_cache.stride(0);
        d.v_stride_h = v_cache.stride(1);
        d.v_stride_t = v_cache.stride(2);
        d.capacity = (int32_t)k_cache.size(2);
    }
    d.seq_lens = seq_lens.data_ptr<int32_t>();
    if (q_rot_out.has_value() && q_rot_out->defined()) {
        check_rows(*q_rot_out, B * Hq * D, "q_rot_out");
        d.q_rot_out = q_rot_out->data_ptr();
    }
    d.rope_theta = (float)rope_theta;
    d.rotary_dim = (int32_t)(rotary_dim < 0 ? D : rotary_dim);
    d.advance = advance ? 1 : 0;
    check_rc(fcci_rope_append(&d, current_stream()), "attn_varlen.rope_append");
}

at::Tensor make_prefill_workspace(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t total_q, int64_t max_seqlen_q,
                                  int64_t capacity, int64_t rotary_dim, const at::Device& dev) {
    const size_t bytes = fcci_prefill_workspace_bytes((int32_t)B, (int32_t)Hq, (int32_t)Hkv, (int32_t)D,
                                                      (int32_t)total_q, (int32_t)max_seqlen_q, (int32_t)capacity,
                                                      (int32_t)rotary_dim);
    TORCH_CHECK(bytes > 0, "fcci_prefill_workspace_bytes: invalid shape");
    at::Tensor ws = at::empty({(int64_t)bytes}, at::TensorOptions().dtype(at::kByte).device(dev));
    check_rc(fcci_prefill_workspace_init(ws.data_ptr(), bytes, current_stream()), "fcci_prefill_workspace_init");
    return ws;
}

// Causal varlen prefill: RoPE(q, k_new) at T_b + i, append into the arena, causal
// attention of the new tokens over all T_b + n_b keys (tcgen05 tensor cores).
void prefill_varlen(at::Tensor q, at::Tensor k_new, at::Tensor v_new, at::Tensor k_cache, at::Tensor v_cache,
                    at::Tensor out, at::Tensor cu_seqlens_q, int64_t max_seqlen_q, c10::optional<at::Tensor> seq_lens,
                    c10::optional<at::Tensor> cu_seqlens_kv, int64_t fixed_len, double scale, double rope_theta,
                    int64_t rotary_dim, bool advance, c10::optional<at::Tensor> workspace, const std::string& part) {
    TORCH_CHECK(part == "all" || part == "prepare" || part == "attend", "part must be 'all', 'prepare' or 'attend'");
    for (auto* t : {&q, &k_new, &v_new, &k_cache, &v_cache, &out}) check_half_cuda(*t, "prefill tensor");
    check_int32_cuda(cu_seqlens_q, "cu_seqlens_q");
    TORCH_CHECK(q.dim() == 3 && q.stride(2) == 1, "q must be [total, Hq, D] with a contiguous last dimension");
    const int64_t total = q.size(0), Hq = q.size(1), D = q.size(2);
    const int64_t B = cu_seqlens_q.numel() - 1;
    TORCH_CHECK(B >= 1, "cu_seqlens_q must have B+1 >= 2 entries");
    TORCH_CHECK(k_new.dim() == 3 && k_new.size(0) == total && k_new.size(2) == D && k_new.stride(2) == 1,
                "k_new must be [total, Hkv, D]");
    const int64_t Hkv = k_new.size(1);
    TORCH_CHECK(v_new.sizes() == k_new.sizes() && v_new.stride(2) == 1, "v_new must be [total, Hkv, D]");
    TORCH_CHECK(out.sizes() == q.sizes() && out.stride(2) == 1, "out must be [total, Hq, D]");
    TORCH_CHECK(Hkv > 0 && Hq % Hkv == 0, "Hq must be a multiple of Hkv");
    const bool packed = cu_seqlens_kv.has_value() && cu_seqlens_kv->defined();
    int64_t cap;
    if (packed) {
        TORCH_CHECK(k_cache.dim() == 3 && k_cache.size(0) == Hkv, "packed arena must be [Hkv, total_tokens, D]");
        check_int32_cuda(*cu_seqlens_kv, "cu_seqlens_kv");
        TORCH_CHECK(cu_seqlens_kv->numel() == B + 1, "cu_seqlens_kv must have B+1 entries");
        cap = k_cache.size(1);
    } else {
        TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(0) == B && k_cache.size(1) == Hkv,
                    "arena must be [B, Hkv, capacity, D]");
        cap = k_cache.size(2);
    }
    TORCH_CHECK(v_cache.sizes() == k_cache.sizes() && k_cache.size(-1) == D, "arena shapes differ");
    TORCH_CHECK(tma_compatible(k_cache) && tma_compatible(v_cache),
                "arena must have a contiguous head_dim, 16-byte aligned base and strides");
    TORCH_CHECK(cap < (int64_t)1 << 31 && total < (int64_t)1 << 31, "sizes exceed int32");
    c10::cuda::CUDAGuard guard(q.device());
    fcci_prefill_desc d;
    std::memset(&d, 0, sizeof(d));
    d.abi_version = FCCI_PREFILL_ABI_VERSION;
    d.B = (int32_t)B;
    d.Hq = (int32_t)Hq;
    d.Hkv = (int32_t)Hkv;
    d.D = (int32_t)D;
    d.total_q = (int32_t)total;
    d.max_seqlen_q = (int32_t)max_seqlen_q;
    d.cu_seqlens_q = cu_seqlens_q.data_ptr<int32_t>();
    d.q = q.data_ptr();
    d.q_stride_t = q.stride(0);
    d.q_stride_h = q.stride(1);
    d.k_new = k_new.data_ptr();
    d.k_new_stride_t = k_new.stride(0);
    d.k_new_stride_h = k_new.stride(1);
    d.v_new = v_new.data_ptr();
    d.v_new_stride_t = v_new.stride(0);
    d.v_new_stride_h = v_new.stride(1);
    d.k_cache = k_cache.data_ptr();
    d.v_cache = v_cache.data_ptr();
    if (packed) {
        d.k_stride_h = k_cache.stride(0);
        d.k_stride_t = k_cache.stride(1);
        d.v_stride_h = v_cache.stride(0);
        d.v_stride_t = v_cache.stride(1);
        d.cu_seqlens_kv = cu_seqlens_kv->data_ptr<int32_t>();
    } else {
        d.k_stride_b = k_cache.stride(0);
        d.k_stride_h = k_cache.stride(1);
        d.k_stride_t = k_cache.stride(2);
        d.v_stride_b = v_cache.stride(0);
        d.v_stride_h = v_cache.stride(1);
        d.v_stride_t = v_cache.stride(2);
    }
    d.capacity = (int32_t)cap;
    if (seq_lens.has_value() && seq_lens->defined()) {
        check_int32_cuda(*seq_lens, "seq_lens");
        TORCH_CHECK(seq_lens->numel() == B, "seq_lens must have B entries");
        d.seq_lens = seq_lens->data_ptr<int32_t>();
    } else {
        TORCH_CHECK(fixed_len >= 0, "give seq_lens or a non-negative fixed_len");
        TORCH_CHECK(!advance, "advance needs seq_lens");
        d.fixed_len = (int32_t)fixed_len;
    }
    d.out = out.data_ptr();
    d.out_stride_t = out.stride(0);
    d.out_stride_h = out.stride(1);
    d.scale = scale > 0 ? (float)scale : (float)(1.0 / std::sqrt((double)D));
    d.rope_theta = (float)rope_theta;
    d.rotary_dim = (int32_t)(rotary_dim < 0 ? D : rotary_dim);
    d.advance = advance ? 1 : 0;
    at::Tensor ws;
    if (workspace.has_value() && workspace->defined()) ws = *workspace;
    else ws = make_prefill_workspace(B, Hq, Hkv, D, total, max_seqlen_q, cap, d.rotary_dim, q.device());
    TORCH_CHECK(ws.is_cuda() && ws.scalar_type() == at::kByte && ws.is_contiguous(),
                "workspace must be a contiguous uint8 CUDA tensor from make_prefill_workspace()");
    d.workspace = ws.data_ptr();
    d.workspace_bytes = (size_t)ws.numel();
    if (part == "prepare") check_rc(fcci_prefill_prepare(&d, current_stream()), "attn_varlen.prefill_varlen(prepare)");
    else if (part == "attend") check_rc(fcci_prefill_attend(&d, current_stream()), "attn_varlen.prefill_varlen(attend)");
    else check_rc(fcci_prefill_attention(&d, current_stream()), "attn_varlen.prefill_varlen");
}

int64_t read_error(at::Tensor workspace, bool clear) {
    TORCH_CHECK(workspace.is_cuda() && workspace.scalar_type() == at::kByte, "workspace must be a uint8 CUDA tensor");
    c10::cuda::CUDAGuard guard(workspace.device());
    uint32_t flags = 0;
    check_rc(fcci_decode_read_error(workspace.data_ptr(), &flags, clear ? 1 : 0, current_stream()),
             "attn_varlen.read_error");
    return (int64_t)flags;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "B200 (sm_100a) varlen decode attention; drop-in for the reference's attn_varlen extension";
    m.def("forward", &forward, "Varlen attention (Q·K^T->softmax->P·V) for one token", py::arg("q"), py::arg("k"),
          py::arg("v"), py::arg("seq_len"), py::arg("scale"));
    m.def("forward_out", &forward_out, "forward() into a caller-owned ctx; allocation-free when given a workspace",
          py::arg("q"), py::arg("k"), py::arg("v"), py::arg("seq_len"), py::arg("scale"), py::arg("out"),
          py::arg("workspace") = py::none());
    m.def("decode", &decode,
          "Batched/varlen decode step: RoPE(q,k_new) at T, append at T, split-KV GQA attention over T+1 keys",
          py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("out"), py::arg("k_new") = py::none(),
          py::arg("v_new") = py::none(), py::arg("seq_lens") = py::none(), py::arg("cu_seqlens") = py::none(),
          py::arg("fixed_len") = -1, py::arg("scale") = -1.0, py::arg("rope_theta") = 10000.0,
          py::arg("rotary_dim") = -1, py::arg("advance") = false, py::arg("workspace") = py::none(),
          py::arg("q_rot_out") = py::none(), py::arg("split") = true, py::arg("prefetch_kv") = false, py::kw_only(),
          py::arg("check_early_read") = false,
          py::arg("peer_out") = std::vector<uint64_t>(), py::arg("peer_flags") = std::vector<uint64_t>(),
          py::arg("exch_flags") = 0, py::arg("exch_epoch") = 0, py::arg("exch_rank") = -1);
    m.def("rope_append", &rope_append, "RoPE(q,k_new) at T and append of k/v at T (no attention)", py::arg("q"),
          py::arg("k_new"), py::arg("v_new"), py::arg("k_cache"), py::arg("v_cache"), py::arg("seq_lens"),
          py::arg("cu_seqlens") = py::none(), py::arg("rope_theta") = 10000.0, py::arg("rotary_dim") = -1,
          py::arg("advance") = false, py::arg("q_rot_out") = py::none());
    m.def(
        "workspace_bytes",
        [](int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t device) {
            return (int64_t)fcci_decode_workspace_bytes((int32_t)B, (int32_t)Hq, (int32_t)Hkv, (int32_t)D, (int)device);
        },
        py::arg("B"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("device") = 0);
    m.def(
        "make_workspace",
        [](int64_t B, int64_t Hq, int64_t Hkv, int64_t D, c10::optional<at::Device> device) {
            at::Device dev = device.has_value() ? *device : at::Device(at::kCUDA, c10::cuda::current_device());
            c10::cuda::CUDAGuard guard(dev);
            return make_workspace(B, Hq, Hkv, D, dev);
        },
        "Zeroed workspace for decode()/forward_out() (allocate outside graph capture)", py::arg("B"), py::arg("Hq"),
        py::arg("Hkv"), py::arg("D"), py::arg("device") = py::none());
    m.def("read_error", &read_error, "Device error word of a workspace (synchronises)", py::arg("workspace"),
          py::arg("clear") = true);
    m.def("prefill_varlen", &prefill_varlen,
          "Causal varlen prefill: RoPE(q,k_new) at T_b+i, append into the arena, causal attention over T_b+n_b keys",
          py::arg("q"), py::arg("k_new"), py::arg("v_new"), py::arg("k_cache"), py::arg("v_cache"), py::arg("out"),
          py::arg("cu_seqlens_q"), py::arg("max_seqlen_q"), py::arg("seq_lens") = py::none(),
          py::arg("cu_seqlens_kv") = py::none(), py::arg("fixed_len") = -1, py::arg("scale") = -1.0,
          py::arg("rope_theta") = 10000.0, py::arg("rotary_dim") = -1, py::arg("advance") = false,
          py::arg("workspace") = py::none(), py::arg("part") = "all");
    m.def(
        "make_prefill_workspace",
        [](int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t total_q, int64_t max_seqlen_q, int64_t capacity,
           int64_t rotary_dim, c10::optional<at::Device> device) {
            at::Device dev = device.has_value() ? *device : at::Device(at::kCUDA, c10::cuda::current_device());
            c10::cuda::CUDAGuard guard(dev);
            return make_prefill_workspace(B, Hq, Hkv, D, total_q, max_seqlen_q, capacity,
                                          rotary_dim < 0 ? D : rotary_dim, dev);
        },
        "Zeroed workspace for prefill_varlen() (allocate outside graph capture)", py::arg("B"), py::arg("Hq"),
        py::arg("Hkv"), py::arg("D"), py::arg("total_q"), py::arg("max_seqlen_q"), py::arg("capacity"),
        py::arg("rotary_dim") = -1, py::arg("device") = py::none());
    m.def(
        "prefill_read_error",
        [](at::Tensor workspace, bool clear) {
            TORCH_CHECK(workspace.is_cuda() && workspace.scalar_type() == at::kByte, "workspace must be uint8 CUDA");
            c10::cuda::CUDAGuard guard(workspace.device());
            uint32_t flags = 0;
            check_rc(fcci_prefill_read_error(workspace.data_ptr(), &flags, clear ? 1 : 0, current_stream()),
                     "attn_varlen.prefill_read_error");
            return (int64_t)flags;
        },
        py::arg("workspace"), py::arg("clear") = true);
    m.def("launch_count", []() { return (int64_t)fcci_launch_count(); });
    // ctx exchange plumbing (fcci_exchange.h): IPC buffers and the bounded flag wait
    m.def(
        "ipc_alloc",
        [](int64_t nbytes, c10::optional<at::Device> device) {
            at::Device dev = device.has_value() ? *device : at::Device(at::kCUDA, c10::cuda::current_device());
            c10::cuda::CUDAGuard guard(dev);
            void* ptr = nullptr;
            std::string handle(FCCI_IPC_HANDLE_BYTES, '\0');
            check_rc(fcci_ipc_alloc((size_t)nbytes, &ptr, &handle[0]), "ipc_alloc");
            at::Tensor t = at::from_blob(
                ptr, {nbytes}, [](void* p) { fcci_ipc_free(p); }, at::TensorOptions().dtype(at::kByte).device(dev));
            return py::make_tuple(t, py::bytes(handle));
        },
        "Zeroed device buffer that peer processes can map, and its IPC handle (bytes)", py::arg("nbytes"),
        py::arg("device") = py::none());
    m.def(
        "ipc_open",
        [](py::bytes handle) {
            std::string h = handle;
            TORCH_CHECK(h.size() == FCCI_IPC_HANDLE_BYTES, "ipc_open: handle must be ", FCCI_IPC_HANDLE_BYTES, " bytes");
            void* ptr = nullptr;
            check_rc(fcci_ipc_open(h.data(), &ptr), "ipc_open");
            return (uint64_t)reinterpret_cast<uintptr_t>(ptr);
        },
        "Map a peer process's buffer on the current device; returns its device address");
    m.def(
        "ipc_close", [](uint64_t ptr) { check_rc(fcci_ipc_close(reinterpret_cast<void*>(ptr)), "ipc_close"); },
        "Unmap a buffer opened with ipc_open");
    m.def(
        "exchange_wait",
        [](at::Tensor flags, int64_t n, at::Tensor epoch, at::Tensor err, int64_t limit_ns) {
            TORCH_CHECK(flags.is_cuda() && epoch.is_cuda() && err.is_cuda(), "exchange_wait: CUDA tensors");
            c10::cuda::CUDAGuard guard(flags.device());
            check_rc(fcci_exchange_wait(static_cast<const uint32_t*>(flags.data_ptr()), (int)n,
                                        static_cast<const uint32_t*>(epoch.data_ptr()),
                                        static_cast<uint32_t*>(err.data_ptr()), (uint64_t)limit_ns, current_stream()),
                     "exchange_wait");
        },
        "Hold the current stream until every flag has reached the epoch (bounded; timeout bit in err)",
        py::arg("flags"), py::arg("n"), py::arg("epoch"), py::arg("err"), py::arg("limit_ns") = 1000000000);
    m.def("clear_workspace_cache", &clear_workspace_cache,
          "Drop the workspaces kept for calls made without one (forward, capture_decode with q); "
          "needed only after a device timeout");
    m.def(
        "set_tuning",
        [](int64_t stages, int64_t ctas, int64_t max_cluster, int64_t solo_tiles, int64_t min_tiles) {
            check_rc(fcci_decode_set_tuning((int)stages, (int)ctas), "set_tuning");
            check_rc(fcci_decode_set_cluster_tuning((int)max_cluster, (int)solo_tiles, (int)min_tiles), "set_tuning");
        },
        "Measurement hook: pipeline stages, CTAs per SM, the largest cluster of the split mode (0 = automatic, "
        "max_cluster 1 = no clusters) and the tiles up to which a pair is not split in a cluster (-1 = automatic)",
        py::arg("stages") = 0, py::arg("ctas_per_sm") = 0, py::arg("max_cluster") = 0, py::arg("solo_tiles") = -1,
        py::arg("min_tiles") = 0);
}
