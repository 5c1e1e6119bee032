// Internal declarations shared by the library's translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

#include "fcci_decode.h"
#include "fcci_exchange.h"

namespace fcci {

// Upper bound of resident decode CTAs per SM; the split-mode workspace is sized for it.
constexpr int kMaxCtasPerSm = 2;

struct Tuning {
    int stages = 0;       // pipeline depth (64-key K+V tiles per CTA); 0 = automatic
    int ctas_per_sm = 0;  // persistent CTAs per SM in split mode; 0 = automatic
    int max_cluster = 0;  // largest cluster of a split launch; 0 = automatic (16), 1 = no clusters
    int solo_tiles = -1;  // pairs of at most this many tiles stay on one CTA of their cluster; -1 = automatic
    int cluster_min_tiles = 0;  // tiles per cluster CTA at full arena capacity, at least; 0 = automatic
};
Tuning& tuning();

struct WorkspaceLayout {
    size_t err, done, pair_cnt, part_lse, part_o, total, zero_bytes;
};
WorkspaceLayout workspace_layout(int B, int Hq, int Hkv, int D, int grid);
int max_grid(int dev);
int device_sm_count(int dev);

int set_status(int code, const char* msg);
// fp16 TMA descriptor with 128-byte swizzle (dims[0] contiguous, byte strides of dims[1..]).
int encode_f16_sw128(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const int64_t* stride_bytes,
                     const uint32_t* box);
int set_cuda_status(cudaError_t e);
void count_launch();

// ex (nullable): the ctx exchange of fcci_decode_attention_exchange
int decode_attention(const fcci_decode_desc* d, cudaStream_t stream, const fcci_ctx_exchange* ex = nullptr);

// Launch `kernel` with programmatic stream serialization: it may start while the
// previous kernel of the stream finishes, and must call griddepcontrol.wait before
// it reads that kernel's results (every kernel launched this way does).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    count_launch();
    return set_cuda_status(e == cudaSuccess ? cudaGetLastError() : e);
}
// The same with `cluster` CTAs per thread-block cluster (1-D); cluster <= 1 launches
// without clusters.
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       int cluster, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster > 1 ? (unsigned)cluster : 1u;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cluster > 1 ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    count_launch();
    return set_cuda_status(e == cudaSuccess ? cudaGetLastError() : e);
}
int rope_append(const fcci_decode_desc* d, cudaStream_t stream);

// The batch-1 projection of gemv.cu with two additions over fcci_gemv_desc: the up
// rows of the SwiGLU mode as a separate matrix W2 (NULL: rows N..2N-1 of W), and mode
// 3, which stores y in fp32 (the vocab projection's logits).
struct GemvArgs {
    const void* W;
    const void* W2;
    int64_t ld_w;
    int32_t N, K;
    const void* x;
    const void* rms_w;
    float eps;
    void* out;
    int32_t mode;
};
int gemv(const GemvArgs* d, cudaStream_t stream);

}  // namespace fcci
