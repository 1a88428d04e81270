// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <utility>

namespace ti {

// Record an error message for ti_last_error() and return `code`.
int set_error(int code, const char* msg);
int set_cuda_error(cudaError_t e, const char* what);
void clear_error();
void count_launch(unsigned n = 1);

// Programmatic dependent launch: every kernel of this library is launched with
// cudaLaunchAttributeProgrammaticStreamSerialization, calls griddepcontrol.wait before it
// touches memory that an earlier kernel may write, and griddepcontrol.launch_dependents once
// it holds all of its on-chip resources.  The next kernel's CTAs then become resident while
// this one drains, hiding the launch gap (and, for the GEMMs, the first weight tiles' fetch).
// On by default; the environment variable TI_PDL=0 turns it off (plain stream ordering).
bool pdl_enabled();

// Launch `kern` on stream `s` (PDL attribute when enabled; clusters of shape `cluster` when it
// has more than one CTA) and count it.  Returns TI_OK or TI_ERR_CUDA with `what` in the message.
template <typename... KArgs, typename... Args>
int launch_kernel_cl(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t s, dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = cluster.x;
    at[n].val.clusterDim.y = cluster.y;
    at[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  count_launch();
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_cuda_error(e, what);
  }
  return 0;
}

// As launch_kernel_cl with a cluster of `cluster_z` CTAs along grid z (none when <= 1).
template <typename... KArgs, typename... Args>
int launch_kernel(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t s, int cluster_z, Args&&... args) {
  return launch_kernel_cl(what, kern, grid, block, smem, s,
                          dim3(1, 1, cluster_z > 1 ? (unsigned)cluster_z : 1u),
                          std::forward<Args>(args)...);
}

// Split-K slots per (sequence, query head) that ti_paged_attention_decode uses with the default
// partitioning (1: the call needs no workspace).
int64_t attn_split_parts(int batch, int num_heads, int num_kv_heads, int head_dim,
                         int max_blocks);

// The weight-streaming greedy lm_head for small token counts (gemv.cu): M <= 64 tokens of A
// (dtype, leading dim lda) against N rows of B (dtype, or int8 with per-row `scale` when int8),
// K <= 896, N % 128 == 0; writes the [M, N / 128] argmax partials.
constexpr int kGemvMaxTokens = 64;
constexpr int kGemvMaxK = 896;
int gemv_argmax(const void* A, int64_t lda, const void* B, int64_t ldb, bool int8,
                const float* scale, int M, int N, int K, float* aux_val, int32_t* aux_idx,
                int dtype, cudaStream_t s);

// CTAs of ti_gemm_qkv_rope's launch for M rows of a hidden size K into N = (NH+2KVH)*64 outputs.
int gemm_qkv_ctas(int M, int N, int K, int dtype);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link needed).
int encode_tensor_map_2d(CUtensorMap* out, CUtensorMapDataType type, void* base,
                         const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                         const cuuint32_t* box, const cuuint32_t* elem_strides,
                         CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo);

}  // namespace ti
