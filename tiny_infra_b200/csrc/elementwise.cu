// Bandwidth-bound per-token kernels: RoPE (in place, and fused with the KV-append write),
// SwiGLU, RMSNorm, embedding gather.  All use 16-byte vector accesses and grids sized in
// multiples of the SM count.
#include <algorithm>

#include "capi_internal.h"
#include "common.cuh"
#include "rmsnorm_row.cuh"

namespace ti {
namespace ew {

constexpr int kThreads = 256;
#ifndef TI_RMS_SMALL_THREADS
#define TI_RMS_SMALL_THREADS 64
#endif
constexpr int kRmsSmallRows = 2048;                   // up to here: the small-CTA RMSNorm grid
constexpr int kRmsSmallThreads = TI_RMS_SMALL_THREADS;

// Rotate 8 dims of the first half (x1) with the matching 8 dims of the second half (x2)
// (reference src/fused_rope.cu:37-50).
__device__ __forceinline__ void rotate8(float* x1, float* x2, const float* c, const float* s) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = x1[i], b = x2[i];
    x1[i] = a * c[i] - b * s[i];
    x2[i] = a * s[i] + b * c[i];
  }
}

// ---- in-place RoPE on separate q / k tensors (drop-in for custom_rope.apply_inplace) --------
template <typename T>
__global__ void rope_inplace_kernel(T* q, int64_t q_stride, T* k, int64_t k_stride,
                                    const float* __restrict__ cos, const float* __restrict__ sin,
                                    const int32_t* __restrict__ pos, int T_, int NH, int KVH,
                                    int HD) {
  pdl_wait();
  pdl_launch_dependents();
  const int half = HD / 2, per_head = half / 8;
  const int64_t per_tok = (int64_t)(NH + KVH) * per_head;
  const int64_t total = per_tok * T_;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / per_tok);
    const int r = (int)(i % per_tok);
    const int h = r / per_head, d0 = (r % per_head) * 8;
    T* base = (h < NH) ? q + t * q_stride + (int64_t)h * HD : k + t * k_stride + (int64_t)(h - NH) * HD;
    const int64_t tab = (int64_t)pos[t] * half + d0;
    float c[8], s[8], x1[8], x2[8];
    load8f(cos + tab, c);
    load8f(sin + tab, s);
    Vec8<T> v1, v2;
    v1.load(base + d0);
    v2.load(base + d0 + half);
    v1.to_float(x1);
    v2.to_float(x2);
    rotate8(x1, x2, c, s);
    v1.from_float(x1);
    v2.from_float(x2);
    v1.store(base + d0);
    v2.store(base + d0 + half);
  }
}

// ---- RoPE fused with the KV-append write ---------------------------------------------------
// Work item per token: NH*P rotations of q (in place), KVH*P rotations of k (written back in
// place and into the pool), KVH*2P copies of 8 v elements into the pool; P = HD/16.
template <typename T>
__global__ void rope_append_kernel(T* qkv, int64_t stride, T* k_cache, T* v_cache,
                                   const int64_t* __restrict__ slot_mapping,
                                   const float* __restrict__ cos, const float* __restrict__ sin,
                                   const int32_t* __restrict__ pos, int T_, int NH, int KVH,
                                   int HD, int bs) {
  pdl_wait();
  pdl_launch_dependents();
  const int half = HD / 2, P = half / 8;
  const int per_tok = (NH + KVH) * P + KVH * 2 * P;
  const int64_t total = (int64_t)per_tok * T_;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / per_tok);
    int r = (int)(i % per_tok);
    T* row = qkv + t * stride;
    const int64_t slot = slot_mapping[t];
    if (r < (NH + KVH) * P) {
      const int h = r / P, d0 = (r % P) * 8;
      T* base = row + (int64_t)h * HD;   // q heads then k heads are contiguous in the row
      const int64_t tab = (int64_t)pos[t] * half + d0;
      float c[8], s[8], x1[8], x2[8];
      load8f(cos + tab, c);
      load8f(sin + tab, s);
      Vec8<T> v1, v2;
      v1.load(base + d0);
      v2.load(base + d0 + half);
      v1.to_float(x1);
      v2.to_float(x2);
      rotate8(x1, x2, c, s);
      v1.from_float(x1);
      v2.from_float(x2);
      v1.store(base + d0);
      v2.store(base + d0 + half);
      if (h >= NH && slot >= 0) {
        const int kh = h - NH;
        const int64_t blk = slot / bs, off = slot % bs;
        T* dst = k_cache + ((blk * KVH + kh) * bs + off) * HD;
        v1.store(dst + d0);
        v2.store(dst + d0 + half);
      }
    } else if (slot >= 0) {
      r -= (NH + KVH) * P;
      const int kh = r / (2 * P), d0 = (r % (2 * P)) * 8;
      const int64_t blk = slot / bs, off = slot % bs;
      Vec8<T> v;
      v.load(row + (int64_t)(NH + KVH) * HD + (int64_t)kh * HD + d0);
      v.store(v_cache + ((blk * KVH + kh) * bs + off) * HD + d0);
    }
  }
}

// ---- SwiGLU (drop-in for custom_swiglu.forward) -------------------------------------------
template <typename T>
__global__ void swiglu_kernel(T* __restrict__ out, const T* __restrict__ x, int64_t T_, int I) {
  pdl_wait();
  pdl_launch_dependents();
  const int per = I / 8;
  const int64_t total = T_ * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per;
    const int c = (int)(i % per) * 8;
    Vec8<T> g, u, o;
    g.load(x + t * 2 * I + c);
    u.load(x + t * 2 * I + I + c);
    float gf[8], uf[8], of[8];
    g.to_float(gf);
    u.to_float(uf);
#pragma unroll
    for (int j = 0; j < 8; ++j) of[j] = gf[j] / (1.0f + expf(-gf[j])) * uf[j];
    o.from_float(of);
    o.store(out + t * I + c);
  }
}

// ---- RMSNorm: one warp per row -------------------------------------------------------------
// y = w * round(x * rstd): the normalised row is rounded to the output dtype before the weight
// multiply, as models/qwen_25.py:36 does (`weight * hidden.to(input_dtype)`).
// RMSNorm with the row in registers (hidden <= NC * 256): each lane holds NC chunks of 8
// elements, so the row is read once; the (static) weight is loaded before the wait on the
// previous kernel.  Rounding as the reference: bf16(w * bf16(x * rstd)) (models/qwen_25.py:34-36).
template <typename TX, typename T, int NC>
__global__ void rmsnorm_reg_kernel(T* __restrict__ out, const TX* __restrict__ x,
                                   const T* __restrict__ w, float eps, int rows, int H) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  float wf[NC][8];
  rms_load_weight<T, NC>(w, H, lane, wf);
  // Dependents launch only after this wait: the decode step relies on it (the attention two
  // kernels later reads the plan written before this kernel without waiting, TI_ATTN_EARLY_KV).
  pdl_wait();
  pdl_launch_dependents();
  for (int r = warp; r < rows; r += nwarps)
    rms_row<TX, T, NC>(out + (int64_t)r * H, x + (int64_t)r * H, wf, eps, H, lane);
}

template <typename TX, typename T>
__global__ void rmsnorm_kernel(T* __restrict__ out, const TX* __restrict__ x,
                               const T* __restrict__ w, float eps, int rows, int H) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int r = warp; r < rows; r += nwarps) {
    const TX* xr = x + (int64_t)r * H;
    float ss = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      float f[8];
      if constexpr (sizeof(TX) == 4) load8f(reinterpret_cast<const float*>(xr) + c, f);
      else { Vec8<TX> v; v.load(xr + c); v.to_float(f); }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss / (float)H + eps);
    for (int c = lane * 8; c < H; c += 256) {
      float f[8], wf[8];
      if constexpr (sizeof(TX) == 4) load8f(reinterpret_cast<const float*>(xr) + c, f);
      else { Vec8<TX> v; v.load(xr + c); v.to_float(f); }
      Vec8<T> wv;
      wv.load(w + c);
      wv.to_float(wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = wf[j] * Elem<T>::to_f(Elem<T>::from_f(f[j] * rstd));
      Vec8<T> o;
      o.from_float(f);
      o.store(out + (int64_t)r * H + c);
    }
  }
}

template <typename T>
__global__ void embedding_kernel(float* __restrict__ out, const T* __restrict__ table,
                                 const int32_t* __restrict__ ids, int rows, int H, int64_t V) {
  pdl_wait();
  pdl_launch_dependents();
  const int per = H / 8;
  const int64_t total = (int64_t)rows * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / per), c = (int)(i % per) * 8;
    const int64_t id = ids[t];
    float f[8];
    if (id >= 0 && id < V) {
      Vec8<T> v;
      v.load(table + id * H + c);
      v.to_float(f);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = 0.f;
    }
    float4* o = reinterpret_cast<float4*>(out + (int64_t)t * H + c);
    o[0] = make_float4(f[0], f[1], f[2], f[3]);
    o[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

static int grid_for(int64_t work) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int64_t blocks = (work + kThreads - 1) / kThreads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * 16));
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace ew
}  // namespace ti

using namespace ti;

extern "C" int ti_rope_inplace(void* q, int64_t q_tok_stride, void* k, int64_t k_tok_stride,
                               const float* cos, const float* sin, const int32_t* pos,
                               int num_tokens, int num_heads, int num_kv_heads, int head_dim,
                               int dtype, void* stream) {
  clear_error();
  if (num_tokens == 0) return TI_OK;
  if (!q || !k || !cos || !sin || !pos || num_tokens < 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "rope: null pointer or negative size");
  if (head_dim % 16 != 0)
    return set_error(TI_ERR_UNSUPPORTED, "rope: head_dim must be a multiple of 16");
  if (!ew::aligned16(q) || !ew::aligned16(k) || !ew::aligned16(cos) || !ew::aligned16(sin) ||
      (q_tok_stride % 8) || (k_tok_stride % 8))
    return set_error(TI_ERR_INVALID_ARGUMENT, "rope: tensors must be 16-byte aligned");
  const int64_t work = (int64_t)num_tokens * (num_heads + num_kv_heads) * (head_dim / 16);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16)
    return launch_kernel("rope launch", ew::rope_inplace_kernel<__nv_bfloat16>,
                         dim3(ew::grid_for(work)), dim3(ew::kThreads), 0, s, 1,
        (__nv_bfloat16*)q, q_tok_stride, (__nv_bfloat16*)k, k_tok_stride, cos, sin, pos,
        num_tokens, num_heads, num_kv_heads, head_dim);
  else if (dtype == TI_DTYPE_FP16)
    return launch_kernel("rope launch", ew::rope_inplace_kernel<__half>,
                         dim3(ew::grid_for(work)), dim3(ew::kThreads), 0, s, 1,
        (__half*)q, q_tok_stride, (__half*)k, k_tok_stride, cos, sin, pos, num_tokens,
        num_heads, num_kv_heads, head_dim);
  else
    return set_error(TI_ERR_UNSUPPORTED, "rope: dtype must be bf16 or fp16");
}

extern "C" int ti_rope_kv_append(void* qkv, int64_t qkv_stride, void* k_cache, void* v_cache,
                                 const int64_t* slot_mapping, const float* cos, const float* sin,
                                 const int32_t* pos, int num_tokens, int num_heads,
                                 int num_kv_heads, int head_dim, int block_size, int dtype,
                                 void* stream) {
  clear_error();
  if (num_tokens == 0) return TI_OK;
  if (!qkv || !k_cache || !v_cache || !slot_mapping || !cos || !sin || !pos || num_tokens < 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "rope_kv_append: null pointer or negative size");
  if (head_dim % 16 != 0 || block_size <= 0)
    return set_error(TI_ERR_UNSUPPORTED, "rope_kv_append: head_dim must be a multiple of 16");
  if (!ew::aligned16(qkv) || !ew::aligned16(k_cache) || !ew::aligned16(v_cache) ||
      !ew::aligned16(cos) || !ew::aligned16(sin) || (qkv_stride % 8))
    return set_error(TI_ERR_INVALID_ARGUMENT, "rope_kv_append: tensors must be 16-byte aligned");
  const int P = head_dim / 16;
  const int64_t work = (int64_t)num_tokens * ((num_heads + num_kv_heads) * P + num_kv_heads * 2 * P);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16)
    return launch_kernel("rope_kv_append launch", ew::rope_append_kernel<__nv_bfloat16>,
                         dim3(ew::grid_for(work)), dim3(ew::kThreads), 0, s, 1,
        (__nv_bfloat16*)qkv, qkv_stride, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache,
        slot_mapping, cos, sin, pos, num_tokens, num_heads, num_kv_heads, head_dim, block_size);
  else if (dtype == TI_DTYPE_FP16)
    return launch_kernel("rope_kv_append launch", ew::rope_append_kernel<__half>,
                         dim3(ew::grid_for(work)), dim3(ew::kThreads), 0, s, 1,
        (__half*)qkv, qkv_stride, (__half*)k_cache, (__half*)v_cache, slot_mapping, cos, sin,
        pos, num_tokens, num_heads, num_kv_heads, head_dim, block_size);
  else
    return set_error(TI_ERR_UNSUPPORTED, "rope_kv_append: dtype must be bf16 or fp16");
}

extern "C" int ti_swiglu(void* out, const void* x, int64_t num_tokens, int inter, int dtype,
                         void* stream) {
  clear_error();
  if (num_tokens == 0) return TI_OK;
  if (!out || !x || num_tokens < 0) return set_error(TI_ERR_INVALID_ARGUMENT, "swiglu: null pointer");
  if (inter % 8 != 0)   // fused_swiglu.cu:68
    return set_error(TI_ERR_INVALID_ARGUMENT, "Hidden size must be a multiple of 8 for vectorized access.");
  if (!ew::aligned16(out) || !ew::aligned16(x))
    return set_error(TI_ERR_INVALID_ARGUMENT, "swiglu: tensors must be 16-byte aligned");
  const int64_t work = num_tokens * (inter / 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16)
    return launch_kernel("swiglu launch", ew::swiglu_kernel<__nv_bfloat16>,
                         dim3(ew::grid_for(work)), dim3(ew::kThreads), 0, s, 1,
        (__nv_bfloat16*)out, (const __nv_bfloat16*)x, num_tokens, inter);
  else if (dtype == TI_DTYPE_FP16)
    return launch_kernel("swiglu launch", ew::swiglu_kernel<__half>,
                         dim3(ew::grid_for(work)), dim3(ew::kThreads), 0, s, 1,
        (__half*)out, (const __half*)x, num_tokens, inter);
  else
    return set_error(TI_ERR_UNSUPPORTED, "swiglu: dtype must be bf16 or fp16");
}

extern "C" int ti_rmsnorm(void* out, const void* x, int x_dtype, const void* weight, float eps,
                          int num_tokens, int hidden, int dtype, void* stream) {
  clear_error();
  if (num_tokens == 0) return TI_OK;
  if (!out || !x || !weight || num_tokens < 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "rmsnorm: null pointer");
  if (hidden % 8 != 0) return set_error(TI_ERR_UNSUPPORTED, "rmsnorm: hidden must be a multiple of 8");
  if (!ew::aligned16(out) || !ew::aligned16(x) || !ew::aligned16(weight))
    return set_error(TI_ERR_INVALID_ARGUMENT, "rmsnorm: tensors must be 16-byte aligned");
  const int64_t work = (int64_t)num_tokens * 32;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int g = ew::grid_for(work);
  if (hidden <= 1024) {   // the row in registers: one read of x
    // decode batches: CTAs of 2 rows, so the rows spread over many SMs (each SM's share of the
    // rows arrives in one L2 round trip); prefill chunks: 8 rows per CTA
    const int bt = num_tokens <= ew::kRmsSmallRows ? ew::kRmsSmallThreads : ew::kThreads;
    const int gr = (int)std::max<int64_t>(1, std::min<int64_t>((work + bt - 1) / bt, 148 * 32));
#define TI_RMS_REG(TX, T)                                                                      \
  return launch_kernel("rmsnorm launch", ew::rmsnorm_reg_kernel<TX, T, 4>, dim3(gr), dim3(bt),   \
                       0, s, 1, (T*)out, (const TX*)x, (const T*)weight, eps, num_tokens, hidden)
    if (dtype == TI_DTYPE_BF16 && x_dtype == TI_DTYPE_FP32) TI_RMS_REG(float, __nv_bfloat16);
    if (dtype == TI_DTYPE_BF16 && x_dtype == TI_DTYPE_BF16) TI_RMS_REG(__nv_bfloat16, __nv_bfloat16);
    if (dtype == TI_DTYPE_FP16 && x_dtype == TI_DTYPE_FP32) TI_RMS_REG(float, __half);
    if (dtype == TI_DTYPE_FP16 && x_dtype == TI_DTYPE_FP16) TI_RMS_REG(__half, __half);
#undef TI_RMS_REG
    return set_error(TI_ERR_UNSUPPORTED, "rmsnorm: unsupported dtype combination");
  }
  if (dtype == TI_DTYPE_BF16 && x_dtype == TI_DTYPE_FP32)
    return launch_kernel("rmsnorm launch", ew::rmsnorm_kernel<float, __nv_bfloat16>,
                         dim3(g), dim3(ew::kThreads), 0, s, 1,
        (__nv_bfloat16*)out, (const float*)x, (const __nv_bfloat16*)weight, eps, num_tokens, hidden);
  else if (dtype == TI_DTYPE_BF16 && x_dtype == TI_DTYPE_BF16)
    return launch_kernel("rmsnorm launch", ew::rmsnorm_kernel<__nv_bfloat16, __nv_bfloat16>,
                         dim3(g), dim3(ew::kThreads), 0, s, 1,
        (__nv_bfloat16*)out, (const __nv_bfloat16*)x, (const __nv_bfloat16*)weight, eps,
        num_tokens, hidden);
  else if (dtype == TI_DTYPE_FP16 && x_dtype == TI_DTYPE_FP32)
    return launch_kernel("rmsnorm launch", ew::rmsnorm_kernel<float, __half>,
                         dim3(g), dim3(ew::kThreads), 0, s, 1,
        (__half*)out, (const float*)x, (const __half*)weight, eps, num_tokens, hidden);
  else if (dtype == TI_DTYPE_FP16 && x_dtype == TI_DTYPE_FP16)
    return launch_kernel("rmsnorm launch", ew::rmsnorm_kernel<__half, __half>,
                         dim3(g), dim3(ew::kThreads), 0, s, 1,
        (__half*)out, (const __half*)x, (const __half*)weight, eps, num_tokens, hidden);
  else
    return set_error(TI_ERR_UNSUPPORTED, "rmsnorm: unsupported dtype combination");
}

extern "C" int ti_embedding(float* out, const void* table, const int32_t* ids, int num_tokens,
                            int hidden, int64_t vocab, int dtype, void* stream) {
  clear_error();
  if (num_tokens == 0) return TI_OK;
  if (!out || !table || !ids || num_tokens < 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "embedding: null pointer");
  if (hidden % 8 != 0) return set_error(TI_ERR_UNSUPPORTED, "embedding: hidden must be a multiple of 8");
  const int64_t work = (int64_t)num_tokens * (hidden / 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16)
    return launch_kernel("embedding launch", ew::embedding_kernel<__nv_bfloat16>,
                         dim3(ew::grid_for(work)), dim3(ew::kThreads), 0, s, 1,
        out, (const __nv_bfloat16*)table, ids, num_tokens, hidden, vocab);
  else if (dtype == TI_DTYPE_FP16)
    return launch_kernel("embedding launch", ew::embedding_kernel<__half>,
                         dim3(ew::grid_for(work)), dim3(ew::kThreads), 0, s, 1,
        out, (const __half*)table, ids, num_tokens, hidden, vocab);
  else
    return set_error(TI_ERR_UNSUPPORTED, "embedding: dtype must be bf16 or fp16");
}
