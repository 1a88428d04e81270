// Weight-only INT8 lm_head for greedy decoding, sm_100a (tcgen05 + TMEM).
//
// The reference lists weight-only INT8/INT4 projections as its next step (README.md:156-157);
// here it is applied to the largest single weight read of a decode step, the tied lm_head
// (151936 x 896, 272 MB in bf16, models/qwen_25.py:237,250).  Each vocab row n is stored as
// int8 q[n, k] with one float32 scale s[n] = max_k |w[n, k]| / 127 (ti_quantize_rows_int8),
// halving the bytes streamed per step.  The logit is s[n] * sum_k x[k] q[n, k]: the int8 values
// convert exactly to bf16, the tensor cores accumulate the exact products in fp32 and the
// epilogue applies the scale before the per-tile argmax, as TI_EPI_ARGMAX does for bf16.
//
// Persistent kernel, one CTA per SM looping over the 128-column vocab tiles, M <= 256 tokens:
//   warp 0    TMA: per K block the activations (256 x 64 bf16, SWIZZLE_128B) and the int8 tile
//             (128 rows x 64 bytes, row-major) into a 3-stage ring;
//   warps 6-9 convert the int8 tile into the bf16 B tile in the canonical SWIZZLE_128B K-major
//             layout (convert_int8_tile, int8_tile.cuh), fence the writes to the async proxy and
//             arrive on the stage's "converted" barrier;
//   warp 1    MMA: two tcgen05.mma M=128 N=128 (both 128-row halves of the tokens) per K step
//             into one of two 256-column TMEM accumulator pairs, commits stages and buffers;
//   warps 2-5 epilogue: tcgen05.ld, multiply by the tile's scales, (max, first argmax) per row
//             and tile into aux_val / aux_idx, overlapping the next tile's MMAs.
// Every wait is bounded (TI_DEVERR_GEMM_WAIT on expiry, then the kernel winds down).
#include <algorithm>
#include <type_traits>

#include "capi_internal.h"
#include "common.cuh"
#include "int8_tile.cuh"
#include "tcgen05.cuh"

namespace ti {
namespace lmi8 {

constexpr int kBN = 128;                              // vocab rows per tile
constexpr int kBK = 64;                               // K per stage
constexpr int kStages = 3;
constexpr int kABytes = 256 * kBK * 2;                // 32 KB (two 128-row halves)
constexpr int kBBytes = kBN * kBK * 2;                // 16 KB bf16, written by the converters
constexpr int kQBytes = kBN * kBK;                    // 8 KB int8, written by TMA
constexpr int kStage = kABytes + kBBytes + kQBytes;   // 56 KB (A and B 1024-byte aligned)
constexpr int kRing = kStages * kStage;               // 168 KB
constexpr int kBars = (3 * kStages + 4) * 8 + 8;      // full, conv, empty; accf / acce x 2; slot
constexpr int kSmem = kRing + kBars + 1024;
constexpr int kThreads = 320;
constexpr int kTmemCols = 512;
static_assert(kStage % 1024 == 0, "stage alignment");

__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
lmhead_argmax_i8_kernel(const __grid_constant__ CUtensorMap amap,
                        const __grid_constant__ CUtensorMap qmap, const float* __restrict__ scale,
                        int M, int K, int ntiles, float* __restrict__ aux_val,
                        int32_t* __restrict__ aux_idx) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* bars = smem + kRing;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t conv0 = full0 + kStages * 8;
  const uint32_t empty0 = conv0 + kStages * 8;
  const uint32_t accf0 = empty0 + kStages * 8;
  const uint32_t acce0 = accf0 + 2 * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + (3 * kStages + 4) * 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = K / kBK;

  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < kStages; ++s) {
        mbar_init(full0 + 8 * s, 1);
        mbar_init(conv0 + 8 * s, 4);      // one arrival per converter warp
        mbar_init(empty0 + 8 * s, 1);
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(accf0 + 8 * b, 1);
        mbar_init(acce0 + 8 * b, 4);      // one arrival per epilogue warp
      }
      fence_mbar_init();
      prefetch_tensormap(&amap);
      prefetch_tensormap(&qmap);
    }
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_last();    // activations: re-read for every tile
      const uint64_t pol_q = l2_policy_evict_first();   // weights: streamed once
      int g = 0;
      bool waited = false, ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kStages;
          if (g >= kStages &&
              !mbar_wait(empty0 + 8 * s, ((g / kStages) & 1) ^ 1, TI_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full0 + 8 * s, kABytes + kQBytes);
          const uint32_t st = sbase + s * kStage;
          tma_load_2d_hint(st + kABytes + kBBytes, &qmap, full0 + 8 * s, kb * kBK, tile * kBN,
                           pol_q);
          if (!waited) { pdl_wait(); waited = true; }   // A is the previous kernel's output
          tma_load_2d_hint(st, &amap, full0 + 8 * s, kb * kBK, 0, pol_a);
        }
      }
      if (!waited) pdl_wait();
    }
    __syncwarp();
  } else if (warp >= 6) {
    // converters: the stage's int8 tile -> its bf16 / fp16 B tile
    const int t = (int)threadIdx.x - 192;
    int g = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb, ++g) {
        const int s = g % kStages;
        if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8 * s, (g / kStages) & 1,
                                                TI_DEVERR_GEMM_WAIT))) {
          ok = false;
          break;
        }
        const uint32_t bt = sbase + s * kStage + kABytes;
        const uint32_t qt = bt + kBBytes;
        convert_int8_tile<T>(qt, bt, t);
        fence_async_shared();             // generic-proxy writes -> the tensor cores' reads
        __syncwarp();
        if (lane == 0) mbar_arrive(conv0 + 8 * s);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(128, kBN, std::is_same<T, __nv_bfloat16>::value,
                                           false, false);
      int g = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++local) {
        const int b = local & 1, use = local >> 1;
        if (use > 0 && !mbar_wait(acce0 + 8 * b, (use & 1) ^ 1, TI_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(b * 256), d1 = d0 + 128;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1;
          if (!mbar_wait(conv0 + 8 * s, ph, TI_DEVERR_GEMM_WAIT) ||
              !mbar_wait(full0 + 8 * s, ph, TI_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + s * kStage;
          const uint64_t da = smem_desc(st), da1 = smem_desc(st + 128 * 128),
                         db = smem_desc(st + kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            tc_mma(d0, da + 2 * k, db + 2 * k, idesc, acc);
            tc_mma(d1, da1 + 2 * k, db + 2 * k, idesc, acc);
          }
          tc_commit(empty0 + 8 * s);
        }
        tc_commit(accf0 + 8 * b);
      }
    }
    __syncwarp();
  } else {
    pdl_wait();   // aux_* may be read by an earlier kernel of the stream
    const int quad = warp & 3;
    int local = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++local) {
      const int b = local & 1, use = local >> 1;
      if (!__all_sync(0xffffffffu, mbar_wait(accf0 + 8 * b, use & 1, TI_DEVERR_GEMM_WAIT))) break;
      tc_fence_after();
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const uint32_t trow =
            tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * 256 + half * 128);
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll 1
        for (int c = 0; c < kBN; c += 32) {
          float v[32];
          tmem_ld32(trow + c, v);
          const float4* sp = reinterpret_cast<const float4*>(scale + (int64_t)tile * kBN + c);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 sc = __ldg(sp + q4);     // the same address in every lane
            const float sv[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float x = v[4 * q4 + j] * sv[j];
              const int idx = tile * kBN + c + 4 * q4 + j;
              if (x > bv || (x == bv && idx < bi)) { bv = x; bi = idx; }
            }
          }
        }
        const int row = half * 128 + quad * 32 + lane;
        if (row < M) {
          aux_val[(int64_t)row * ntiles + tile] = bv;
          aux_idx[(int64_t)row * ntiles + tile] = bi;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * b);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Per-row symmetric int8 quantisation: one warp per row, scale = max|w| / 127 (1 for an all-zero
// row), q = round-to-nearest-even(w / scale) (IEEE division), clamped to [-127, 127].
template <typename T>
__global__ void quantize_rows_kernel(const T* __restrict__ w, int64_t ldw, int rows, int cols,
                                     int8_t* __restrict__ q, int64_t ldq,
                                     float* __restrict__ scale) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += nw) {
    const T* wr = w + (int64_t)r * ldw;
    float amax = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
      const uint4 raw = *reinterpret_cast<const uint4*>(wr + c);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = Elem<T>::unpack2(u[i]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
    amax = warp_max(amax);
    const float s = amax > 0.f ? amax / 127.f : 1.f;
    for (int c = lane * 8; c < cols; c += 256) {
      const uint4 raw = *reinterpret_cast<const uint4*>(wr + c);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = Elem<T>::unpack2(u[i]);
        const int a = (int)fminf(127.f, fmaxf(-127.f, rintf(f.x / s)));
        const int b = (int)fminf(127.f, fmaxf(-127.f, rintf(f.y / s)));
        packed[i >> 1] |= ((uint32_t)(a & 0xff) << (16 * (i & 1))) |
                          ((uint32_t)(b & 0xff) << (16 * (i & 1) + 8));
      }
      *reinterpret_cast<uint2*>(q + (int64_t)r * ldq + c) = make_uint2(packed[0], packed[1]);
    }
    if (lane == 0) scale[r] = s;
  }
}

}  // namespace lmi8
}  // namespace ti

using namespace ti;

extern "C" int ti_quantize_rows_int8(const void* w, int64_t ldw, int rows, int cols, int8_t* q,
                                     int64_t ldq, float* scale, int dtype, void* stream) {
  clear_error();
  if (rows == 0) return TI_OK;
  if (!w || !q || !scale || rows < 0 || cols <= 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "quantize_rows_int8: null pointer or bad size");
  if (dtype != TI_DTYPE_BF16 && dtype != TI_DTYPE_FP16)
    return set_error(TI_ERR_UNSUPPORTED, "quantize_rows_int8: dtype must be bf16 or fp16");
  if (cols % 8 || ldw % 8 || ldq % 8 ||
      (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(q) & 7))
    return set_error(TI_ERR_INVALID_ARGUMENT, "quantize_rows_int8: cols / strides must be multiples of 8, aligned rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int blocks = std::min(148 * 8, (rows + 7) / 8);
  if (dtype == TI_DTYPE_BF16)
    return launch_kernel("quantize_rows_int8 launch", lmi8::quantize_rows_kernel<__nv_bfloat16>,
                         dim3(blocks), dim3(256), 0, s, 1, (const __nv_bfloat16*)w, ldw, rows,
                         cols, q, ldq, scale);
  return launch_kernel("quantize_rows_int8 launch", lmi8::quantize_rows_kernel<__half>,
                       dim3(blocks), dim3(256), 0, s, 1, (const __half*)w, ldw, rows, cols, q,
                       ldq, scale);
}

extern "C" int ti_lm_head_argmax_int8(const void* A, int64_t lda, const int8_t* Bq, int64_t ldb,
                                      const float* scale, int M, int N, int K, float* aux_val,
                                      int32_t* aux_idx, int dtype, void* stream) {
  clear_error();
  if (M == 0) return TI_OK;
  if (!A || !Bq || !scale || !aux_val || !aux_idx || M < 0 || N <= 0 || K <= 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "lm_head_argmax_int8: null pointer or bad size");
  if (M > 256) return set_error(TI_ERR_UNSUPPORTED, "lm_head_argmax_int8: at most 256 rows");
  if (dtype != TI_DTYPE_BF16 && dtype != TI_DTYPE_FP16)
    return set_error(TI_ERR_UNSUPPORTED, "lm_head_argmax_int8: dtype must be bf16 or fp16");
  if (N % lmi8::kBN || K % lmi8::kBK)
    return set_error(TI_ERR_UNSUPPORTED, "lm_head_argmax_int8: N % 128 == 0 and K % 64 == 0 required");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(Bq) |
       reinterpret_cast<uintptr_t>(scale)) & 15 || (lda % 8) || (ldb % 16))
    return set_error(TI_ERR_INVALID_ARGUMENT, "lm_head_argmax_int8: operands must be 16-byte aligned (lda % 8, ldb % 16)");
  if (M <= kGemvMaxTokens && K <= kGemvMaxK)   // few tokens: the weight-streaming kernel
    return gemv_argmax(A, lda, Bq, ldb, true, scale, M, N, K, aux_val, aux_idx, dtype,
                       reinterpret_cast<cudaStream_t>(stream));
  CUtensorMap am, qm;
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)lda * 2};
    cuuint32_t box[2] = {(cuuint32_t)lmi8::kBK, 256};
    cuuint32_t es[2] = {1, 1};
    const CUtensorMapDataType ty = dtype == TI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    int rc = encode_tensor_map_2d(&am, ty, const_cast<void*>(A), dims, strides, box, es,
                                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (rc) return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)ldb};
    cuuint32_t box[2] = {(cuuint32_t)lmi8::kBK, (cuuint32_t)lmi8::kBN};
    cuuint32_t es[2] = {1, 1};
    int rc = encode_tensor_map_2d(&qm, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<int8_t*>(Bq),
                                  dims, strides, box, es, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (rc) return rc;
  }
  static int set_dev[2] = {-1, -1}, sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  const int di = dtype == TI_DTYPE_BF16 ? 0 : 1;
  auto kern = di == 0 ? lmi8::lmhead_argmax_i8_kernel<__nv_bfloat16>
                      : lmi8::lmhead_argmax_i8_kernel<__half>;
  if (set_dev[di] != dev) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           lmi8::kSmem);
    if (err != cudaSuccess) return set_cuda_error(err, "cudaFuncSetAttribute(lm_head int8)");
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    set_dev[di] = dev;
  }
  const int ntiles = N / lmi8::kBN;
  return launch_kernel("lm_head int8 launch", kern, dim3(std::min(sms, ntiles)),
                       dim3(lmi8::kThreads), lmi8::kSmem, reinterpret_cast<cudaStream_t>(stream),
                       1, am, qm, scale, M, K, ntiles, aux_val, aux_idx);
}
