// Weight-streaming projections for small token counts (decode batches of <= 64 sequences),
// sm_100a (tcgen05 + TMEM).
//
// At a few dozen tokens the lm_head and the layer projections read each weight once and do
// little math with it: the GEMM kernels' 128-token tiles would be mostly padding, and re-loading
// the activations for every 128-wide weight tile makes them read more activation bytes than
// weight bytes.  Here the roles are swapped: the WEIGHTS are the MMA's M operand (a 128-row tile
// of an nn.Linear weight, streamed once from HBM through a shared-memory ring) and the tokens the
// N operand (all <= 64 of them, loaded once per CTA and kept in shared memory for every tile):
//   D[128 weight rows, NP tokens] = W[n0 : n0+128, K] . X[0 : NP, K]^T   (fp32 in TMEM)
// so a TMEM lane is one output feature and its columns are the tokens.
//
// gemv_argmax_kernel: the greedy lm_head (models/qwen_25.py:250 + the greedy pick of
// engine/scheduler.py:153): persistent over the vocab's 128-row tiles, per tile and token the
// (max, first argmax) over the tile's rows, into the same [tokens, tiles] partials as the GEMM's
// TI_EPI_ARGMAX (ti_argmax_finish reduces them).  bf16 / fp16 weights, or weight-only int8 with a
// float32 scale per row: four converter warps turn each streamed int8 tile (TMA, 64-byte
// swizzle) exactly into bf16 / fp16, one weight row per thread, and store it into tensor memory,
// from where the MMA reads it as its A operand -- the 16-bit tile never passes through shared
// memory, whose bandwidth the earlier shared-memory conversion exhausted.
//   warp 0    TMA: the tokens (once, after the wait on the previous kernel) and the weight tiles
//             (the first stages before that wait: weights are no earlier kernel's output);
//   warp 1    MMA (M=128, N=NP, K=16 per instruction) into one of two TMEM accumulators;
//   warps 2-5 epilogue: tcgen05.ld, scale (int8), per token a warp max / first argmax over its 32
//             rows by shuffles and over the 4 warps through shared memory;
//   warps 6-9 int8 only: converters (shared-memory int8 stage -> tensor-memory A slot).
// Every wait is bounded (TI_DEVERR_GEMM_WAIT on expiry, then the kernel winds down).
#include <algorithm>
#include <type_traits>

#include "capi_internal.h"
#include "common.cuh"
#include "int8_tile.cuh"
#include "tcgen05.cuh"

namespace ti {
namespace gemv {

constexpr int kBM = 128;                 // weight rows per tile (the MMA's M)
constexpr int kBK = 64;                  // K per stage (one 128-byte swizzle row of 16-bit)
constexpr int kWTile = kBM * kBK * 2;    // 16 KB of 16-bit weights
constexpr int kQTile = kBM * kBK;        // 8 KB of int8 weights

template <int NP, bool I8>
struct Cfg {
  static constexpr int kMaxK = 896;                           // tokens held for K <= 896
  static constexpr int kXBytes = kMaxK / kBK * NP * 128;      // the resident token tiles
  // weight tiles in flight (int8: 8 KB each, so more of them for the same bytes in flight)
  static constexpr int kStages = I8 ? (NP <= 32 ? 20 : 13) : 6;
  // int8: converted 16-bit weight tiles live in tensor memory (the MMA's A operand), kConv
  // slots of 32 columns (64 K elements) after the two accumulators
  static constexpr int kConv = I8 ? 4 : 0;
  static constexpr int kRing = kStages * (I8 ? kQTile : kWTile);
  static constexpr int kRed = 4 * NP * 8;                     // (max, argmax) per warp, token
  static constexpr int kBars = (2 * kStages + 2 * kConv + 1 + 4) * 8 + 8;
  static constexpr int kSmem = kXBytes + kRing + kRed + kBars + 1024;
  static constexpr int kAccCols = NP <= 16 ? 32 : 2 * NP;     // two accumulators
  static constexpr int kUsedCols = kAccCols + kConv * (kBK / 2);
  static constexpr int kTmemCols = kUsedCols <= 32 ? 32 : kUsedCols <= 64 ? 64
                                 : kUsedCols <= 128 ? 128 : kUsedCols <= 256 ? 256 : 512;
  static constexpr int kThreads = I8 ? 320 : 192;
  static_assert(kSmem <= 227 * 1024, "shared memory");
  static_assert((kXBytes + kRing) % 1024 == 0, "tile alignment");
  static_assert(kUsedCols <= 512, "tensor memory");
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <typename T, bool I8, int NP>
__global__ void __launch_bounds__(Cfg<NP, I8>::kThreads, 1)
gemv_argmax_kernel(const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap wmap, const float* __restrict__ scale,
                   int M, int K, int ntiles, float* __restrict__ aux_val,
                   int32_t* __restrict__ aux_idx) {
  using C = Cfg<NP, I8>;
  constexpr int S = C::kStages;
  constexpr int CS = C::kConv;
  constexpr int kW = I8 ? kQTile : kWTile;          // bytes of one streamed weight stage
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t xbase = smem_u32(smem);
  const uint32_t wbase = xbase + C::kXBytes;                 // streamed stages
  float2* red = reinterpret_cast<float2*>(smem + C::kXBytes + C::kRing);
  uint8_t* bars = smem + C::kXBytes + C::kRing + C::kRed;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + S * 8;
  const uint32_t cfull0 = empty0 + S * 8;                    // converted tile ready (int8)
  const uint32_t cempty0 = cfull0 + CS * 8;                  // converted tile consumed (int8)
  // (int8) tensor-memory column of converted slot c: C::kAccCols + c * kBK / 2
  const uint32_t xfull = cempty0 + CS * 8;
  const uint32_t accf0 = xfull + 8;
  const uint32_t acce0 = accf0 + 2 * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + (2 * S + 2 * CS + 1 + 4) * 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = K / kBK;

  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < S; ++s) {
        mbar_init(full0 + 8 * s, 1);
        mbar_init(empty0 + 8 * s, I8 ? 4 : 1);   // int8: the converter warps free the stage
      }
      for (int s = 0; s < CS; ++s) {
        mbar_init(cfull0 + 8 * s, 4);
        mbar_init(cempty0 + 8 * s, 1);
      }
      mbar_init(xfull, 1);
      for (int b = 0; b < 2; ++b) {
        mbar_init(accf0 + 8 * b, 1);
        mbar_init(acce0 + 8 * b, 4);
      }
      fence_mbar_init();
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&wmap);
    }
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  // the (tile, K block) sequence this CTA streams: g = local_tile * nkb + kb
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int total = my_tiles * nkb;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      bool ok = true;
      const int pre = min(total, S);
      for (int g = 0; g < pre; ++g) {           // weights first: no earlier kernel writes them
        const int tile = blockIdx.x + (g / nkb) * gridDim.x;
        mbar_arrive_expect_tx(full0 + 8 * g, kW);
        tma_load_2d_hint(wbase + g * kW, &wmap, full0 + 8 * g, (g % nkb) * kBK, tile * kBM, pol_w);
      }
      pdl_wait();                               // the tokens are the previous kernel's output
      mbar_arrive_expect_tx(xfull, nkb * NP * 128);
      for (int kb = 0; kb < nkb; ++kb)
        tma_load_2d_hint(xbase + kb * NP * 128, &xmap, xfull, kb * kBK, 0, pol_x);
      for (int g = pre; g < total && ok; ++g) {
        const int s = g % S;
        if (!mbar_wait(empty0 + 8 * s, ((g / S) & 1) ^ 1, TI_DEVERR_GEMM_WAIT)) { ok = false; break; }
        const int tile = blockIdx.x + (g / nkb) * gridDim.x;
        mbar_arrive_expect_tx(full0 + 8 * s, kW);
        tma_load_2d_hint(wbase + s * kW, &wmap, full0 + 8 * s, (g % nkb) * kBK, tile * kBM, pol_w);
      }
    }
    __syncwarp();
  } else if (warp >= 6) {   // int8 only (the 16-bit kernels have 6 warps)
    if constexpr (I8) {
      // converters: thread = weight row (the TMEM lane its warp may access: warp w reaches lanes
      // 32 (w % 4) ..); its 64 int8 of stage g -> 32 columns of tensor-memory slot g % CS
      // Pipelined by one stage: stage g is loaded and converted while the tensor-memory store
      // of stage g - 1 completes; its slot is announced only then.
      const int r = (warp & 3) * 32 + lane;
      const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
      int pend = -1;                                  // stage whose store is in flight
      for (int g = 0; g < total; ++g) {
        const int s = g % S, c = g % CS;
        if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8 * s, (g / S) & 1, TI_DEVERR_GEMM_WAIT)))
          break;
        uint32_t w[32];
        convert_int8_row<T>(wbase + s * kW, r, w);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);   // the int8 stage may be refilled
        if (pend >= 0) {
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(cfull0 + 8 * (pend % CS));   // slot of stage g - 1 ready
          pend = -1;
        }
        if (g >= CS && !__all_sync(0xffffffffu, mbar_wait(cempty0 + 8 * c, ((g / CS) & 1) ^ 1,
                                                          TI_DEVERR_GEMM_WAIT)))
          break;
        tc_fence_after();
        tmem_st32_u(tmem + lane_base + (uint32_t)(C::kAccCols + c * (kBK / 2)), w);
        pend = g;
      }
      if (pend >= 0) {
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(cfull0 + 8 * (pend % CS));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kBM, NP, std::is_same<T, __nv_bfloat16>::value,
                                           false, false);
      bool ok = mbar_wait(xfull, 0, TI_DEVERR_GEMM_WAIT);
      tc_fence_after();
      int g = 0;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int b = lt & 1, use = lt >> 1;
        if (use > 0 && !mbar_wait(acce0 + 8 * b, (use & 1) ^ 1, TI_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * NP);
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const uint64_t db = smem_desc(xbase + kb * NP * 128);
          if constexpr (I8) {
            const int c = g % CS;
            if (!mbar_wait(cfull0 + 8 * c, (g / CS) & 1, TI_DEVERR_GEMM_WAIT)) { ok = false; break; }
            tc_fence_after();
            const uint32_t ta = tmem + (uint32_t)(C::kAccCols + c * (kBK / 2));
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)   // 16 K elements = 8 columns of A
              tc_mma_tmem_a(d, ta + 8 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            tc_commit(cempty0 + 8 * c);
          } else {
            const int s = g % S;
            if (!mbar_wait(full0 + 8 * s, (g / S) & 1, TI_DEVERR_GEMM_WAIT)) { ok = false; break; }
            tc_fence_after();
            const uint64_t da = smem_desc(wbase + s * kWTile);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              tc_mma(d, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            tc_commit(empty0 + 8 * s);
          }
        }
        tc_commit(accf0 + 8 * b);
      }
    }
    __syncwarp();
  } else if (warp >= 2 && warp < 6) {
    pdl_wait();   // aux_* may be read by an earlier kernel of the stream
    const int quad = warp & 3, et = (int)threadIdx.x - 64;
    for (int lt = 0; lt < my_tiles; ++lt) {
      const int b = lt & 1, use = lt >> 1;
      const int tile = blockIdx.x + lt * gridDim.x;
      if (!__all_sync(0xffffffffu, mbar_wait(accf0 + 8 * b, use & 1, TI_DEVERR_GEMM_WAIT))) break;
      tc_fence_after();
      const int row = tile * kBM + quad * 32 + lane;          // this thread's vocab row
      const float sc = I8 ? __ldg(scale + row) : 1.f;
#pragma unroll 1
      for (int c = 0; c < NP; c += 32) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * NP + c), v);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float bv = v[j] * sc;
          int bi = row;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {                  // larger value, then lower row
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
          }
          if (lane == j) red[quad * NP + c + j] = make_float2(bv, __int_as_float(bi));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * b);             // the accumulator may be reused
      epi_bar();
      if (et < NP && et < M) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 r = red[q * NP + et];
          const int ri = __float_as_int(r.y);
          if (r.x > bv || (r.x == bv && ri < bi)) { bv = r.x; bi = ri; }
        }
        aux_val[(int64_t)et * ntiles + tile] = bv;
        aux_idx[(int64_t)et * ntiles + tile] = bi;
      }
      epi_bar();                                             // red is free for the next tile
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <typename T, bool I8, int NP>
static int launch_argmax(const CUtensorMap& xm, const CUtensorMap& wm, const float* scale, int M,
                         int K, int ntiles, float* aux_val, int32_t* aux_idx, cudaStream_t s) {
  using C = Cfg<NP, I8>;
  auto kern = gemv_argmax_kernel<T, I8, NP>;
  static int set_dev = -1, sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(gemv argmax)");
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    set_dev = dev;
  }
  return launch_kernel("gemv argmax launch", kern, dim3(std::min(sms, ntiles)), dim3(C::kThreads),
                       C::kSmem, s, 1, xm, wm, scale, M, K, ntiles, aux_val, aux_idx);
}

}  // namespace gemv

// Token-count limit and dispatch of the swapped (weight-streaming) greedy lm_head; used by
// ti_gemm's TI_EPI_ARGMAX path (bf16 / fp16 weights, scale == nullptr) and by
// ti_lm_head_argmax_int8 (int8 weights) when M <= 64 and K <= 896.
int gemv_argmax(const void* A, int64_t lda, const void* B, int64_t ldb, bool int8,
                const float* scale, int M, int N, int K, float* aux_val, int32_t* aux_idx,
                int dtype, cudaStream_t s) {
  const int np = M <= 32 ? 32 : 64;
  CUtensorMap xm, wm;
  const CUtensorMapDataType ty = dtype == TI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)lda * 2};
    cuuint32_t box[2] = {(cuuint32_t)gemv::kBK, (cuuint32_t)np};
    cuuint32_t es[2] = {1, 1};
    int rc = encode_tensor_map_2d(&xm, ty, const_cast<void*>(A), dims, strides, box, es,
                                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (rc) return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)(int8 ? ldb : ldb * 2)};
    cuuint32_t box[2] = {(cuuint32_t)gemv::kBK, (cuuint32_t)gemv::kBM};
    cuuint32_t es[2] = {1, 1};
    int rc = encode_tensor_map_2d(&wm, int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : ty,
                                  const_cast<void*>(B), dims, strides, box, es,
                                  int8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (rc) return rc;
  }
  const int ntiles = N / gemv::kBM;
  const bool bf = dtype == TI_DTYPE_BF16;
#define TI_GEMV_ARGMAX(T, I8)                                                                  \
  return np == 32 ? gemv::launch_argmax<T, I8, 32>(xm, wm, scale, M, K, ntiles, aux_val, aux_idx, s) \
                  : gemv::launch_argmax<T, I8, 64>(xm, wm, scale, M, K, ntiles, aux_val, aux_idx, s);
  if (bf && int8) { TI_GEMV_ARGMAX(__nv_bfloat16, true) }
  if (bf) { TI_GEMV_ARGMAX(__nv_bfloat16, false) }
  if (int8) { TI_GEMV_ARGMAX(__half, true) }
  TI_GEMV_ARGMAX(__half, false)
#undef TI_GEMV_ARGMAX
}

}  // namespace ti
