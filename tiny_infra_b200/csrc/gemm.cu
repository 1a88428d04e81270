// Projection GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   D[M, N] = A[M, K] . B[N, K]^T      A = activations (bf16/fp16, K-major)
//                                      B = nn.Linear weight [out, in] (K-major)
//
// Replaces the reference's nn.Linear projections (models/qwen_25.py:46-49,66-68,130,136-151,237)
// and fuses what follows each of them:
//   TI_EPI_STORE     out = D (+ bias)                       q/k/v projection (bias), logits
//   TI_EPI_SWIGLU    out = silu(gate) * up                   gate/up projection + SwiGLU
//                    (fused_swiglu.cu:39-50; no [T, 2I] intermediate, no torch.cat)
//   TI_EPI_RESIDUAL  x_f32 += D                              o_proj / down_proj + residual add
//                    (models/qwen_25.py:182,191), split-K partials reduced with red.add
//   TI_EPI_ARGMAX    per-row (max, first argmax) of each N tile, logits optionally stored
//                    (greedy decoding without writing [M, vocab] logits)
//
// Kernel structure (one 128 x BN output tile per CTA, 192 threads):
//   warp 0    one elected thread issues TMA tile loads (A: 128 x 64, B: BN x 64, SWIZZLE_128B)
//             into a STAGES-deep shared-memory ring, mbarrier full/empty handshake;
//   warp 1    one elected thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN,
//             K=16 per instruction) from shared-memory descriptors into a TMEM accumulator and
//             frees each stage with tcgen05.commit;
//   warps 2-5 epilogue: tcgen05.ld 32 columns at a time from the TMEM lanes of their quadrant
//             (warp w reads rows 32*(w%4)..+31), apply the fused epilogue, store.
// Every wait is bounded (about 2 s): on expiry the kernel records TI_DEVERR_GEMM_WAIT, skips
// the rest of its work, frees its TMEM and returns.
#include <algorithm>
#include <type_traits>
#include <mutex>
#include <unordered_map>

#include "capi_internal.h"
#include "common.cuh"

namespace ti {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;                 // one 128-byte swizzle atom of bf16 per row
constexpr int kThreads = 192;

// ---- tcgen05 wrappers --------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 32 columns of 32-bit: thread t of the warp receives 32 consecutive columns of
// TMEM lane (quadrant base + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, K-major operand in the canonical SWIZZLE_128B layout:
// rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), LBO unused (1), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor for kind::f16: fp32 accumulator, A/B bf16 (1) or fp16 (0), both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t instr_desc(int n, bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// ---- epilogues ----------------------------------------------------------------------------
struct EpiArgs {
  void* out;
  int64_t ldo;
  const void* bias;
  float* aux_val;     // argmax: [M, ntiles]
  int32_t* aux_idx;
  int M, N;
  int ntiles;
  int atomic;         // residual: split-K > 1
  // QKV + RoPE + KV append (TI_EPI_QKV_ROPE): one 64-wide N tile is one head
  const int32_t* pos;
  const int64_t* slot_mapping;
  const float* cos;
  const float* sin;
  void* k_cache;
  void* v_cache;
  int num_heads, num_kv_heads, block_size;
};

template <typename T>
__device__ __forceinline__ void store_row_chunk(T* dst, const float* v) {   // 32 values
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = Elem<T>::pack2(v[i * 8 + 2 * j], v[i * 8 + 2 * j + 1]);
    *reinterpret_cast<uint4*>(dst + i * 8) = u;
  }
}

template <typename T, int BN, int KIND>
__device__ __forceinline__ void epilogue(const EpiArgs& e, uint32_t tmem_row, int row, int n0,
                                         int tile_n) {
  const bool live = row < e.M;
  if constexpr (KIND == TI_EPI_STORE) {
    T* o = reinterpret_cast<T*>(e.out) + (int64_t)row * e.ldo + n0;
    const T* b = reinterpret_cast<const T*>(e.bias);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32(tmem_row + c, v);
      if (b) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += Elem<T>::to_f(b[n0 + c + i]);
      }
      if (live) store_row_chunk<T>(o + c, v);
    }
  } else if constexpr (KIND == TI_EPI_SWIGLU) {
    // tile columns [0, BN/2) are gate rows g0..g0+BN/2-1, [BN/2, BN) the matching up rows
    T* o = reinterpret_cast<T*>(e.out) + (int64_t)row * e.ldo + n0 / 2;
#pragma unroll 1
    for (int c = 0; c < BN / 2; c += 32) {
      float g[32], u[32];
      tmem_ld32(tmem_row + c, g);
      tmem_ld32(tmem_row + BN / 2 + c, u);
#pragma unroll
      for (int i = 0; i < 32; ++i) g[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
      if (live) store_row_chunk<T>(o + c, g);
    }
  } else if constexpr (KIND == TI_EPI_RESIDUAL) {
    float* x = reinterpret_cast<float*>(e.out) + (int64_t)row * e.ldo + n0;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32(tmem_row + c, v);
      if (!live) continue;
      if (e.atomic) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(x + c + i),
                       "f"(v[i]), "f"(v[i + 1]), "f"(v[i + 2]), "f"(v[i + 3])
                       : "memory");
      } else {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 a = *reinterpret_cast<float4*>(x + c + i);
          a.x += v[i]; a.y += v[i + 1]; a.z += v[i + 2]; a.w += v[i + 3];
          *reinterpret_cast<float4*>(x + c + i) = a;
        }
      }
    }
  } else if constexpr (KIND == TI_EPI_QKV_ROPE) {
    // BN == head_dim == 64: columns [0,32) and [32,64) of the tile are the rotate-half pairs.
    // RoPE runs on the fp32 accumulators (+bias) and each value is rounded once, q into `out`,
    // k and v straight into the pool (src/fused_rope.cu:37-50, engine/cache_manager.py:95-99).
    static_assert(BN == 64, "one head per tile");
    const int head = n0 / 64;
    float x1[32], x2[32];
    tmem_ld32(tmem_row, x1);
    tmem_ld32(tmem_row + 32, x2);
    if (!live) return;
    const T* b = reinterpret_cast<const T*>(e.bias);
    if (b) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        x1[i] += Elem<T>::to_f(b[n0 + i]);
        x2[i] += Elem<T>::to_f(b[n0 + 32 + i]);
      }
    }
    if (head < e.num_heads + e.num_kv_heads) {
      const float* cs = e.cos + (int64_t)e.pos[row] * 32;
      const float* sn = e.sin + (int64_t)e.pos[row] * 32;
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 c = *reinterpret_cast<const float4*>(cs + i);
        const float4 s = *reinterpret_cast<const float4*>(sn + i);
        const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = x1[i + j], bb = x2[i + j];
          x1[i + j] = a * cc[j] - bb * ss[j];
          x2[i + j] = a * ss[j] + bb * cc[j];
        }
      }
    }
    if (head < e.num_heads) {
      T* o = reinterpret_cast<T*>(e.out) + (int64_t)row * e.ldo + n0;
      store_row_chunk<T>(o, x1);
      store_row_chunk<T>(o + 32, x2);
    } else {
      const int64_t slot = e.slot_mapping[row];
      if (slot < 0) return;
      const bool is_k = head < e.num_heads + e.num_kv_heads;
      const int kh = is_k ? head - e.num_heads : head - e.num_heads - e.num_kv_heads;
      T* pool = reinterpret_cast<T*>(is_k ? e.k_cache : e.v_cache);
      T* dst = pool + (((slot / e.block_size) * e.num_kv_heads + kh) * e.block_size +
                       slot % e.block_size) * 64;
      store_row_chunk<T>(dst, x1);
      store_row_chunk<T>(dst + 32, x2);
    }
  } else {   // TI_EPI_ARGMAX
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    T* o = e.out ? reinterpret_cast<T*>(e.out) + (int64_t)row * e.ldo + n0 : nullptr;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32(tmem_row + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (v[i] > best) { best = v[i]; bidx = n0 + c + i; }   // first index on ties
      if (o && live) store_row_chunk<T>(o + c, v);
    }
    if (live) {
      e.aux_val[(int64_t)row * e.ntiles + tile_n] = best;
      e.aux_idx[(int64_t)row * e.ntiles + tile_n] = bidx;
    }
  }
}

template <int BN, int STAGES>
struct Cfg {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStage = kABytes + kBBytes;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = STAGES * kStage + (2 * STAGES + 1) * 8 + 16 + 1024;
};

template <typename T, int BN, int STAGES, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
            int K, int kb_per_split, EpiArgs e) {
  using C = Cfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t full0 = sbase + STAGES * C::kStage;
  const uint32_t empty0 = full0 + STAGES * 8;
  const uint32_t accum = empty0 + STAGES * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + STAGES * C::kStage + (2 * STAGES + 1) * 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile_n = blockIdx.x;
  const int n0 = tile_n * BN, m0 = blockIdx.y * BM;
  const int nkb = K / BK;
  const int kb0 = blockIdx.z * kb_per_split;
  const int kb1 = min(nkb, kb0 + kb_per_split);
  const int nk = max(0, kb1 - kb0);

  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s) {
        mbar_init(full0 + 8 * s, 1);
        mbar_init(empty0 + 8 * s, 1);
      }
      mbar_init(accum, 1);
      fence_mbar_init();
      prefetch_tensormap(&amap);
      prefetch_tensormap(&bmap);
    }
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_last();    // activations: re-read by many CTAs
      const uint64_t pol_b = l2_policy_evict_first();   // weights: streamed once
      for (int it = 0; it < nk; ++it) {
        const int s = it % STAGES;
        if (it >= STAGES && !mbar_wait(empty0 + 8 * s, ((it / STAGES) & 1) ^ 1, TI_DEVERR_GEMM_WAIT))
          break;
        mbar_arrive_expect_tx(full0 + 8 * s, C::kStage);
        const uint32_t sa = sbase + s * C::kStage;
        const int kx = (kb0 + it) * BK;
        tma_load_2d_hint(sa, &amap, full0 + 8 * s, kx, m0, pol_a);
        tma_load_2d_hint(sa + C::kABytes, &bmap, full0 + 8 * s, kx, n0, pol_b);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BN, std::is_same<T, __nv_bfloat16>::value);
      bool ok = true;
      for (int it = 0; it < nk && ok; ++it) {
        const int s = it % STAGES;
        ok = mbar_wait(full0 + 8 * s, (it / STAGES) & 1, TI_DEVERR_GEMM_WAIT);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sa = sbase + s * C::kStage;
        const uint64_t da = smem_desc(sa), db = smem_desc(sa + C::kABytes);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)   // +32 bytes along K inside the swizzle atom
          tc_mma(tmem, da + 2 * k, db + 2 * k, idesc, (it > 0 || k > 0) ? 1u : 0u);
        tc_commit(empty0 + 8 * s);
      }
      tc_commit(accum);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int row = m0 + quad * 32 + lane;
    const bool ok = mbar_wait(accum, 0, TI_DEVERR_GEMM_WAIT);
    tc_fence_after();
    if (ok && nk > 0) epilogue<T, BN, KIND>(e, tmem + ((uint32_t)(quad * 32) << 16), row, n0, tile_n);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---- host side ----------------------------------------------------------------------------
struct MapKey {
  const void* p;
  int64_t rows, cols, ld;
  int box_rows, dtype;
  bool operator==(const MapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && ld == o.ld &&
           box_rows == o.box_rows && dtype == o.dtype;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.p);
    h ^= std::hash<int64_t>()(k.rows * 1315423911LL + k.cols * 2654435761LL + k.ld) + 0x9e3779b9 + (h << 6);
    return h ^ (size_t)(k.box_rows * 131 + k.dtype);
  }
};

// K-major operand [rows, cols=K] with leading dimension ld elements; box BK x box_rows.
static int operand_map(CUtensorMap* m, const void* p, int64_t rows, int64_t cols, int64_t ld,
                       int box_rows, int dtype) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{p, rows, cols, ld, box_rows, dtype};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) { *m = it->second; return TI_OK; }
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {BK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  int rc = encode_tensor_map_2d(m, dtype == TI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                const_cast<void*>(p), dims, strides, box, es,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, *m);
  return TI_OK;
}

template <typename T, int BN, int STAGES, int KIND>
static int launch_t(const CUtensorMap& am, const CUtensorMap& bm, int M, int N, int K, int splits,
                    const EpiArgs& e, cudaStream_t s) {
  using C = Cfg<BN, STAGES>;
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t err = cudaFuncSetAttribute(gemm_kernel<T, BN, STAGES, KIND>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (err != cudaSuccess) return set_cuda_error(err, "cudaFuncSetAttribute(gemm)");
    set_dev = dev;
  }
  const int nkb = K / BK;
  const int per = (nkb + splits - 1) / splits;
  const int z = (nkb + per - 1) / per;   // no empty split
  dim3 grid(N / BN, (M + BM - 1) / BM, z);
  gemm_kernel<T, BN, STAGES, KIND><<<grid, kThreads, C::kSmem, s>>>(am, bm, K, per, e);
  count_launch();
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? TI_OK : set_cuda_error(err, "gemm launch");
}

template <typename T>
static int launch_qkv(const CUtensorMap& am, const CUtensorMap& bm, int M, int N, int K,
                      const EpiArgs& e, cudaStream_t s) {
  return launch_t<T, 64, 4, TI_EPI_QKV_ROPE>(am, bm, M, N, K, 1, e, s);
}

template <typename T, int KIND>
static int dispatch_bn(int bn, const CUtensorMap& am, const CUtensorMap& bm, int M, int N, int K,
                       int splits, const EpiArgs& e, cudaStream_t s) {
  switch (bn) {
    case 64: return launch_t<T, 64, 4, KIND>(am, bm, M, N, K, splits, e, s);
    case 128: return launch_t<T, 128, 3, KIND>(am, bm, M, N, K, splits, e, s);
    case 256: return launch_t<T, 256, 3, KIND>(am, bm, M, N, K, splits, e, s);
    default: return set_error(TI_ERR_UNSUPPORTED, "gemm: block_n must be 64, 128 or 256");
  }
}

}  // namespace gemm
}  // namespace ti

using namespace ti;

extern "C" int ti_gemm(int epilogue, const void* A, int64_t lda, const void* B, int64_t ldb,
                       int M, int N, int K, void* out, int64_t ldo, const void* bias,
                       float* aux_val, int32_t* aux_idx, int dtype, int block_n, int split_k,
                       void* stream) {
  clear_error();
  if (M == 0) return TI_OK;
  if (!A || !B || M < 0 || N <= 0 || K <= 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "gemm: null operand or bad size");
  if (dtype != TI_DTYPE_BF16 && dtype != TI_DTYPE_FP16)
    return set_error(TI_ERR_UNSUPPORTED, "gemm: dtype must be bf16 or fp16");
  if (block_n <= 0) block_n = 128;
  if (N % block_n || K % gemm::BK)
    return set_error(TI_ERR_UNSUPPORTED, "gemm: N must be a multiple of block_n and K of 64");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15 || (lda % 8) || (ldb % 8))
    return set_error(TI_ERR_INVALID_ARGUMENT, "gemm: operands must be 16-byte aligned with ld % 8 == 0");
  if (split_k <= 0) split_k = 1;
  if (split_k > 1 && epilogue != TI_EPI_RESIDUAL)
    return set_error(TI_ERR_UNSUPPORTED, "gemm: split-K only with the residual epilogue");
  if (epilogue == TI_EPI_ARGMAX && (!aux_val || !aux_idx))
    return set_error(TI_ERR_INVALID_ARGUMENT, "gemm: argmax epilogue needs aux_val / aux_idx");
  if (epilogue != TI_EPI_ARGMAX && !out)
    return set_error(TI_ERR_INVALID_ARGUMENT, "gemm: null output");
  if (epilogue == TI_EPI_SWIGLU && block_n < 64)
    return set_error(TI_ERR_UNSUPPORTED, "gemm: SwiGLU epilogue needs block_n >= 64");
  if (out && ((reinterpret_cast<uintptr_t>(out) & 15) || (ldo % 8)))
    return set_error(TI_ERR_INVALID_ARGUMENT, "gemm: output must be 16-byte aligned, ldo % 8 == 0");
  if ((int64_t)((M + gemm::BM - 1) / gemm::BM) > 65535)
    return set_error(TI_ERR_UNSUPPORTED, "gemm: M too large");

  CUtensorMap am, bm;
  int rc = gemm::operand_map(&am, A, M, K, lda, gemm::BM, dtype);
  if (rc) return rc;
  rc = gemm::operand_map(&bm, B, N, K, ldb, block_n, dtype);
  if (rc) return rc;
  gemm::EpiArgs e{};
  e.out = out; e.ldo = ldo; e.bias = bias; e.aux_val = aux_val; e.aux_idx = aux_idx;
  e.M = M; e.N = N; e.ntiles = N / block_n; e.atomic = split_k > 1 ? 1 : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
#define TI_GEMM_KIND(T)                                                                       \
  switch (epilogue) {                                                                         \
    case TI_EPI_STORE: return gemm::dispatch_bn<T, TI_EPI_STORE>(block_n, am, bm, M, N, K, split_k, e, s); \
    case TI_EPI_SWIGLU: return gemm::dispatch_bn<T, TI_EPI_SWIGLU>(block_n, am, bm, M, N, K, split_k, e, s); \
    case TI_EPI_RESIDUAL: return gemm::dispatch_bn<T, TI_EPI_RESIDUAL>(block_n, am, bm, M, N, K, split_k, e, s); \
    case TI_EPI_ARGMAX: return gemm::dispatch_bn<T, TI_EPI_ARGMAX>(block_n, am, bm, M, N, K, split_k, e, s); \
    default: return set_error(TI_ERR_INVALID_ARGUMENT, "gemm: unknown epilogue");             \
  }
  if (dtype == TI_DTYPE_BF16) { TI_GEMM_KIND(__nv_bfloat16) }
  TI_GEMM_KIND(__half)
#undef TI_GEMM_KIND
}

extern "C" int ti_gemm_qkv_rope(const void* A, int64_t lda, const void* W, int64_t ldw,
                                const void* bias, int M, int hidden, int num_heads,
                                int num_kv_heads, int head_dim, void* q_out, int64_t ldq,
                                void* k_cache, void* v_cache, const int64_t* slot_mapping,
                                const float* cos, const float* sin, const int32_t* pos,
                                int block_size, int dtype, void* stream) {
  clear_error();
  if (M == 0) return TI_OK;
  if (!A || !W || !q_out || !k_cache || !v_cache || !slot_mapping || !cos || !sin || !pos ||
      M < 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "gemm_qkv_rope: null pointer");
  if (head_dim != 64) return set_error(TI_ERR_UNSUPPORTED, "gemm_qkv_rope: head_dim must be 64");
  if (dtype != TI_DTYPE_BF16 && dtype != TI_DTYPE_FP16)
    return set_error(TI_ERR_UNSUPPORTED, "gemm_qkv_rope: dtype must be bf16 or fp16");
  if (hidden % gemm::BK || (lda % 8) || (ldw % 8) || (ldq % 8) ||
      ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W) |
        reinterpret_cast<uintptr_t>(q_out) | reinterpret_cast<uintptr_t>(k_cache) |
        reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(cos) |
        reinterpret_cast<uintptr_t>(sin)) & 15))
    return set_error(TI_ERR_INVALID_ARGUMENT, "gemm_qkv_rope: alignment");
  const int N = (num_heads + 2 * num_kv_heads) * head_dim;
  CUtensorMap am, bm;
  int rc = gemm::operand_map(&am, A, M, hidden, lda, gemm::BM, dtype);
  if (rc) return rc;
  rc = gemm::operand_map(&bm, W, N, hidden, ldw, 64, dtype);
  if (rc) return rc;
  gemm::EpiArgs e{};
  e.out = q_out; e.ldo = ldq; e.bias = bias; e.M = M; e.N = N; e.ntiles = N / 64;
  e.pos = pos; e.slot_mapping = slot_mapping; e.cos = cos; e.sin = sin;
  e.k_cache = k_cache; e.v_cache = v_cache;
  e.num_heads = num_heads; e.num_kv_heads = num_kv_heads; e.block_size = block_size;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16) return gemm::launch_qkv<__nv_bfloat16>(am, bm, M, N, hidden, e, s);
  return gemm::launch_qkv<__half>(am, bm, M, N, hidden, e, s);
}
