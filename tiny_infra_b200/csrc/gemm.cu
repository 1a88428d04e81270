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
//   TI_EPI_SWIGLU16  the same with gate/up rows interleaved in groups of 8, so that any tile
//                    width that is a multiple of 16 pairs them: decode batches take 80- or
//                    144-wide tiles that fill the SMs in one wave
//   TI_EPI_RESIDUAL  x_f32 += D                              o_proj / down_proj + residual add
//                    (models/qwen_25.py:182,191), one red.add per element and K slice
//   TI_EPI_RESIDUAL_DET  the same with the K slices summed in a fixed order on a cluster
//                    first (one add per element: x is bit-reproducible)
//   TI_EPI_ARGMAX    per-row (max, first argmax) of each N tile, logits optionally stored
//                    (greedy decoding without writing [M, vocab] logits)
//   TI_EPI_QKV_ROPE  bias + RoPE on q and k, q stored, k and v written into the paged pool
//
// Kernel structure (one 128 x BN output tile per cluster of CL CTAs, 192 threads per CTA):
//   warp 0    set-up (barriers, TMEM allocation);
//   warp 1    one elected thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN,
//             K=16 per instruction) from shared-memory descriptors into a TMEM accumulator and
//             frees each stage with tcgen05.commit;
//   warps 2-5 first the TMA tile loads (A: 128 x 64, B: BN x 64, SWIZZLE_128B) into a ~192 KB
//             shared-memory ring (mbarrier full/empty handshake), lane 0 of each warp every
//             4th K block; weight tiles of the first stages are fetched before the wait on the
//             previous kernel.  Then the epilogue: tcgen05.ld from the TMEM lanes of their
//             quadrant (warp w reads rows
//             32*(w%4)..+31).  Split-K: for the residual every K slice red.adds its partial
//             tile into x (or, deterministic, runs on a cluster as below); for the other
//             epilogues (nonlinear in the sum) the slices run on a
//             cluster of CL CTAs, each parks its partial tile in shared memory and finishes
//             128/CL rows by summing the cluster's partials through distributed shared memory
//             in a fixed order.  The finished tile is staged in shared memory (swizzled rows) and
//             written out with every warp store covering whole lines (red.add for the
//             residual).
// A kernel that uses TMEM runs one CTA per SM, so the ring is sized for one CTA.  Every wait
// is bounded (about 2 s): on expiry the kernel records TI_DEVERR_GEMM_WAIT, skips the rest of
// its work, frees its TMEM and returns.
#include <algorithm>
#include <cstring>
#include <type_traits>
#include <mutex>
#include <unordered_map>

#include "capi_internal.h"
#include "common.cuh"
#include "tcgen05.cuh"

#ifndef TI_RESIDUAL_TMA_REDUCE
#define TI_RESIDUAL_TMA_REDUCE 1
#endif

namespace ti {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;                 // one 128-byte swizzle atom of bf16 per row
constexpr int kThreads = 192;

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
  // QKV + RoPE + KV append (TI_EPI_QKV_ROPE): one 64-wide N tile is one head
  const int32_t* pos;
  const int64_t* slot_mapping;
  const float* cos;
  const float* sin;
  void* k_cache;
  void* v_cache;
  int num_heads, num_kv_heads, block_size;
};

struct Best {
  float v;
  int i;
  __device__ __forceinline__ void take(float x, int idx) {   // larger value, then lower index
    if (x > v || (x == v && idx < i)) { v = x; i = idx; }
  }
};

// ---- output staging -----------------------------------------------------------------------
// The finished tile is written to shared memory as panels of R rows x PB bytes (PB = 128, or
// 64 for 64-byte output rows) with the 16-byte chunk index XORed by row % 8 (PB = 128) or
// (row / 2) % 4 (PB = 64), so that thread-per-row writes and chunk-per-thread reads are both
// free of bank conflicts; store_tile then writes it out line by line.
// Rows whose 16-byte chunk count is odd (80- and 144-byte rows of the 80- / 144-wide SwiGLU16
// tiles) are staged row-major without a swizzle (PB = the row's bytes): 8 consecutive rows then
// start on 8 different 16-byte bank groups, and chunk-per-thread reads are contiguous.
template <int PB>
__device__ __forceinline__ uint32_t stage_off(int r, int byte_col, int R) {
  if constexpr (PB != 64 && PB != 128) return (uint32_t)(r * PB + byte_col);
  const int panel = byte_col / PB;
  const int chunk = (byte_col % PB) >> 4;
  const int sw = PB == 128 ? (r & 7) : ((r >> 1) & 3);
  return (uint32_t)(panel * R * PB + r * PB + ((chunk ^ sw) << 4) + (byte_col & 15));
}
__device__ __forceinline__ void st_shared_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z,
                                             uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void st_shared_v2(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a)
               : "memory");
  return v;
}
// NV values for staged row r, tile columns col..col+NV-1, converted to OT (panels of PB bytes).
template <typename OT, int NV, int PB>
__device__ __forceinline__ void stage_vals(uint32_t base, int R, int r, int col, const float* v) {
  static_assert(NV % 4 == 0, "chunks of 4");
  if constexpr (sizeof(OT) == 4) {
#pragma unroll
    for (int g = 0; g < NV; g += 4)
      st_shared_v4(base + stage_off<PB>(r, (col + g) * 4, R), __float_as_uint(v[g]),
                   __float_as_uint(v[g + 1]), __float_as_uint(v[g + 2]), __float_as_uint(v[g + 3]));
  } else if constexpr (NV % 8 == 0) {
#pragma unroll
    for (int g = 0; g < NV; g += 8)
      st_shared_v4(base + stage_off<PB>(r, (col + g) * 2, R), Elem<OT>::pack2(v[g], v[g + 1]),
                   Elem<OT>::pack2(v[g + 2], v[g + 3]), Elem<OT>::pack2(v[g + 4], v[g + 5]),
                   Elem<OT>::pack2(v[g + 6], v[g + 7]));
  } else {
    st_shared_v2(base + stage_off<PB>(r, col * 2, R), Elem<OT>::pack2(v[0], v[1]),
                 Elem<OT>::pack2(v[2], v[3]));
  }
}
__device__ __forceinline__ void epilogue_bar() {   // the 4 epilogue warps
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Staged tile: columns and element size per epilogue kind.
template <typename T, int BN, int KIND>
struct Out {
  using OT = typename std::conditional<KIND == TI_EPI_RESIDUAL, float, T>::type;
  static constexpr int kCols = KIND == TI_EPI_SWIGLU || KIND == TI_EPI_SWIGLU16 ? BN / 2 : BN;
  static constexpr int kBytes = kCols * (int)sizeof(OT);   // per staged row
  static constexpr int kPanelBytes = (kBytes / 16) % 2 ? kBytes : kBytes < 128 ? 64 : 128;
  static_assert(kBytes % kPanelBytes == 0, "whole panels");
};

// Epilogue operands that do not depend on the accumulator (bias, RoPE table rows, pool slot),
// loaded by the epilogue threads while the MMAs still run (split-K path: chunks of NV <= 32).
template <typename T, int BN, int KIND, int NV>
struct Pre {
  static constexpr bool kBias = KIND == TI_EPI_STORE || KIND == TI_EPI_QKV_ROPE;
  static constexpr bool kRope = KIND == TI_EPI_QKV_ROPE;
  float a[kBias ? NV : 1], b[kBias ? NV : 1];   // bias for the lo / hi chunk
  float cs[kRope ? NV : 1], sn[kRope ? NV : 1];
  bool has_bias;

  __device__ __forceinline__ void load(const EpiArgs& e, int row, int n0, int c) {
    constexpr int H2 = BN / 2;
    if constexpr (kBias) {
      const T* bp = reinterpret_cast<const T*>(e.bias);
      has_bias = bp != nullptr;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        a[i] = bp ? Elem<T>::to_f(bp[n0 + c + i]) : 0.f;
        b[i] = bp ? Elem<T>::to_f(bp[n0 + H2 + c + i]) : 0.f;
      }
    }
    if constexpr (kRope) {
      if (n0 / 64 < e.num_heads + e.num_kv_heads) {
        const int64_t pr = (int64_t)e.pos[row] * 32 + c;
#pragma unroll
        for (int i = 0; i < NV; i += 4) {
          const float4 cv = *reinterpret_cast<const float4*>(e.cos + pr + i);
          const float4 sv = *reinterpret_cast<const float4*>(e.sin + pr + i);
          cs[i] = cv.x; cs[i + 1] = cv.y; cs[i + 2] = cv.z; cs[i + 3] = cv.w;
          sn[i] = sv.x; sn[i + 1] = sv.y; sn[i + 2] = sv.z; sn[i + 3] = sv.w;
        }
      }
    }
  }
};

// silu(g) * u with the reference's formula g / (1 + e^-g) * u and its __expf
// (src/fused_swiglu.cu:44-48); the division is the fast x * rcp form (a few fp32 ulp, far
// below the bf16 rounding of the result) -- the IEEE divide costs about 4x the whole epilogue.
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// The epilogue of one output row on two column chunks of the 128 x BN tile: `lo` holds tile
// columns [c, c + NV), `hi` the columns [BN/2 + c, BN/2 + c + NV) -- the pairs that SwiGLU
// (gate, up) and rotate-half RoPE (x1, x2) combine.  Values are the finished fp32 sums; the
// results go to staged row `lr` (R staged rows).  `row` is the global row (< M when live).
template <typename T, int BN, int KIND, int NV, bool PRE>
__device__ __forceinline__ void epilogue_chunk(const EpiArgs& e, int row, bool live, int lr, int n0,
                                               int c, float* lo, float* hi, Best& best,
                                               const Pre<T, BN, KIND, PRE ? NV : 4>& pre,
                                               uint32_t stage, int R) {
  constexpr int H2 = BN / 2;
  constexpr int PB = Out<T, BN, KIND>::kPanelBytes;
  if constexpr (KIND == TI_EPI_STORE || KIND == TI_EPI_QKV_ROPE) {
    if constexpr (PRE) {
      if (pre.has_bias) {
#pragma unroll
        for (int i = 0; i < NV; ++i) { lo[i] += pre.a[i]; hi[i] += pre.b[i]; }
      }
    } else {
      const T* b = reinterpret_cast<const T*>(e.bias);
      if (b) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          lo[i] += Elem<T>::to_f(b[n0 + c + i]);
          hi[i] += Elem<T>::to_f(b[n0 + H2 + c + i]);
        }
      }
    }
  }
  if constexpr (KIND == TI_EPI_QKV_ROPE) {
    // BN == head_dim == 64: lo = x1 (dims c..), hi = x2 (dims 32 + c..), the rotate-half pairs.
    // RoPE runs on the fp32 accumulators (+bias) and each value is rounded once, q into `out`,
    // k and v into the pool (src/fused_rope.cu:37-50, engine/cache_manager.py:95-99).
    static_assert(BN == 64, "one head per tile");
    if (n0 / 64 < e.num_heads + e.num_kv_heads) {
      float cc[NV], ss[NV];
      if constexpr (PRE) {
#pragma unroll
        for (int i = 0; i < NV; ++i) { cc[i] = pre.cs[i]; ss[i] = pre.sn[i]; }
      } else {
        const int64_t pr = (int64_t)(live ? e.pos[row] : 0) * 32 + c;
#pragma unroll
        for (int i = 0; i < NV; i += 4) {
          const float4 cv = *reinterpret_cast<const float4*>(e.cos + pr + i);
          const float4 sv = *reinterpret_cast<const float4*>(e.sin + pr + i);
          cc[i] = cv.x; cc[i + 1] = cv.y; cc[i + 2] = cv.z; cc[i + 3] = cv.w;
          ss[i] = sv.x; ss[i + 1] = sv.y; ss[i + 2] = sv.z; ss[i + 3] = sv.w;
        }
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const float x1 = lo[i], x2 = hi[i];
        lo[i] = x1 * cc[i] - x2 * ss[i];
        hi[i] = x1 * ss[i] + x2 * cc[i];
      }
    }
  }
  if constexpr (KIND == TI_EPI_SWIGLU) {
    // tile columns [0, BN/2) are gate rows g0..g0+BN/2-1, [BN/2, BN) the matching up rows
#pragma unroll
    for (int i = 0; i < NV; ++i) lo[i] = silu_mul(lo[i], hi[i]);
    stage_vals<T, NV, PB>(stage, R, lr, c, lo);
  } else if constexpr (KIND == TI_EPI_ARGMAX) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      best.take(lo[i], n0 + c + i);
      best.take(hi[i], n0 + H2 + c + i);
    }
    if (e.out) {
      stage_vals<T, NV, PB>(stage, R, lr, c, lo);
      stage_vals<T, NV, PB>(stage, R, lr, H2 + c, hi);
    }
  } else {
    using OT = typename Out<T, BN, KIND>::OT;
    stage_vals<OT, NV, PB>(stage, R, lr, c, lo);
    stage_vals<OT, NV, PB>(stage, R, lr, H2 + c, hi);
  }
}

// SwiGLU16 epilogue of one accumulator row (TMEM lane of this thread): every 32 accumulator
// columns are two groups of (8 gate, 8 matching up) and give 16 outputs; a tile width of 16
// mod 32 ends on one group (the 16 columns read past it are allocated TMEM that the MMA did not
// write, and are dropped).
template <typename T, int BN>
__device__ __forceinline__ void swiglu16_rows(uint32_t trow, int lr, uint32_t stage) {
  constexpr int PB = Out<T, BN, TI_EPI_SWIGLU16>::kPanelBytes;
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    float v[32], o[16];
    tmem_ld32(trow + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i] = silu_mul(v[i], v[8 + i]);
      o[8 + i] = silu_mul(v[16 + i], v[24 + i]);
    }
    if (c + 32 <= BN) stage_vals<T, 16, PB>(stage, BM, lr, c / 2, o);
    else stage_vals<T, 8, PB>(stage, BM, lr, c / 2, o);
  }
}

// Pool slots of the rows one epilogue thread stores in a k / v tile of the QKV epilogue (rows
// t / 8 + 16 j of the R staged rows, t = the thread's index among the 128), loaded before the
// accumulator wait so that the stores do not wait on a dependent load; -1: no store.
template <int KIND, int R>
struct KvSlots {
  static constexpr int kN = KIND == TI_EPI_QKV_ROPE ? R / 16 : 1;
  int64_t s[kN];
  __device__ __forceinline__ void load(const EpiArgs& e, int n0, int y0) {
    if constexpr (KIND == TI_EPI_QKV_ROPE) {
      const int t = (int)threadIdx.x - 64;
      const bool kv = n0 / 64 >= e.num_heads;
#pragma unroll
      for (int j = 0; j < kN; ++j) {
        const int row = y0 + (t >> 3) + 16 * j;
        s[j] = kv && row < e.M ? e.slot_mapping[row] : -1;
      }
    }
  }
};

// Write the staged tile (R rows starting at global row y0) to global memory: the 128 epilogue
// threads walk it in 16-byte chunks, consecutive threads on consecutive chunks of a row, so
// each warp store covers whole lines; the residual adds with red.global.add (one add per
// element: deterministic).  The k / v heads of the QKV epilogue go to their pool slots, one
// 128-byte row per token.  Fire-and-forget: the CTA does not wait for the writes.
template <typename T, int BN, int KIND, int R>
__device__ __forceinline__ void store_tile(const EpiArgs& e, uint32_t stage, int n0, int y0,
                                           bool ok, const KvSlots<KIND, R>& kv,
                                           const CUtensorMap* xmap) {
  using O = Out<T, BN, KIND>;
  constexpr int PB = O::kPanelBytes;
  constexpr int CPR = O::kBytes / 16;   // 16-byte chunks per staged row
#if TI_RESIDUAL_TMA_REDUCE
  if constexpr (KIND == TI_EPI_RESIDUAL) {
    // The staged fp32 tile is R rows x 128-byte panels in the 128-byte swizzle: one bulk tensor
    // reduce-add per panel (rows past M clipped by the tensor map) instead of a red.add per
    // 16 bytes.  The staging writes are made visible to the async proxy first.
    static_assert(PB == 128, "fp32 residual tiles stage 128-byte panels");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    epilogue_bar();
    if (!ok || threadIdx.x != 64) return;
#pragma unroll
    for (int pnl = 0; pnl < O::kBytes / 128; ++pnl)
      asm volatile(
          "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group"
          " [%0, {%1, %2}], [%3];" ::"l"(reinterpret_cast<uint64_t>(xmap)),
          "r"(n0 + pnl * 32), "r"(y0), "r"(stage + (uint32_t)(pnl * R * 128))
          : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // shared memory read
    return;
  }
#endif
  epilogue_bar();                       // the whole tile is staged
  if (!ok) return;
  const int t = (int)threadIdx.x - 64;
  if constexpr (KIND == TI_EPI_QKV_ROPE) {
    if (n0 / 64 >= e.num_heads) {
      const int head = n0 / 64;
      const bool is_k = head < e.num_heads + e.num_kv_heads;
      const int kh = is_k ? head - e.num_heads : head - e.num_heads - e.num_kv_heads;
      T* pool = reinterpret_cast<T*>(is_k ? e.k_cache : e.v_cache);
      static_assert(R % 16 == 0, "whole rounds of 16 rows");
#pragma unroll
      for (int j = 0; j < R / 16; ++j) {   // 8 threads per 128-byte row
        const int r = (t >> 3) + 16 * j, ch = t & 7;
        const int64_t slot = kv.s[j];
        if (slot < 0) continue;
        const uint4 v = ld_shared_v4(stage + stage_off<PB>(r, ch * 16, R));
        T* dst = pool + (((slot / e.block_size) * e.num_kv_heads + kh) * e.block_size +
                         slot % e.block_size) * 64 + ch * 8;
        *reinterpret_cast<uint4*>(dst) = v;
      }
      return;
    }
  }
  if constexpr (KIND == TI_EPI_ARGMAX) {
    if (!e.out) return;
  }
  using OT = typename O::OT;
  const int x0 = KIND == TI_EPI_SWIGLU || KIND == TI_EPI_SWIGLU16 ? n0 / 2 : n0;
  uint8_t* base = reinterpret_cast<uint8_t*>(e.out) + (int64_t)x0 * (int64_t)sizeof(OT);
  const int64_t pitch = e.ldo * (int64_t)sizeof(OT);
  // the last SwiGLU16 tile may reach past N: its chunks beyond N / 2 outputs are not stored
  const int live_chunks = KIND == TI_EPI_SWIGLU16 ? min(CPR, (e.N / 2 - x0) / 8) : CPR;
  for (int idx = t; idx < R * CPR; idx += 128) {
    const int r = idx / CPR, ch = idx % CPR;
    const int row = y0 + r;
    if (row >= e.M || ch >= live_chunks) continue;
    const uint4 v = ld_shared_v4(stage + stage_off<PB>(r, ch * 16, R));
    uint8_t* dst = base + row * pitch + ch * 16;
    if constexpr (KIND == TI_EPI_RESIDUAL) {
      asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst),
                   "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
                   "f"(__uint_as_float(v.w))
                   : "memory");
    } else {
      *reinterpret_cast<uint4*>(dst) = v;
    }
  }
}

constexpr int kMaxSmem = 227 * 1024;

// AR: activation rows loaded per stage.  Batches of at most 32 / 64 rows load 32 / 64 (the MMA
// still reads 128 rows: the rows past AR come from the rest of the stage and are garbage that
// only reaches accumulator rows >= M, which are never stored), so that a stage is small enough
// for the ring to hold every K block of the tile at once.
// PAIR: the tile is computed by a CTA pair (a cluster of two consecutive CTAs along grid x)
// with M = 256 MMAs (cta_group::2): each CTA loads its own 128 rows of A and half of the tile's
// BN rows of B, so each SM streams a quarter fewer bytes per output than a 1-SM tile of the same
// width.
template <int BN, int STAGES, int CL, int AR = BM, bool PAIR = false>
struct Cfg {
  static constexpr int kABytes = AR * BK * 2;
  static constexpr int kBRows = PAIR ? BN / 2 : BN;   // B rows this CTA loads per stage
  static constexpr int kBBytes = kBRows * BK * 2;
  static constexpr int kStage = kABytes + kBBytes;
  // the last stage's 128-row A read reaches this far past the ring
  static constexpr int kAOver = (BM - AR) * BK * 2 > kBBytes ? (BM - AR) * BK * 2 - kBBytes : 0;
  static constexpr int kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  // mbarriers (full, empty per stage; accumulator) and the TMEM address slot (sized for STAGES,
  // an upper bound of the ring depth)
  static constexpr int kBarBytes = (2 * STAGES + 1) * 8 + 8;
  // split-K across a cluster of CL CTAs: CTA r finishes rows r * BM / CL .. of the cluster's
  // tile.  Every CTA pushes each row of its fp32 partial tile into the receive buffer of the
  // CTA that finishes that row ([source rank][row][column], rows padded by 16 bytes against
  // bank conflicts), so after one cluster barrier the owner sums the CL partials from its own
  // shared memory.  The receive buffer lies beside the stage ring, because a peer may push
  // while this CTA's MMAs still read the ring; the ring gives up stages to make room.
  static constexpr int kRedStride = BN + 4;
  static constexpr int kRecvBytes = CL > 1 ? BM * kRedStride * 4 : 0;
  static constexpr int kRecvOff = CL > 1 ? (kBarBytes + 127) / 128 * 128 : 0;   // after the ring
  static constexpr int kStages =
      CL > 1 ? (STAGES < (kMaxSmem - 1024 - kRecvOff - kRecvBytes) / kStage
                    ? STAGES
                    : (kMaxSmem - 1024 - kRecvOff - kRecvBytes) / kStage)
             : STAGES;
  static constexpr int kRing = kStages * kStage;
  static constexpr int kStageOff = 0;              // output staging: the drained ring
  static constexpr int kRows = BM / CL;            // rows each CTA of the cluster finishes
  static constexpr int kW = BN / 2 / CL;           // chunk width per thread
  // The ring starts on a 1024-byte boundary (128-byte swizzle atoms); the barriers go into
  // the alignment slack below it when that has room, else right after the ring (where the
  // receive buffer leaves them kRecvOff bytes).
  static constexpr int kSmem = kRing + 1024 + (CL > 1 ? kRecvOff + kRecvBytes : 0) + kAOver;
  static_assert(2 * kBarBytes <= 1024, "barriers fit beside the ring in the 1 KB slack");
  static_assert(CL == 1 || kW % 4 == 0, "cluster chunks must be multiples of 4 columns");
  static_assert(kStages >= 2, "a ring of at least two stages");
  static_assert(AR == BM || (CL == 1 && AR % 8 == 0 && kABytes % 1024 == 0),
                "short activation boxes: unsplit tiles, 1024-byte aligned stages");
  static_assert(!PAIR || (CL == 1 && AR == BM && kBRows % 8 == 0 && kBBytes % 1024 == 0),
                "CTA pairs: no split-K cluster, full activation boxes, whole 8-row B groups");
  static_assert(kSmem <= kMaxSmem, "shared memory");
};

// Whether the staged output tile fits the drained stage ring.
template <typename T, int BN, int STAGES, int KIND, int CL, int AR = BM, bool PAIR = false>
constexpr bool ring_fits() {
  using C = Cfg<BN, STAGES, CL, AR, PAIR>;
  return C::kStageOff + C::kRows * Out<T, BN, KIND>::kBytes <= C::kRing;
}

// One 128 x BN output tile per cluster of CL CTAs (CL = split-K factor along grid z); PAIR: a
// 256 x BN tile per CTA pair, each CTA finishing its own 128 rows.
template <typename T, int BN, int STAGES, int KIND, int CL, int AR = BM, bool PAIR = false>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
            const __grid_constant__ CUtensorMap xmap, int K, int kb_per_split, EpiArgs e) {
  using C = Cfg<BN, STAGES, CL, AR, PAIR>;
  constexpr int S = C::kStages;   // ring depth (a cluster kernel's receive buffer takes stages)
  static_assert(ring_fits<T, BN, STAGES, KIND, CL, AR, PAIR>(), "staged tile fits the ring");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* bars = (smem - smem_raw >= C::kBarBytes) ? smem_raw : smem + C::kRing;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + S * 8;
  const uint32_t accum = empty0 + S * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + (2 * S + 1) * 8);
  const uint32_t recv = sbase + C::kRing + C::kRecvOff;   // cluster receive buffer (CL > 1)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // a CTA pair is two consecutive CTAs along grid x (the 128-row M tiles); else x runs over N
  const int tile_n = PAIR ? blockIdx.y : blockIdx.x;
  const int n0 = tile_n * BN, m0 = (PAIR ? blockIdx.x : blockIdx.y) * BM;
  const int nkb = K / BK;
  const int kb0 = blockIdx.z * kb_per_split;
  const int kb1 = min(nkb, kb0 + kb_per_split);
  const int nk = max(0, kb1 - kb0);

  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < S; ++s) {
        mbar_init(full0 + 8 * s, 1);
        mbar_init(empty0 + 8 * s, 1);
      }
      mbar_init(accum, 1);
      fence_mbar_init();
      prefetch_tensormap(&amap);
      prefetch_tensormap(&bmap);
    }
    __syncwarp();
    if constexpr (PAIR) tmem_alloc_pair(smem_u32(tmem_slot), C::kTmemCols);
    else tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // All on-chip resources are held: the next kernel may be scheduled.
  pdl_launch_dependents();
  // CTA pair: both CTAs' barriers and TMEM exist before the odd CTA's loads complete on the even
  // CTA's barriers and the even CTA's MMAs and commits reach the odd one.
  const uint32_t prank = PAIR ? cluster_rank() : 0u;
  if constexpr (PAIR) cluster_sync();
  // Cluster barrier phase 1 (arrive now, wait before the first push): every CTA of the
  // cluster has started, so its shared memory may be written.
  if constexpr (CL > 1) cluster_arrive_relaxed();

  // split-K: the row / columns this thread finishes after the cluster reduction
  const int red_t = (int)threadIdx.x - 64;
  const uint32_t rank = CL > 1 ? cluster_rank() : 0u;
  const int red_lr = (red_t >= 0 ? red_t : 0) / CL;   // row within this CTA's kRows
  const int red_c = ((red_t >= 0 ? red_t : 0) % CL) * C::kW;
  const int red_row = m0 + (int)rank * C::kRows + red_lr;
  const bool red_live = red_t >= 0 && red_row < e.M;
  Pre<T, BN, KIND, (CL > 1 ? C::kW : 4)> pre;
  KvSlots<KIND, C::kRows> kv;
  bool ok = true;

  if (warp == 1) {
    // the MMA issuer: lane 0 (of the even CTA of a pair, for both)
    if (lane == 0 && prank == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idesc = PAIR ? idesc_f16(2 * BM, BN, kBf16, false, false)
                                      : instr_desc(BN, kBf16);
      // a pair's commits arrive on the barrier at the same offset in both CTAs
      const uint32_t odd = PAIR ? map_peer(full0, 1u) - full0 : 0u;
      for (int it = 0; it < nk; ++it) {
        const int s = it % S;
        if (!mbar_wait(full0 + 8 * s, (it / S) & 1, TI_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t sa = sbase + s * C::kStage;
        const uint64_t da = smem_desc(sa), db = smem_desc(sa + C::kABytes);
        if constexpr (PAIR) {
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_pair(tmem, da + 2 * k, db + 2 * k, idesc, (it > 0 || k > 0) ? 1u : 0u);
          tc_commit_pair(empty0 + 8 * s);
          tc_commit_pair(empty0 + 8 * s + odd);
        } else {
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)   // +32 bytes along K inside the swizzle atom
            tc_mma(tmem, da + 2 * k, db + 2 * k, idesc, (it > 0 || k > 0) ? 1u : 0u);
          tc_commit(empty0 + 8 * s);
        }
      }
      if constexpr (PAIR) {
        tc_commit_pair(accum);
        tc_commit_pair(accum + odd);
      } else {
        tc_commit(accum);
      }
    }
    __syncwarp();
  } else if (warp >= 2) {
    // Producers: lane 0 of kProd epilogue warps issues the TMA loads of every kProd-th K block
    // (one issuing thread's loads complete one after another, the streams overlap).  The empty
    // barrier waits are parity waits: a producer about to refill a stage for its u-th use must
    // know that use u - 2 was consumed, which holds when its own previous K block (kProd
    // earlier) waited for a consumption at least S - kProd blocks later than that use,
    // hence kProd <= S.
    constexpr int kProd = S < 4 ? S : 4;
    if (lane == 0 && warp - 2 < kProd) {
      const int p = warp - 2;
      const uint64_t pol_a = l2_policy_evict_last();    // activations: re-read by many CTAs
      const uint64_t pol_b = l2_policy_evict_first();   // weights: streamed once
      // A pair's loads all complete on the even CTA's full barriers, which expect both CTAs'
      // bytes; each CTA loads its own B rows (the second half of the tile for the odd CTA).
      const uint32_t fullx = PAIR ? map_peer(full0, 0u) : full0;
      const int nb = n0 + (int)prank * C::kBRows;
      auto expect = [&](int s) {
        if (prank == 0) mbar_arrive_expect_tx(full0 + 8 * s, PAIR ? 2 * C::kStage : C::kStage);
      };
      auto load = [&](uint32_t dst, const CUtensorMap* map, int s, int x, int y, uint64_t pol) {
        if constexpr (PAIR) tma_load_2d_pair(dst, map, fullx + 8 * s, x, y, pol);
        else tma_load_2d_hint(dst, map, full0 + 8 * s, x, y, pol);
      };
      // Weights do not depend on earlier kernels: fetch the first stages' B tiles before
      // waiting for the producer of the activations.
      const int pre_n = min(nk, S);
      for (int it = p; it < pre_n; it += kProd) {
        expect(it);
        load(sbase + it * C::kStage + C::kABytes, &bmap, it, (kb0 + it) * BK, nb, pol_b);
      }
      pdl_wait();
      for (int it = p; it < pre_n; it += kProd)
        load(sbase + it * C::kStage, &amap, it, (kb0 + it) * BK, m0, pol_a);
      for (int it = p; it < nk; it += kProd) {
        if (it < pre_n) continue;
        const int s = it % S;
        if (!mbar_wait(empty0 + 8 * s, ((it / S) & 1) ^ 1, TI_DEVERR_GEMM_WAIT)) break;
        expect(s);
        const uint32_t sa = sbase + s * C::kStage;
        const int kx = (kb0 + it) * BK;
        load(sa, &amap, s, kx, m0, pol_a);
        load(sa + C::kABytes, &bmap, s, kx, nb, pol_b);
      }
    }
    __syncwarp();
    pdl_wait();   // the epilogue reads and writes memory of earlier kernels
    const int quad = warp & 3;
    if constexpr (CL > 1) {
      if (red_live) pre.load(e, red_row, n0, red_c);
    }
    kv.load(e, n0, m0 + (int)rank * C::kRows);
    // tcgen05.ld is warp-collective: the warp goes on only when all its lanes saw the phase
    ok = __all_sync(0xffffffffu, mbar_wait(accum, 0, TI_DEVERR_GEMM_WAIT));
    tc_fence_after();
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    if constexpr (CL == 1) {
      const int lr = quad * 32 + lane;
      const int row = m0 + lr;
      const bool live = row < e.M;
      Best best{-INFINITY, 0x7fffffff};
      if constexpr (KIND == TI_EPI_SWIGLU16) {
        if (ok && nk > 0) swiglu16_rows<T, BN>(trow, lr, sbase);
      } else if (ok && nk > 0) {
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          float lo[32], hi[32];
          tmem_ld32(trow + c, lo);
          tmem_ld32(trow + BN / 2 + c, hi);
          epilogue_chunk<T, BN, KIND, 32, false>(e, row, live, lr, n0, c, lo, hi, best,
                                                 Pre<T, BN, KIND, 4>{}, sbase, BM);
        }
        if constexpr (KIND == TI_EPI_ARGMAX) {
          if (live) {
            e.aux_val[(int64_t)row * e.ntiles + tile_n] = best.v;
            e.aux_idx[(int64_t)row * e.ntiles + tile_n] = best.i;
          }
        }
      }
      store_tile<T, BN, KIND, BM>(e, sbase, n0, m0, ok && nk > 0, kv, &xmap);
    } else {
      // this CTA's fp32 partial tile (zeros for an empty split), row by row, into the receive
      // buffer of the CTA that finishes the row: slot [this rank][row % kRows]
      cluster_wait_acquire();   // phase 1: every CTA of the cluster has started
      const int lr = quad * 32 + lane;
      const uint32_t dst = map_peer(
          recv + (uint32_t)(((int)rank * C::kRows + lr % C::kRows) * C::kRedStride) * 4u,
          (uint32_t)(lr / C::kRows));
      // a warp whose 32 rows all lie past M pushes nothing (their sums are never stored)
      const bool rows_live = m0 + quad * 32 < e.M;
#pragma unroll 1
      for (int c = 0; c < (rows_live ? BN : 0); c += 32) {
        float v[32];
        if (ok && nk > 0) {
          tmem_ld32(trow + c, v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          st_peer_f4(dst + 4u * (uint32_t)(c + i), v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
    }
  }
  if constexpr (CL > 1) {
    if (warp < 2) cluster_wait_acquire();   // phase 1 (the epilogue warps took it above)
    // phase 2: every partial of the rows this CTA finishes is in its receive buffer
    cluster_arrive_release();
    cluster_wait_acquire();
    if (warp >= 2) {
      float lo[C::kW], hi[C::kW];
#pragma unroll
      for (int i = 0; i < C::kW; ++i) lo[i] = hi[i] = 0.f;
      const uint32_t mine = recv + (uint32_t)(red_lr * C::kRedStride + red_c) * 4u;
#pragma unroll
      for (int src = 0; src < CL; ++src) {   // fixed order: the sum is deterministic
        const uint32_t a = mine + (uint32_t)(src * C::kRows * C::kRedStride) * 4u;
#pragma unroll
        for (int i = 0; i < C::kW; i += 4) {
          const uint4 x = ld_shared_v4(a + 4u * i);
          const uint4 y = ld_shared_v4(a + 4u * (BN / 2 + i));
          lo[i] += __uint_as_float(x.x); lo[i + 1] += __uint_as_float(x.y);
          lo[i + 2] += __uint_as_float(x.z); lo[i + 3] += __uint_as_float(x.w);
          hi[i] += __uint_as_float(y.x); hi[i + 1] += __uint_as_float(y.y);
          hi[i + 2] += __uint_as_float(y.z); hi[i + 3] += __uint_as_float(y.w);
        }
      }
      Best best{-INFINITY, 0x7fffffff};
      const uint32_t stage = sbase + C::kStageOff;
      epilogue_chunk<T, BN, KIND, C::kW, true>(e, red_row, red_live, red_lr, n0, red_c, lo, hi,
                                               best, pre, stage, C::kRows);
      if constexpr (KIND == TI_EPI_ARGMAX) {
#pragma unroll
        for (int o = CL / 2; o > 0; o >>= 1) {   // the CL threads of a row are adjacent lanes
          const float v = __shfl_xor_sync(0xffffffffu, best.v, o);
          const int i = __shfl_xor_sync(0xffffffffu, best.i, o);
          best.take(v, i);
        }
        if (red_live && red_t % CL == 0) {
          e.aux_val[(int64_t)red_row * e.ntiles + tile_n] = best.v;
          e.aux_idx[(int64_t)red_row * e.ntiles + tile_n] = best.i;
        }
      }
      store_tile<T, BN, KIND, C::kRows>(e, stage, n0, m0 + (int)rank * C::kRows, ok, kv, &xmap);
    }
    // no closing cluster barrier: after phase 2 no CTA touches another's shared memory
  }
  tc_fence_before();
  __syncthreads();
  // CTA pair: neither CTA frees its TMEM or exits while the other may still use its barriers
  if constexpr (PAIR) cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, C::kTmemCols);
    else tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---- persistent greedy lm_head: argmax of D = A . B^T per 128-column tile, M <= 256 -----------
// One CTA per SM loops over the N tiles.  Both 128-row halves of A (up to 256 tokens) share each
// B stage (two MMAs per K step), and the accumulators alternate between two 256-column TMEM
// buffers, so the epilogue of one tile (per row: max and first argmax of its 128 columns)
// overlaps the MMAs of the next while the TMA ring keeps streaming across tiles.
//   warp 0    TMA: A 256 x 64 + B 128 x 64 per K block (48 KB stages);
//   warp 1    MMA: 2 x tcgen05.mma M=128 N=128 per K=16 step, commits stages and buffers;
//   warps 2-5 epilogue: tcgen05.ld both halves, write (max, first argmax) per row and tile.
namespace lmh {
constexpr int kBN = 128;
constexpr int kStages = 4;
constexpr int kABytes = 256 * BK * 2;                 // 32 KB
constexpr int kBBytes = kBN * BK * 2;                 // 16 KB
constexpr int kStage = kABytes + kBBytes;             // 48 KB
constexpr int kRing = kStages * kStage;               // 192 KB
constexpr int kBars = (2 * kStages + 4) * 8 + 8;
constexpr int kSmem = kRing + 1024;
constexpr int kTmemCols = 512;                        // 2 buffers x (2 halves x 128 columns)
static_assert(2 * kBars <= 1024, "barriers fit the slack");
}  // namespace lmh

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
lmhead_argmax_kernel(const __grid_constant__ CUtensorMap amap,
                     const __grid_constant__ CUtensorMap bmap, int M, int K, int ntiles,
                     float* __restrict__ aux_val, int32_t* __restrict__ aux_idx) {
  using namespace lmh;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* bars = (smem - smem_raw >= kBars) ? smem_raw : smem + kRing;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + kStages * 8;
  const uint32_t accf0 = empty0 + kStages * 8;          // accumulator buffer b ready
  const uint32_t acce0 = accf0 + 2 * 8;                 // accumulator buffer b drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + (2 * kStages + 4) * 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = K / BK;

  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < kStages; ++s) {
        mbar_init(full0 + 8 * s, 1);
        mbar_init(empty0 + 8 * s, 1);
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(accf0 + 8 * b, 1);
        mbar_init(acce0 + 8 * b, 4);                    // one arrival per epilogue warp
      }
      fence_mbar_init();
      prefetch_tensormap(&amap);
      prefetch_tensormap(&bmap);
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
      const uint64_t pol_a = l2_policy_evict_last();
      const uint64_t pol_b = l2_policy_evict_first();
      int g = 0;          // K blocks issued so far (all tiles)
      bool waited = false, ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kStages;
          if (g >= kStages &&
              !mbar_wait(empty0 + 8 * s, ((g / kStages) & 1) ^ 1, TI_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full0 + 8 * s, kStage);
          const uint32_t sa = sbase + s * kStage;
          tma_load_2d_hint(sa + kABytes, &bmap, full0 + 8 * s, kb * BK, tile * kBN, pol_b);
          if (!waited) { pdl_wait(); waited = true; }   // A is the previous kernel's output
          tma_load_2d_hint(sa, &amap, full0 + 8 * s, kb * BK, 0, pol_a);
        }
      }
      if (!waited) pdl_wait();
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(kBN, std::is_same<T, __nv_bfloat16>::value);
      int g = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++local) {
        const int b = local & 1, use = local >> 1;
        if (use > 0 && !mbar_wait(acce0 + 8 * b, (use & 1) ^ 1, TI_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(b * 256), d1 = d0 + 128;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kStages;
          if (!mbar_wait(full0 + 8 * s, (g / kStages) & 1, TI_DEVERR_GEMM_WAIT)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = sbase + s * kStage;
          const uint64_t da = smem_desc(sa), da1 = smem_desc(sa + 128 * 128), db = smem_desc(sa + kABytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
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
        const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * 256 + half * 128);
        Best best{-INFINITY, 0x7fffffff};
#pragma unroll 1
        for (int c = 0; c < kBN; c += 32) {
          float v[32];
          tmem_ld32(trow + c, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) best.take(v[i], tile * kBN + c + i);
        }
        const int row = half * 128 + quad * 32 + lane;
        if (row < M) {
          aux_val[(int64_t)row * ntiles + tile] = best.v;
          aux_idx[(int64_t)row * ntiles + tile] = best.i;
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

template <typename T>
static int launch_lmhead_argmax(const CUtensorMap& am, const CUtensorMap& bm, int M, int N, int K,
                                float* aux_val, int32_t* aux_idx, cudaStream_t s) {
  auto kern = lmhead_argmax_kernel<T>;
  static int set_dev = -1, sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lmh::kSmem);
    if (err != cudaSuccess) return set_cuda_error(err, "cudaFuncSetAttribute(lm_head gemm)");
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    set_dev = dev;
  }
  const int ntiles = N / lmh::kBN;
  return launch_kernel("lm_head gemm launch", kern, dim3(std::min(sms, ntiles)), dim3(kThreads),
                       lmh::kSmem, s, 1, am, bm, M, K, ntiles, aux_val, aux_idx);
}

// ---- host side ----------------------------------------------------------------------------
struct MapKey {
  const void* p;
  int64_t rows, cols, ld_bytes;
  int box_cols, box_rows, type;
  bool operator==(const MapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && ld_bytes == o.ld_bytes &&
           box_cols == o.box_cols && box_rows == o.box_rows && type == o.type;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.p);
    h ^= std::hash<int64_t>()(k.rows * 1315423911LL + k.cols * 2654435761LL + k.ld_bytes) +
         0x9e3779b9 + (h << 6);
    return h ^ (size_t)(k.box_rows * 131 + k.box_cols * 7 + k.type);
  }
};

// 2-D tile map over a row-major [rows, cols] matrix (row pitch ld_bytes), box box_cols x
// box_rows with 128-byte rows (SWIZZLE_128B).  Cached per argument set.
static int tile_map(CUtensorMap* m, const void* p, CUtensorMapDataType type, int64_t rows,
                    int64_t cols, int64_t ld_bytes, int box_cols, int box_rows) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{p, rows, cols, ld_bytes, box_cols, box_rows, (int)type};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) { *m = it->second; return TI_OK; }
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  int rc = encode_tensor_map_2d(m, type, const_cast<void*>(p), dims, strides, box, es,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, *m);
  return TI_OK;
}

static CUtensorMapDataType tma_type(int dtype) {
  return dtype == TI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// K-major operand [rows, K] (leading dimension ld elements): 64 x box_rows boxes.
static int operand_map(CUtensorMap* m, const void* p, int64_t rows, int64_t cols, int64_t ld,
                       int box_rows, int dtype) {
  return tile_map(m, p, tma_type(dtype), rows, cols, ld * 2, BK, box_rows);
}

template <typename T, int BN, int STAGES, int KIND, int CL, int AR = BM, bool PAIR = false>
static int launch_t(const CUtensorMap& am, const CUtensorMap& bm, int M, int N, int K,
                    const EpiArgs& e, cudaStream_t s, int zsplits = 1) {
  if constexpr (!ring_fits<T, BN, STAGES, KIND, CL, AR, PAIR>()) {
    return set_error(TI_ERR_UNSUPPORTED, "gemm: this tile width and epilogue do not fit the stage ring");
  } else {
    using C = Cfg<BN, STAGES, CL, AR, PAIR>;
    auto kern = gemm_kernel<T, BN, STAGES, KIND, CL, AR, PAIR>;
    if (AR < BM && M > AR)
      return set_error(TI_ERR_INVALID_ARGUMENT, "gemm: short activation box for a taller batch");
    static int set_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (set_dev != dev) {
      cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
      if (err != cudaSuccess) return set_cuda_error(err, "cudaFuncSetAttribute(gemm)");
      set_dev = dev;
    }
    const int nkb = K / BK;
    const int zs = CL > 1 ? CL : zsplits;
    const int per = (nkb + zs - 1) / zs;   // a split may be empty (it contributes zeros)
    // a pair covers 256 rows: an even number of 128-row tiles, along x (clusters of 2 x 1 x 1)
    const int mt = PAIR ? (M + 2 * BM - 1) / (2 * BM) * 2 : (M + BM - 1) / BM;
    const int nt = (N + BN - 1) / BN, zt = CL > 1 ? CL : (nkb + per - 1) / per;
    const dim3 grid = PAIR ? dim3(mt, nt, zt) : dim3(nt, mt, zt);
    // residual: tensor map over x (fp32) for the bulk reduce-add of staged tiles
    CUtensorMap xm = am;
    if constexpr (KIND == TI_EPI_RESIDUAL && TI_RESIDUAL_TMA_REDUCE) {
      const int rc = tile_map(&xm, e.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, M, N, e.ldo * 4, 32,
                              C::kRows);
      if (rc) return rc;
    }
    return launch_kernel_cl("gemm launch", kern, grid, dim3(kThreads), C::kSmem, s,
                            dim3(PAIR ? 2 : 1, 1, CL > 1 ? CL : 1), am, bm, xm, K, per, e);
  }
}

// Which batches run on CTA pairs (2-SM MMAs): TI_GEMM_PAIR=1 every batch of more than 128 rows,
// =0 none, unset only those above kDeepRingMaxM rows (prefill).  At 256 decode rows each pair
// launch measured ~1 us slower than the 1-SM tiles (gate/up 9.2 -> 10.1, down 7.1 -> 8.0, o_proj
// 3.7 -> 4.8 us): those GEMMs wait on load round trips, not on the bytes each SM streams.
constexpr int kDeepRingMaxM = 256;
static int pair_mode() {
  static const int mode = [] {
    const char* v = getenv("TI_GEMM_PAIR");
    return v && v[0] == '0' ? 0 : v && v[0] == '1' ? 1 : 2;
  }();
  return mode;
}
inline bool pair_rows(int M) {
  const int mode = pair_mode();
  return mode == 1 ? M > BM : mode == 2 ? M > kDeepRingMaxM : false;
}

// Clusters of one CTA pair of this kernel the GPU keeps resident at once; cached per device.
template <typename T, int BN, int STAGES, int KIND>
static int max_pairs() {
  if constexpr (!ring_fits<T, BN, STAGES, KIND, 1, BM, true>()) {
    return 0;
  } else {
    static int cached_dev = -1, value = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (cached_dev != dev) {
      using C = Cfg<BN, STAGES, 1, BM, true>;
      auto kern = gemm_kernel<T, BN, STAGES, KIND, 1, BM, true>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, 1, 1);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = C::kSmem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = 0;   // unknown: no pairs
      }
      value = n;
      cached_dev = dev;
    }
    return value;
  }
}

// How many clusters of CL CTAs of this kernel the GPU keeps resident at once (a cluster needs
// CL free SMs in one GPC, so this is below 148 / CL); cached per device.
template <typename T, int BN, int STAGES, int KIND, int CL>
static int max_clusters() {
  if constexpr (!ring_fits<T, BN, STAGES, KIND, CL>()) {
    return 0;
  } else {
    static int cached_dev = -1, value = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (cached_dev != dev) {
      using C = Cfg<BN, STAGES, CL>;
      auto kern = gemm_kernel<T, BN, STAGES, KIND, CL>;
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 1, CL);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = C::kSmem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 1;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = CL;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = 148 / CL / 2;   // conservative when the query is unavailable
      }
      value = n;
      cached_dev = dev;
    }
    return value;
  }
}

// Cluster size of a nonlinear-epilogue GEMM: the largest of 8 / 4 / 2 (at most `cl`) whose
// clusters for all output tiles are resident at once and that leaves at least two K blocks per
// split; else 1.
template <typename T, int BN, int STAGES, int KIND>
static int pick_cl(int cl, int M, int N, int K) {
  const int64_t tiles = (int64_t)(N / BN) * ((M + BM - 1) / BM);
  const int nkb = K / BK;
  if (cl >= 8 && nkb >= 16 && tiles <= max_clusters<T, BN, STAGES, KIND, 8>()) return 8;
  if (cl >= 4 && nkb >= 8 && tiles <= max_clusters<T, BN, STAGES, KIND, 4>()) return 4;
  if (cl >= 2 && nkb >= 4 && tiles <= max_clusters<T, BN, STAGES, KIND, 2>()) return 2;
  return 1;
}

// split-K factor -> cluster size: 1, 2, 4 or 8 (the largest power of two <= split, at most 8)
static int cluster_for(int split) {
  return split >= 8 ? 8 : split >= 4 ? 4 : split >= 2 ? 2 : 1;
}
constexpr int kMaxResidualSplit = 16;

// Launch with the largest cluster size <= `cl` whose clusters for all `tiles` output tiles are
// resident at once (a second wave would double the time) and that leaves at least two K blocks
// per split.
// DET (residual only): split K over a cluster and sum the slices in a fixed order instead of
// letting every slice red.add on its own, so that `x` is bit-reproducible.
// Ring depth of a pair tile: decode batches (one wave) 8 stages; above kDeepRingMaxM rows
// (many waves) rings of ~96 KB, two CTAs per SM as for the 1-SM tiles.
constexpr int kPairStagesDeep = 8;
template <int BN>
constexpr int pair_stages_shallow() { return BN <= 128 ? 4 : 3; }

// PSTAGES: the ring depth of the pair variant of this tile.
template <typename T, int BN, int STAGES, int KIND, bool DET = false, int PSTAGES = kPairStagesDeep>
static int dispatch_cl(int cl, const CUtensorMap& am, const CUtensorMap& bm, int M, int N, int K,
                       const EpiArgs& e, cudaStream_t s, const CUtensorMap* bm_pair = nullptr) {
  if constexpr (KIND == TI_EPI_ARGMAX) {   // argmax tiles are never split
    return launch_t<T, BN, STAGES, KIND, 1>(am, bm, M, N, K, e, s);
  } else if constexpr (KIND == TI_EPI_RESIDUAL && !DET) {
    // The residual is linear: every K slice adds its partial tile into x on its own (red.add),
    // no cluster needed.  At most `cl` slices, at least two K blocks each, one wave.
    const int64_t tiles = (int64_t)(N / BN) * ((M + BM - 1) / BM);
    int z = std::max(1, std::min(cl, K / BK / 2));
    while (z > 1 && tiles * z > 148) --z;
    // pairs: one wave of them at decode sizes; any number of waves above
    const int64_t pairs = tiles * z / 2, room = max_pairs<T, BN, PSTAGES, KIND>();
    if (bm_pair && pair_rows(M) && room > 0 && (M > kDeepRingMaxM || pairs <= room))
      return launch_t<T, BN, PSTAGES, KIND, 1, BM, true>(am, *bm_pair, M, N, K, e, s, z);
    return launch_t<T, BN, STAGES, KIND, 1>(am, bm, M, N, K, e, s, z);
  } else {
    switch (pick_cl<T, BN, STAGES, KIND>(cl, M, N, K)) {
      case 8: return launch_t<T, BN, STAGES, KIND, 8>(am, bm, M, N, K, e, s);
      case 4: return launch_t<T, BN, STAGES, KIND, 4>(am, bm, M, N, K, e, s);
      case 2: return launch_t<T, BN, STAGES, KIND, 2>(am, bm, M, N, K, e, s);
      default: return launch_t<T, BN, STAGES, KIND, 1>(am, bm, M, N, K, e, s);
    }
  }
}

#ifndef TI_GEMM_STAGES_64
#define TI_GEMM_STAGES_64 8
#endif
#ifndef TI_GEMM_STAGES_128
#define TI_GEMM_STAGES_128 6
#endif
#ifndef TI_GEMM_STAGES_256
#define TI_GEMM_STAGES_256 4
#endif
// Ring depth per tile width.  Up to kDeepRingMaxM rows (decode batches: one wave of tiles) about
// 192 KB of loads in flight for the one CTA on the SM; above (prefill: many waves) ~96 KB rings,
// so two CTAs share an SM and one's epilogue runs under the other's main loop (measured at 4096
// tokens: gate/up 780 -> 933 TFLOP/s; at 256 tokens the deep rings are 5 % faster per step).
template <typename T, int KIND, bool DET = false>
static int dispatch_bn(int bn, int cl, const CUtensorMap& am, const CUtensorMap& bm, int M, int N,
                       int K, const EpiArgs& e, cudaStream_t s,
                       const CUtensorMap* bm_pair = nullptr) {
  const bool deep = M <= kDeepRingMaxM;
  switch (bn) {
    case 64:
      return deep ? dispatch_cl<T, 64, TI_GEMM_STAGES_64, KIND, DET>(cl, am, bm, M, N, K, e, s, bm_pair)
                  : dispatch_cl<T, 64, 4, KIND, DET, pair_stages_shallow<64>()>(cl, am, bm, M, N,
                                                                              K, e, s, bm_pair);
    case 128:
      return deep ? dispatch_cl<T, 128, TI_GEMM_STAGES_128, KIND, DET>(cl, am, bm, M, N, K, e, s, bm_pair)
                  : dispatch_cl<T, 128, 3, KIND, DET, pair_stages_shallow<128>()>(cl, am, bm, M,
                                                                                N, K, e, s, bm_pair);
    case 256:   // never split
      return deep ? launch_t<T, 256, TI_GEMM_STAGES_256, KIND, 1>(am, bm, M, N, K, e, s)
                  : launch_t<T, 256, 2, KIND, 1>(am, bm, M, N, K, e, s);
    default: return set_error(TI_ERR_UNSUPPORTED, "gemm: block_n must be 64, 128 or 256");
  }
}

#ifndef TI_QKV_MAX_SPLIT
#define TI_QKV_MAX_SPLIT 8
#endif
#ifndef TI_GEMM_STAGES_QKV
#define TI_GEMM_STAGES_QKV TI_GEMM_STAGES_64
#endif
// QKV: as much split-K as keeps one wave.
template <typename T>
static int launch_qkv(const CUtensorMap& am, const CUtensorMap& bm, int M, int N, int K,
                      const EpiArgs& e, cudaStream_t s) {
  return M <= kDeepRingMaxM
             ? dispatch_cl<T, 64, TI_GEMM_STAGES_QKV, TI_EPI_QKV_ROPE>(TI_QKV_MAX_SPLIT, am, bm, M, N, K, e, s)
             : dispatch_cl<T, 64, 4, TI_EPI_QKV_ROPE>(8, am, bm, M, N, K, e, s);
}

// CTAs of the QKV GEMM's launch for M rows (the decode attention plan uses it: the SMs this
// grid holds are the ones on which the attention's CTAs start late).
template <typename T>
static int qkv_ctas_t(int M, int N, int K) {
  const int64_t tiles = (int64_t)(N / 64) * ((M + BM - 1) / BM);
  const int cl = M <= kDeepRingMaxM
                     ? pick_cl<T, 64, TI_GEMM_STAGES_QKV, TI_EPI_QKV_ROPE>(TI_QKV_MAX_SPLIT, M, N, K)
                     : pick_cl<T, 64, 4, TI_EPI_QKV_ROPE>(8, M, N, K);
  return (int)std::min<int64_t>(tiles * cl, 1 << 30);
}

#ifndef TI_GEMM_STAGES_80
#define TI_GEMM_STAGES_80 8
#endif
#ifndef TI_GEMM_STAGES_144
#define TI_GEMM_STAGES_144 6
#endif
// SwiGLU16 tile width: up to kDeepRingMaxM rows the narrowest of 80 / 144 whose tiles cover all
// rows in one wave of the GPU (at 256 tokens and N = 2 x 4864: 136 CTAs of 144 columns instead
// of 76 of 256, so more SMs stream the weights and each re-reads less of the activations);
// above, 256 (many waves).
static int swiglu16_bn(int M, int N) {
  static int cached_dev = -1, sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cached_dev != dev) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      sms = 148;
    cached_dev = dev;
  }
  if (M <= kDeepRingMaxM) {
    const int64_t mt = (M + BM - 1) / BM;
    if (mt * ((N + 79) / 80) <= sms) return 80;
    if (mt * ((N + 143) / 144) <= sms) return 144;
  }
  return 256;
}
// Rows of the activation box for an M-row SwiGLU16 GEMM: 32 / 64 when the batch fits and the
// whole hidden size (K <= 896, 14 K blocks) then fits the deeper ring, else BM.
static int swiglu16_box_rows(int M, int K, int bn) {
  if (bn != 80 || K > 896) return BM;
  return M <= 32 ? 32 : M <= 64 ? 64 : BM;
}
template <typename T>
static int launch_swiglu16(int bn, const CUtensorMap& am, const CUtensorMap& bm, int M, int N,
                           int K, const EpiArgs& e, cudaStream_t s,
                           const CUtensorMap* bm_pair = nullptr) {
  if (bm_pair && pair_rows(M)) {
    if (bn == 144 && (N + 143) / 144 <= max_pairs<T, 144, kPairStagesDeep, TI_EPI_SWIGLU16>())
      return launch_t<T, 144, kPairStagesDeep, TI_EPI_SWIGLU16, 1, BM, true>(am, *bm_pair, M, N, K,
                                                                              e, s);
    constexpr int kPs = pair_stages_shallow<256>();
    if (bn == 256 && M > kDeepRingMaxM && max_pairs<T, 256, kPs, TI_EPI_SWIGLU16>() > 0)
      return launch_t<T, 256, kPs, TI_EPI_SWIGLU16, 1, BM, true>(am, *bm_pair, M, N, K, e, s);
  }
  const int ar = swiglu16_box_rows(M, K, bn);
  if (ar == 32) return launch_t<T, 80, 14, TI_EPI_SWIGLU16, 1, 32>(am, bm, M, N, K, e, s);
  if (ar == 64) return launch_t<T, 80, 12, TI_EPI_SWIGLU16, 1, 64>(am, bm, M, N, K, e, s);
  switch (bn) {
    case 80: return launch_t<T, 80, TI_GEMM_STAGES_80, TI_EPI_SWIGLU16, 1>(am, bm, M, N, K, e, s);
    case 144: return launch_t<T, 144, TI_GEMM_STAGES_144, TI_EPI_SWIGLU16, 1>(am, bm, M, N, K, e, s);
    default:
      return M <= kDeepRingMaxM
                 ? launch_t<T, 256, TI_GEMM_STAGES_256, TI_EPI_SWIGLU16, 1>(am, bm, M, N, K, e, s)
                 : launch_t<T, 256, 2, TI_EPI_SWIGLU16, 1>(am, bm, M, N, K, e, s);
  }
}

}  // namespace gemm

int gemm_qkv_ctas(int M, int N, int K, int dtype) {
  return dtype == TI_DTYPE_BF16 ? gemm::qkv_ctas_t<__nv_bfloat16>(M, N, K)
                                : gemm::qkv_ctas_t<__half>(M, N, K);
}

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
  if (epilogue == TI_EPI_SWIGLU16) {   // the library picks the tile width; no split-K
    if (N % 16 || K % gemm::BK)
      return set_error(TI_ERR_UNSUPPORTED, "gemm: SwiGLU16 needs N % 16 == 0 and K % 64 == 0");
    block_n = gemm::swiglu16_bn(M, N);
    split_k = 1;
  } else {
    if (block_n <= 0) block_n = 128;
    if (N % block_n || K % gemm::BK)
      return set_error(TI_ERR_UNSUPPORTED, "gemm: N must be a multiple of block_n and K of 64");
  }
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15 || (lda % 8) || (ldb % 8))
    return set_error(TI_ERR_INVALID_ARGUMENT, "gemm: operands must be 16-byte aligned with ld % 8 == 0");
  const int cl = epilogue == TI_EPI_RESIDUAL ? std::max(1, std::min(split_k, gemm::kMaxResidualSplit))
                                             : gemm::cluster_for(split_k);
  if (cl > 1 && epilogue == TI_EPI_ARGMAX)
    return set_error(TI_ERR_UNSUPPORTED, "gemm: no split-K with the argmax epilogue");
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
  int rc;
  if (epilogue == TI_EPI_ARGMAX && !out && block_n == gemm::lmh::kBN && M <= kGemvMaxTokens &&
      K <= kGemvMaxK) {
    // few tokens: stream the weights through the swapped kernel, tokens resident (gemv.cu)
    return gemv_argmax(A, lda, B, ldb, false, nullptr, M, N, K, aux_val, aux_idx, dtype,
                       reinterpret_cast<cudaStream_t>(stream));
  }
  if (epilogue == TI_EPI_ARGMAX && !out && M <= 256 && block_n == gemm::lmh::kBN) {
    // greedy lm_head: persistent kernel, both 128-row halves per CTA
    rc = gemm::operand_map(&am, A, M, K, lda, 256, dtype);
    if (rc) return rc;
    rc = gemm::operand_map(&bm, B, N, K, ldb, gemm::lmh::kBN, dtype);
    if (rc) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    return dtype == TI_DTYPE_BF16
               ? gemm::launch_lmhead_argmax<__nv_bfloat16>(am, bm, M, N, K, aux_val, aux_idx, s)
               : gemm::launch_lmhead_argmax<__half>(am, bm, M, N, K, aux_val, aux_idx, s);
  }
  const int a_rows = epilogue == TI_EPI_SWIGLU16 ? gemm::swiglu16_box_rows(M, K, block_n) : gemm::BM;
  rc = gemm::operand_map(&am, A, M, K, lda, a_rows, dtype);
  if (rc) return rc;
  rc = gemm::operand_map(&bm, B, N, K, ldb, block_n, dtype);
  if (rc) return rc;
  // CTA pairs load half of each B tile per CTA (bf16 / fp16 SwiGLU16 and residual epilogues)
  CUtensorMap bm2;
  const CUtensorMap* bm_pair = nullptr;
  if (gemm::pair_rows(M) &&
      (epilogue == TI_EPI_SWIGLU16 || epilogue == TI_EPI_RESIDUAL)) {
    rc = gemm::operand_map(&bm2, B, N, K, ldb, block_n / 2, dtype);
    if (rc) return rc;
    bm_pair = &bm2;
  }
  gemm::EpiArgs e{};
  e.out = out; e.ldo = ldo; e.bias = bias; e.aux_val = aux_val; e.aux_idx = aux_idx;
  e.M = M; e.N = N; e.ntiles = N / block_n;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
#define TI_GEMM_KIND(T)                                                                       \
  switch (epilogue) {                                                                         \
    case TI_EPI_STORE: return gemm::dispatch_bn<T, TI_EPI_STORE>(block_n, cl, am, bm, M, N, K, e, s); \
    case TI_EPI_SWIGLU: return gemm::dispatch_bn<T, TI_EPI_SWIGLU>(block_n, cl, am, bm, M, N, K, e, s); \
    case TI_EPI_RESIDUAL:                                                                     \
      return gemm::dispatch_bn<T, TI_EPI_RESIDUAL>(block_n, cl, am, bm, M, N, K, e, s, bm_pair); \
    case TI_EPI_RESIDUAL_DET:                                                                 \
      return gemm::dispatch_bn<T, TI_EPI_RESIDUAL, true>(block_n, cl, am, bm, M, N, K, e, s);   \
    case TI_EPI_ARGMAX: return gemm::dispatch_bn<T, TI_EPI_ARGMAX>(block_n, 1, am, bm, M, N, K, e, s); \
    case TI_EPI_SWIGLU16:                                                                     \
      return gemm::launch_swiglu16<T>(block_n, am, bm, M, N, K, e, s, bm_pair);               \
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
