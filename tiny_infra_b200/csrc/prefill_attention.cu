// Ragged causal prefill attention over the paged KV pool, sm_100a.
//
// The reference prefills one whole prompt per call with F.scaled_dot_product_attention over
// that call's own K/V (models/qwen_25.py:89-104), which is only correct because prefill always
// starts at position 0.  This kernel reads K/V from the paged pool instead, so a chunk of new
// tokens at positions start..start+S-1 attends to every earlier token of its sequence (chunked
// prefill) and any number of sequences are packed in one launch; for start == 0 it computes the
// same causal attention as the reference (scale 1/sqrt(D), GQA by repetition).
//
// Work decomposition: one CTA per (query tile of 16 tokens of one sequence, kv head).  Warp w
// (w < G) owns query head kvh*G + w for the 16 tokens (M = 16 rows of mma.sync m16n8k16);
// warp G is a TMA producer that streams the sequence's KV blocks (16 tokens x D per block and
// kv head, SWIZZLE_128B) through a 4-stage ring; all G compute warps share every K/V tile, so
// each KV byte is read once per CTA for the whole GQA group.
#include <cstdlib>
#include <type_traits>
#include <cstring>

#include "capi_internal.h"
#include "common.cuh"
#include "tcgen05.cuh"

namespace ti {
namespace prefill {

constexpr int kBlock = 16;
constexpr int kStages = 4;
constexpr int kTileQ = 16;
constexpr int kMaxGroup = 16;

struct Params {
  void* out;
  const void* q;
  int64_t out_stride, q_stride;      // elements between consecutive query tokens
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* row_index;          // [nseq] block-table row of each sequence
  const int32_t* start_pos;          // [nseq] position of the chunk's first token
  const int32_t* cu_seqlens;         // [nseq+1] query-row offsets of each chunk
  const int32_t* tile_seq;           // [num_tiles] sequence of each query tile
  const int32_t* tile_q0;            // [num_tiles] first query token (within the chunk)
  int num_heads, num_kv_heads, group;
  int64_t num_blocks;
  float scale_log2;
};

template <int HD>
struct Smem {
  static constexpr int kTile = kBlock * HD * 2;
  static constexpr int kStage = 2 * kTile;
  static constexpr int kTotal = kStages * kStage + 2 * kStages * 8 + 1024;
};

template <typename T, int HD>
__global__ void prefill_kernel(const __grid_constant__ CUtensorMap kmap,
                               const __grid_constant__ CUtensorMap vmap, Params p) {
  pdl_wait();
  pdl_launch_dependents();
  using S = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t full0 = smem_u32(smem + kStages * S::kStage);
  const uint32_t empty0 = full0 + kStages * 8;
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.group;

  const int seq = p.tile_seq[tile];
  const int q0 = p.tile_q0[tile];
  const int row0 = p.cu_seqlens[seq] + q0;
  const int nq = min(kTileQ, p.cu_seqlens[seq + 1] - row0);
  const int start = p.start_pos[seq];
  const int last_pos = start + q0 + nq - 1;           // causal bound of this tile
  const int nblk = last_pos / kBlock + 1;
  const int32_t* bt = p.block_tables + (int64_t)p.row_index[seq] * p.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, G);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == G) {   // ---- producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();   // later query tiles re-read these blocks
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kStages;
        if (j >= kStages &&
            !mbar_wait(empty0 + 8 * s, ((j / kStages) & 1) ^ 1, TI_DEVERR_PREFILL_WAIT))
          break;
        int pb = bt[j];
        if (pb < 0 || (int64_t)pb >= p.num_blocks) pb = 0;   // never read outside the pool
        const uint32_t dst = smem_u32(smem + s * S::kStage);
        mbar_arrive_expect_tx(full0 + 8 * s, S::kStage);
        const int y = (pb * p.num_kv_heads + kvh) * kBlock;
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d_hint(dst + c * kBlock * 128, &kmap, full0 + 8 * s, c * 64, y, pol);
          tma_load_2d_hint(dst + S::kTile + c * kBlock * 128, &vmap, full0 + 8 * s, c * 64, y, pol);
        }
      }
    }
    return;
  }

  // ---- compute warps: head h, 16 query tokens as the M rows
  const int h = kvh * G + warp;
  const int g = lane >> 2, t4 = lane & 3;
  const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)row0 * p.q_stride + (int64_t)h * HD;
  uint32_t qa[HD / 16][4];
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int tr = g + ((r & 1) ? 8 : 0);
      const int col = ks * 16 + 2 * t4 + ((r & 2) ? 8 : 0);
      qa[ks][r] = (tr < nq) ? *reinterpret_cast<const uint32_t*>(qb + (int64_t)tr * p.q_stride + col) : 0u;
    }
  const int qpos0 = start + q0 + g, qpos1 = qpos0 + 8;   // positions of rows g and g+8

  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (int j = 0; j < nblk; ++j) {
    const int s = j % kStages;
    if (!mbar_wait(full0 + 8 * s, (j / kStages) & 1, TI_DEVERR_PREFILL_WAIT)) break;
    const uint32_t kb = smem_u32(smem + s * S::kStage);
    const uint32_t vb = kb + S::kTile;
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const int mi = lane >> 3;
      const int tok = ((mi & 2) ? 8 : 0) + (lane & 7);
      const int chunk = ks * 2 + (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kb + (chunk >> 3) * kBlock * 128 + swz128(tok, chunk & 7), b0, b1, b2, b3);
      Mma<T>::run(sc[0], qa[ks], b0, b1);
      Mma<T>::run(sc[1], qa[ks], b2, b3);
    }
    const int kv0 = j * kBlock;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kp = kv0 + nt * 8 + 2 * t4 + (e & 1);
        const int qp = (e & 2) ? qpos1 : qpos0;
        sc[nt][e] = (kp <= qp) ? sc[nt][e] * p.scale_log2 : -INFINITY;
      }
    float mx[2];
    mx[0] = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    mx[1] = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mn = fmaxf(m_r[r], mx[r]);
      // block 0 always holds position 0 <= every query position, so mn is finite from j = 0
      alpha[r] = fast_exp2(m_r[r] - mn);
      m_r[r] = mn;
    }
    float pr[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) pr[nt][e] = fast_exp2(sc[nt][e] - m_r[e >> 1]);
    l_r[0] = l_r[0] * alpha[0] + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    l_r[1] = l_r[1] * alpha[1] + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0]; o[i][1] *= alpha[0];
      o[i][2] *= alpha[1]; o[i][3] *= alpha[1];
    }
    uint32_t pa[4], pl[4];
    split_p<T>(pr, pa, pl);
    // keys past the last query position of the tile are masked (P = 0); their V rows hold
    // whatever the pool has there, finite values written by earlier appends or the zero fill
#pragma unroll
    for (int nt = 0; nt < HD / 8; nt += 2) {
      const int mi = lane >> 3;
      const int tok = ((mi & 1) ? 8 : 0) + (lane & 7);
      const int chunk = nt + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vb + (chunk >> 3) * kBlock * 128 + swz128(tok, chunk & 7), b0, b1, b2, b3);
      Mma<T>::run(o[nt], pa, b0, b1);
      Mma<T>::run(o[nt + 1], pa, b2, b3);
      if constexpr (kSplitP<T>) {
        Mma<T>::run(o[nt], pl, b0, b1);
        Mma<T>::run(o[nt + 1], pl, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  T* ob = reinterpret_cast<T*>(p.out) + (int64_t)row0 * p.out_stride + (int64_t)h * HD;
  const float inv0 = 1.f / l_r[0], inv1 = 1.f / l_r[1];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int col = i * 8 + 2 * t4;
    if (g < nq)
      *reinterpret_cast<uint32_t*>(ob + (int64_t)g * p.out_stride + col) =
          Elem<T>::pack2(o[i][0] * inv0, o[i][1] * inv0);
    if (g + 8 < nq)
      *reinterpret_cast<uint32_t*>(ob + (int64_t)(g + 8) * p.out_stride + col) =
          Elem<T>::pack2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

template <typename T, int HD>
static int launch(const Params& p, const CUtensorMap& km, const CUtensorMap& vm, int num_tiles,
                  cudaStream_t s) {
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel<T, HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<HD>::kTotal);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(prefill)");
    set_dev = dev;
  }
  dim3 grid(num_tiles, p.num_kv_heads);
  return launch_kernel("prefill attention launch", prefill_kernel<T, HD>, grid,
                       dim3((p.group + 1) * 32), Smem<HD>::kTotal, s, 1, km, vm, p);
}


// ==========================================================================================
// tcgen05 variant (head_dim 64, GQA groups <= 8): one CTA per (query tile of 16 tokens, kv
// head); the 128 MMA rows are (query head slot h < 8) x (token t < 16), row = 16 h + t.
//   S = Q K^T   M=128, N=64 keys, K=64 dims: Q (K-major) once in shared memory, a 64-key chunk of
//               K (4 pool blocks, K-major) per step; fp32 S in one of two TMEM buffers;
//   softmax     warps 2-5, one row per thread, straight from TMEM: causal mask, running max kept
//               until a row's max grows by more than 2^8 (then O is rescaled in TMEM), P = 2^(s-m)
//               split into bf16 hi + lo (~2^-17 relative, as the mma.sync kernels) and written
//               to shared memory in the MMA's K-major layout;
//   O += P V    M=128, N=64 dims, K=64 keys, twice (hi, lo), with V read in place as an MN-major
//               operand (rows = keys); fp32 O in TMEM.
// Warp 0 streams K/V chunks through a 3-stage TMA ring, warp 1 issues the MMAs (S of chunk j
// before P.V of chunk j-1, so the softmax of j overlaps the P.V of j-1).  Every wait is bounded.
// ==========================================================================================
namespace tc {
__device__ __forceinline__ void st_shared_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z,
                                             uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
constexpr int kChunk = 64;                     // keys per step
constexpr int kStages = 3;
constexpr int kTile = kChunk * 128;            // 64 rows x 128 bytes: K or V of one chunk
constexpr int kQ = 0, kPhi = 16384, kPlo = 32768, kKV = 49152;
constexpr int kStageBytes = 2 * kTile;
constexpr int kBarOff = kKV + kStages * kStageBytes;       // 98304
constexpr int kSmem = kBarOff + 256 + 1024;                 // barriers + alignment slack
constexpr int kTmemCols = 256;                 // S buffers at 0 and 64, O at 128
constexpr int kThreads = 192;
// Split-key cluster: each CTA's un-normalised partial (O rows, then (m, l) per row) goes over
// its drained K/V ring; rows padded to 68 floats so that 8 consecutive rows start on 8
// different 16-byte bank groups.
constexpr int kPartStride = 68;
constexpr int kPartMl = kKV + 128 * kPartStride * 4;
static_assert(kPartMl + 128 * 16 <= kBarOff, "partials fit the K/V ring");

template <typename T>
__global__ void __launch_bounds__(kThreads)
prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                  Params p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const uint32_t bars = sb + kBarOff;
  const uint32_t kv_full = bars, kv_empty = bars + 8 * kStages;
  const uint32_t s_full = bars + 16 * kStages, s_free = s_full + 16;
  const uint32_t p_ready = s_free + 16, pv_done = p_ready + 8;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kBarOff + 128);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int G = p.group;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < kStages; ++i) {
        mbar_init(kv_full + 8 * i, 1);
        mbar_init(kv_empty + 8 * i, 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(s_full + 8 * i, 1);
        mbar_init(s_free + 8 * i, 4);
      }
      mbar_init(p_ready, 4);
      mbar_init(pv_done, 1);
      fence_mbar_init();
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    __syncwarp();
    tmem_alloc(smem_u32(tslot), kTmemCols);
  }
  pdl_wait();   // q, the pool's K/V and the tables come from earlier kernels

  const int seq = p.tile_seq[tile];
  const int q0 = p.tile_q0[tile];
  const int row0 = p.cu_seqlens[seq] + q0;
  const int nq = min(kTileQ, p.cu_seqlens[seq + 1] - row0);
  const int start = p.start_pos[seq];
  const int nkeys = start + q0 + nq;                  // keys 0 .. last query position
  const int nchunks = (nkeys + kChunk - 1) / kChunk;
  const int32_t* bt = p.block_tables + (int64_t)p.row_index[seq] * p.bt_stride;
  // Split-key cluster (gridDim.z == 2): CTA 0 takes key chunks [0, c_mid), CTA 1 the rest, and
  // the two partials are merged through distributed shared memory, so a long prefix costs each
  // CTA about half of it.  c_mid never passes the tile's first query position: every row of
  // CTA 1 sees a key in its first chunk, so its running max is finite from the start.
  const bool split = gridDim.z > 1;
  const int c_mid = split ? min(nchunks / 2, (start + q0) / kChunk) : 0;
  const int c_begin = split && blockIdx.z == 1 ? c_mid : 0;
  const int n_local = split ? (blockIdx.z == 0 ? c_mid : nchunks - c_mid) : nchunks;

  // ---- Q tile: row 16 h + t = query head kvh*G + h of token row0 + t (zero when h >= G or
  //      t >= nq), swizzled K-major
  for (int i = tid; i < 128 * 8; i += kThreads) {
    const int r = i >> 3, c = i & 7, h = r >> 4, t = r & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (h < G && t < nq)
      v = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) +
                                          (int64_t)(row0 + t) * p.q_stride +
                                          (int64_t)(kvh * G + h) * 64 + c * 8);
    *reinterpret_cast<uint4*>(smem + kQ + r * 128 + ((c ^ (r & 7)) << 4)) = v;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---- producer: chunk j = blocks 4j .. 4j+3 (past the keys: block 0, masked later)
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();   // later query tiles re-read these blocks
      for (int jj = 0; jj < n_local; ++jj) {
        const int j = c_begin + jj, st = jj % kStages;
        if (jj >= kStages &&
            !mbar_wait(kv_empty + 8 * st, ((jj / kStages) - 1) & 1, TI_DEVERR_PREFILL_WAIT))
          break;
        const uint32_t dst = sb + kKV + st * kStageBytes;
        mbar_arrive_expect_tx(kv_full + 8 * st, kStageBytes);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int blk = 4 * j + b;
          int pb = blk * kBlock < nkeys ? bt[blk] : 0;
          if (pb < 0 || (int64_t)pb >= p.num_blocks) pb = 0;   // never read outside the pool
          const int y = (pb * p.num_kv_heads + kvh) * kBlock;
          tma_load_2d_hint(dst + b * 2048, &kmap, kv_full + 8 * st, 0, y, pol);
          tma_load_2d_hint(dst + kTile + b * 2048, &vmap, kv_full + 8 * st, 0, y, pol);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t id_s = idesc_f16(128, kChunk, bf, false, false);
      constexpr uint32_t id_pv = idesc_f16(128, 64, bf, false, true);
      bool ok = true;
      for (int j = 0; j <= n_local && ok; ++j) {   // this CTA's chunks, counted from 0
        if (j < n_local) {
          const int st = j % kStages, b = j & 1;
          ok = mbar_wait(kv_full + 8 * st, (j / kStages) & 1, TI_DEVERR_PREFILL_WAIT);
          if (ok && j >= 2) ok = mbar_wait(s_free + 8 * b, ((j >> 1) - 1) & 1, TI_DEVERR_PREFILL_WAIT);
          if (!ok) break;
          tc_fence_after();
          const uint32_t kt = sb + kKV + st * kStageBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma(tmem + b * kChunk, smem_desc_sw128(sb + kQ + 32 * k, false),
                   smem_desc_sw128(kt + 32 * k, false), id_s, k > 0 ? 1u : 0u);
          tc_commit(s_full + 8 * b);
        }
        if (j >= 1) {
          const int jp = j - 1, sp = jp % kStages;
          ok = mbar_wait(p_ready, jp & 1, TI_DEVERR_PREFILL_WAIT);
          if (!ok) break;
          tc_fence_after();
          const uint32_t vt = sb + kKV + sp * kStageBytes + kTile;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma(tmem + 128, smem_desc_sw128(sb + kPhi + 32 * k, false),
                   smem_desc_sw128(vt + 2048 * k, true), id_pv, (jp > 0 || k > 0) ? 1u : 0u);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma(tmem + 128, smem_desc_sw128(sb + kPlo + 32 * k, false),
                   smem_desc_sw128(vt + 2048 * k, true), id_pv, 1u);
          tc_commit(pv_done);
          tc_commit(kv_empty + 8 * sp);
        }
      }
    }
  } else {
    // ---- softmax and epilogue: thread <-> row (TMEM lane) r
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int h = r >> 4, t = r & 15;
    const int qp = start + q0 + t;                    // query position of the row
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    // the TMEM loads / stores after a wait are warp-collective: a warp goes on only when all
    // its lanes saw the phase (a timeout in one lane stops the whole warp)
    auto wait_all = [&](uint32_t bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, TI_DEVERR_PREFILL_WAIT));
    };
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_local; ++j) {   // this CTA's chunks, counted from 0
      const int b = j & 1;
      if (!wait_all(s_full + 8 * b, (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      float sv[kChunk];
      tmem_ld32(trow + b * kChunk, sv);
      tmem_ld32(trow + b * kChunk + 32, sv + 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free + 8 * b);
      const int k0 = (c_begin + j) * kChunk;
      // only chunks that reach past the tile's first query position need the causal mask (the
      // test is the same for the whole CTA)
      if (k0 + kChunk - 1 > start + q0) {
#pragma unroll
        for (int c = 0; c < kChunk; ++c) sv[c] = (k0 + c <= qp) ? sv[c] : -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kChunk; ++c) mx = fmaxf(mx, sv[c]);
      mx *= p.scale_log2;   // the scale is positive: max(s) * scale = max(s * scale)
      // the first chunk holds a key <= every query position, so m is finite from the start
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m = mx;
      } else if (mx > m + 8.f) {
        alpha = fast_exp2(m - mx);
        m = mx;
        rescale = true;
      }
      l *= alpha;
      uint32_t hi[kChunk / 2], lo[kChunk / 2];
#pragma unroll
      for (int c = 0; c < kChunk; c += 2) {
        const float p0 = fast_exp2(fmaf(sv[c], p.scale_log2, -m));   // 2^(s scale - m)
        const float p1 = fast_exp2(fmaf(sv[c + 1], p.scale_log2, -m));
        l += p0 + p1;
        const uint32_t h2 = Elem<T>::pack2(p0, p1);
        const float2 hf = Elem<T>::unpack2(h2);
        hi[c / 2] = h2;
        lo[c / 2] = Elem<T>::pack2(p0 - hf.x, p1 - hf.y);
      }
      if (j >= 1) {   // P.V of the previous chunk is done: P buffers free, O current
        if (!wait_all(pv_done, (j - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        // tcgen05.ld / st are warp-collective (.sync.aligned): the whole warp takes the branch
        // when any of its rows rescales (alpha is 1 for the others)
        if (__any_sync(0xffffffffu, rescale)) {
          float ov[32];
#pragma unroll
          for (int c = 0; c < 64; c += 32) {
            tmem_ld32(trow + 128 + c, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_st32(trow + 128 + c, ov);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {   // 16-byte chunk c = keys 8c .. 8c+7
        const uint32_t off = (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
        st_shared_v4(sb + kPhi + off, hi[4 * c], hi[4 * c + 1], hi[4 * c + 2], hi[4 * c + 3]);
        st_shared_v4(sb + kPlo + off, lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
    }
    bool have = false;
    float ov[64];
    if (ok && n_local > 0 && wait_all(pv_done, (n_local - 1) & 1)) {
      tc_fence_after();
      tmem_ld32(trow + 128, ov);
      tmem_ld32(trow + 160, ov + 32);
      have = true;
    }
    if (split) {
      // this CTA's partial row (zeros, m = -inf and l = 0 without chunks) for the cluster merge
      const uint32_t po = sb + kKV + (uint32_t)(r * kPartStride) * 4;
#pragma unroll
      for (int c = 0; c < 64; c += 4)
        st_shared_v4(po + c * 4, __float_as_uint(have ? ov[c] : 0.f),
                     __float_as_uint(have ? ov[c + 1] : 0.f), __float_as_uint(have ? ov[c + 2] : 0.f),
                     __float_as_uint(have ? ov[c + 3] : 0.f));
      st_shared_v4(sb + kPartMl + r * 16, __float_as_uint(have ? m : -INFINITY),
                   __float_as_uint(have ? l : 0.f), 0u, 0u);
    } else if (have) {
      if (h < G && t < nq) {
        const float inv = 1.f / l;
        T* dst = reinterpret_cast<T*>(p.out) + (int64_t)(row0 + t) * p.out_stride +
                 (int64_t)(kvh * G + h) * 64;
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          uint4 u;
          u.x = Elem<T>::pack2(ov[c] * inv, ov[c + 1] * inv);
          u.y = Elem<T>::pack2(ov[c + 2] * inv, ov[c + 3] * inv);
          u.z = Elem<T>::pack2(ov[c + 4] * inv, ov[c + 5] * inv);
          u.w = Elem<T>::pack2(ov[c + 6] * inv, ov[c + 7] * inv);
          *reinterpret_cast<uint4*>(dst + c) = u;
        }
      }
    }
  }
  if (split) {
    __syncwarp();     // warps 0 / 1: lane 0 ran the producer / MMA loop alone
    cluster_sync();   // both CTAs' partials are in shared memory
    if (warp >= 2) {
      // rows [64 z, 64 z + 64) of the tile: two threads per row, 32 dims each; the two partials
      // are read in a fixed order (deterministic)
      const int i = tid - 64;
      const int row = (int)blockIdx.z * 64 + (i >> 1), half = i & 1;
      const int hh = row >> 4, tt = row & 15;
      const uint32_t po = sb + kKV + (uint32_t)(row * kPartStride + half * 32) * 4;
      const uint32_t pm = sb + kPartMl + (uint32_t)row * 16;
      const float4 a = ld_peer_f4(map_peer(pm, 0)), b = ld_peer_f4(map_peer(pm, 1));
      const float mm = fmaxf(a.x, b.x);
      const float fa = a.x == -INFINITY ? 0.f : fast_exp2(a.x - mm);
      const float fb = b.x == -INFINITY ? 0.f : fast_exp2(b.x - mm);
      const float inv = 1.f / (fa * a.y + fb * b.y);
      const uint32_t pa = map_peer(po, 0), pb = map_peer(po, 1);
      if (hh < G && tt < nq) {
        T* dst = reinterpret_cast<T*>(p.out) + (int64_t)(row0 + tt) * p.out_stride +
                 (int64_t)(kvh * G + hh) * 64 + half * 32;
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          const float4 x0 = ld_peer_f4(pa + c * 4), x1 = ld_peer_f4(pa + c * 4 + 16);
          const float4 y0 = ld_peer_f4(pb + c * 4), y1 = ld_peer_f4(pb + c * 4 + 16);
          uint4 u;
          u.x = Elem<T>::pack2((fa * x0.x + fb * y0.x) * inv, (fa * x0.y + fb * y0.y) * inv);
          u.y = Elem<T>::pack2((fa * x0.z + fb * y0.z) * inv, (fa * x0.w + fb * y0.w) * inv);
          u.z = Elem<T>::pack2((fa * x1.x + fb * y1.x) * inv, (fa * x1.y + fb * y1.y) * inv);
          u.w = Elem<T>::pack2((fa * x1.z + fb * y1.z) * inv, (fa * x1.w + fb * y1.w) * inv);
          *reinterpret_cast<uint4*>(dst + c) = u;
        }
      }
    }
    cluster_sync();   // the peer has finished reading this CTA's partials
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

static bool split_keys() {
  const char* e = getenv("TI_PREFILL_ATTN_SPLIT");
  return !(e && !strcmp(e, "0"));
}

template <typename T>
static int launch(const Params& p, const CUtensorMap& km, const CUtensorMap& vm, int num_tiles,
                  cudaStream_t s) {
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(prefill tc)");
    set_dev = dev;
  }
  // every tile as a cluster of two CTAs splitting its keys (TI_PREFILL_ATTN_SPLIT=0: one CTA)
  const int z = split_keys() ? 2 : 1;
  return launch_kernel("prefill attention launch", prefill_tc_kernel<T>,
                       dim3(num_tiles, p.num_kv_heads, z), dim3(kThreads), kSmem, s, z, km, vm, p);
}
}  // namespace tc

// TI_PREFILL_ATTN_KERNEL=mma forces the mma.sync kernel (comparisons and tests).
static bool use_tc(int head_dim, int group) {
  const char* e = getenv("TI_PREFILL_ATTN_KERNEL");
  if (e && !strcmp(e, "mma")) return false;
  return head_dim == 64 && group <= 8;
}
}  // namespace prefill
}  // namespace ti

using namespace ti;

extern "C" int ti_paged_prefill_attention(
    void* out, int64_t out_tok_stride, const void* q, int64_t q_tok_stride, const void* k_cache,
    const void* v_cache, int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
    const int32_t* row_index, const int32_t* start_pos, const int32_t* cu_seqlens,
    const int32_t* tile_seq, const int32_t* tile_q0, int num_tiles, int num_heads,
    int num_kv_heads, int head_dim, int block_size, int dtype, void* stream) {
  clear_error();
  if (num_tiles == 0) return TI_OK;
  if (!out || !q || !k_cache || !v_cache || !block_tables || !row_index || !start_pos ||
      !cu_seqlens || !tile_seq || !tile_q0 || num_tiles < 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "prefill attention: null pointer");
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads ||
      num_heads / num_kv_heads > prefill::kMaxGroup)
    return set_error(TI_ERR_UNSUPPORTED, "prefill attention: 1..16 query heads per kv head");
  if (head_dim != 64 && head_dim != 128)
    return set_error(TI_ERR_UNSUPPORTED, "prefill attention: head_dim must be 64 or 128");
  if (block_size != prefill::kBlock)
    return set_error(TI_ERR_UNSUPPORTED, "prefill attention: block_size must be 16");
  if (dtype != TI_DTYPE_BF16 && dtype != TI_DTYPE_FP16)
    return set_error(TI_ERR_UNSUPPORTED, "prefill attention: dtype must be bf16 or fp16");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (q_tok_stride & 1) ||
      (reinterpret_cast<uintptr_t>(out) & 3) || (out_tok_stride & 1))
    return set_error(TI_ERR_INVALID_ARGUMENT, "prefill attention: q/out must be 4-byte aligned");
  if (num_tiles > 0x7fffffff || num_kv_heads > 65535)
    return set_error(TI_ERR_UNSUPPORTED, "prefill attention: grid too large");
  prefill::Params p{};
  p.out = out; p.q = q; p.out_stride = out_tok_stride; p.q_stride = q_tok_stride;
  p.block_tables = block_tables; p.bt_stride = bt_stride; p.row_index = row_index;
  p.start_pos = start_pos; p.cu_seqlens = cu_seqlens; p.tile_seq = tile_seq; p.tile_q0 = tile_q0;
  p.num_heads = num_heads; p.num_kv_heads = num_kv_heads; p.group = num_heads / num_kv_heads;
  p.num_blocks = num_blocks;
  p.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  const int64_t rows = num_blocks * num_kv_heads * prefill::kBlock;
  cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)prefill::kBlock};
  cuuint32_t es[2] = {1, 1};
  const CUtensorMapDataType tt =
      dtype == TI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap km, vm;
  int rc = encode_tensor_map_2d(&km, tt, const_cast<void*>(k_cache), dims, strides, box, es,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  rc = encode_tensor_map_2d(&vm, tt, const_cast<void*>(v_cache), dims, strides, box, es,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (prefill::use_tc(head_dim, p.group))
    return dtype == TI_DTYPE_BF16 ? prefill::tc::launch<__nv_bfloat16>(p, km, vm, num_tiles, s)
                                  : prefill::tc::launch<__half>(p, km, vm, num_tiles, s);
  if (dtype == TI_DTYPE_BF16)
    return head_dim == 64 ? prefill::launch<__nv_bfloat16, 64>(p, km, vm, num_tiles, s)
                          : prefill::launch<__nv_bfloat16, 128>(p, km, vm, num_tiles, s);
  return head_dim == 64 ? prefill::launch<__half, 64>(p, km, vm, num_tiles, s)
                        : prefill::launch<__half, 128>(p, km, vm, num_tiles, s);
}
