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
#include "capi_internal.h"
#include "common.cuh"

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
  if (dtype == TI_DTYPE_BF16)
    return head_dim == 64 ? prefill::launch<__nv_bfloat16, 64>(p, km, vm, num_tiles, s)
                          : prefill::launch<__nv_bfloat16, 128>(p, km, vm, num_tiles, s);
  return head_dim == 64 ? prefill::launch<__half, 64>(p, km, vm, num_tiles, s)
                        : prefill::launch<__half, 128>(p, km, vm, num_tiles, s);
}
