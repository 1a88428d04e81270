// Per-step packing kernels of the decode/prefill step (device side of the scheduler's
// engine/scheduler.py:224-281 and the model's pos_id / context-length glue,
// models/qwen_25.py:114-115,218-222), so a decode step needs no host-side tensor building:
//
//   ti_decode_prepare   apply this step's new block-table entries, then per row: position,
//                       pool slot, context length (seq_len + 1) and the embedding row
//   ti_argmax_finish    reduce the lm_head argmax partials to one token per row and advance
//                       seq_len of every live slot (the reference does seq_len += 1 after the
//                       forward, engine/scheduler.py:266)
//   ti_kv_scatter       write new K/V rows into the pool at given slots
//                       (engine/cache_manager.py:95-99)
#include <algorithm>

#include "capi_internal.h"
#include "common.cuh"

namespace ti {
namespace step {

template <typename T>
__global__ void decode_prepare_kernel(const int32_t* __restrict__ tokens,
                                      const int32_t* __restrict__ slots,
                                      const int32_t* __restrict__ new_block,
                                      const int32_t* __restrict__ seq_len, int32_t* block_tables,
                                      int64_t bt_stride, int num_slots, int max_blocks,
                                      int64_t num_blocks, int bs, int32_t* __restrict__ positions,
                                      int64_t* __restrict__ slot_mapping,
                                      int32_t* __restrict__ ctx_lens, float* __restrict__ hidden,
                                      const T* __restrict__ embed, int H, int64_t V, int rows) {
  pdl_wait();
  pdl_launch_dependents();
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int slot = slots[r];
  __shared__ int s_tok;
  if (threadIdx.x == 0) {
    int tok = tokens[r];
    // a slot outside the table, or a position past its last block column, is an input error
    // the host planner rules out: flagged, and the row is treated as padding (no writes)
    const int pos = (slot >= 0 && slot < num_slots) ? seq_len[slot] : -1;
    if (slot >= num_slots || (slot >= 0 && (pos < 0 || pos / bs >= max_blocks)))
      raise_device_error(TI_DEVERR_BAD_INPUT);
    if (slot < 0 || slot >= num_slots || pos < 0 || pos / bs >= max_blocks) {
      positions[r] = 0;
      slot_mapping[r] = -1;
      ctx_lens[r] = 0;
      tok = -1;
    } else {
      int32_t* row = block_tables + (int64_t)slot * bt_stride;
      const int nb = new_block[r];
      if (nb >= num_blocks) raise_device_error(TI_DEVERR_BAD_INPUT);
      else if (nb >= 0) row[pos / bs] = nb;
      const int blk = row[pos / bs];
      positions[r] = pos;
      // a block id outside the pool gets no KV write (attention treats it as absent too)
      slot_mapping[r] = (blk >= 0 && blk < num_blocks) ? (int64_t)blk * bs + pos % bs : -1;
      ctx_lens[r] = pos + 1;
    }
    s_tok = tok;
  }
  __syncthreads();
  const int64_t tok = s_tok;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float f[8];
    if (tok >= 0 && tok < V) {
      const uint4 u = *reinterpret_cast<const uint4*>(embed + tok * H + c);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 v = Elem<T>::unpack2(w[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = 0.f;
    }
    float4* o = reinterpret_cast<float4*>(hidden + (int64_t)r * H + c);
    o[0] = make_float4(f[0], f[1], f[2], f[3]);
    o[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

// One warp per row: max over the tiles, lowest token index among equal maxima.
__global__ void argmax_finish_kernel(const float* __restrict__ val, const int32_t* __restrict__ idx,
                                     int ntiles, int rows, int32_t* __restrict__ out_tokens,
                                     const int32_t* __restrict__ slots, int32_t* seq_len, int inc) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = lane; t < ntiles; t += 32) {
    const float v = val[(int64_t)warp * ntiles + t];
    const int i = idx[(int64_t)warp * ntiles + t];
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, best, o);
    const int i = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
  if (lane == 0) {
    out_tokens[warp] = (bi == 0x7fffffff) ? 0 : bi;   // an all-NaN row yields token 0
    if (seq_len && slots) {
      const int s = slots[warp];
      if (s >= 0) seq_len[s] += inc;
    }
  }
}

template <typename T>
__global__ void kv_scatter_kernel(T* k_cache, T* v_cache, const T* __restrict__ k,
                                  int64_t k_tok_stride, int64_t k_head_stride,
                                  const T* __restrict__ v, int64_t v_tok_stride,
                                  int64_t v_head_stride, const int64_t* __restrict__ slots,
                                  int64_t pool_slots, int tokens, int KVH, int HD, int bs) {
  pdl_wait();
  pdl_launch_dependents();
  const int per = KVH * (HD / 8);
  const int64_t total = (int64_t)tokens * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / per);
    const int r = (int)(i % per);
    const int h = r / (HD / 8), d = (r % (HD / 8)) * 8;
    const int64_t slot = slots[t];
    if (slot < 0) continue;
    if (slot >= pool_slots) {          // outside the pool: flagged, not written
      if (r == 0) raise_device_error(TI_DEVERR_BAD_INPUT);
      continue;
    }
    const int64_t dst = (((slot / bs) * KVH + h) * bs + slot % bs) * HD + d;
    *reinterpret_cast<uint4*>(k_cache + dst) =
        *reinterpret_cast<const uint4*>(k + t * k_tok_stride + h * k_head_stride + d);
    *reinterpret_cast<uint4*>(v_cache + dst) =
        *reinterpret_cast<const uint4*>(v + t * v_tok_stride + h * v_head_stride + d);
  }
}

}  // namespace step
}  // namespace ti

using namespace ti;

extern "C" int ti_decode_prepare(const int32_t* tokens, const int32_t* slots,
                                 const int32_t* new_block, const int32_t* seq_len,
                                 int32_t* block_tables, int64_t bt_stride, int num_slots,
                                 int max_blocks_per_seq, int64_t num_blocks, int block_size,
                                 int32_t* positions, int64_t* slot_mapping, int32_t* ctx_lens,
                                 float* hidden, const void* embed, int hidden_size, int64_t vocab,
                                 int rows, int dtype, void* stream) {
  clear_error();
  if (rows == 0) return TI_OK;
  if (!tokens || !slots || !new_block || !seq_len || !block_tables || !positions ||
      !slot_mapping || !ctx_lens || !hidden || !embed || rows < 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "decode_prepare: null pointer");
  if (num_slots <= 0 || max_blocks_per_seq <= 0 || num_blocks <= 0 || block_size <= 0 ||
      bt_stride < max_blocks_per_seq)
    return set_error(TI_ERR_INVALID_ARGUMENT, "decode_prepare: bad block-table or pool shape");
  if (hidden_size % 8) return set_error(TI_ERR_UNSUPPORTED, "decode_prepare: hidden % 8 != 0");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16)
    return launch_kernel("decode_prepare launch", step::decode_prepare_kernel<__nv_bfloat16>,
                         dim3(rows), dim3(128), 0, s, 1,
        tokens, slots, new_block, seq_len, block_tables, bt_stride, num_slots, max_blocks_per_seq,
        num_blocks, block_size, positions, slot_mapping, ctx_lens, hidden,
        (const __nv_bfloat16*)embed, hidden_size, vocab, rows);
  else if (dtype == TI_DTYPE_FP16)
    return launch_kernel("decode_prepare launch", step::decode_prepare_kernel<__half>,
                         dim3(rows), dim3(128), 0, s, 1,
        tokens, slots, new_block, seq_len, block_tables, bt_stride, num_slots, max_blocks_per_seq,
        num_blocks, block_size, positions, slot_mapping, ctx_lens, hidden, (const __half*)embed,
        hidden_size, vocab, rows);
  else
    return set_error(TI_ERR_UNSUPPORTED, "decode_prepare: dtype must be bf16 or fp16");
}

extern "C" int ti_argmax_finish(const float* part_val, const int32_t* part_idx, int ntiles,
                                int rows, int32_t* out_tokens, const int32_t* slots,
                                int32_t* seq_len, int seq_inc, void* stream) {
  clear_error();
  if (rows == 0) return TI_OK;
  if (!part_val || !part_idx || !out_tokens || ntiles <= 0 || rows < 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "argmax_finish: bad arguments");
  const int threads = 256;
  const int blocks = (rows * 32 + threads - 1) / threads;
  return launch_kernel("argmax_finish launch", step::argmax_finish_kernel,
                       dim3(blocks), dim3(threads), 0, reinterpret_cast<cudaStream_t>(stream), 1,
      part_val, part_idx, ntiles, rows, out_tokens, slots, seq_len, seq_inc);
}

extern "C" int ti_kv_scatter(void* k_cache, void* v_cache, const void* k, int64_t k_tok_stride,
                             int64_t k_head_stride, const void* v, int64_t v_tok_stride,
                             int64_t v_head_stride, const int64_t* slot_mapping, int num_tokens,
                             int64_t num_blocks, int num_kv_heads, int head_dim, int block_size,
                             int dtype, void* stream) {
  clear_error();
  if (num_tokens == 0) return TI_OK;
  if (!k_cache || !v_cache || !k || !v || !slot_mapping || num_tokens < 0 || num_blocks <= 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "kv_scatter: null pointer or empty pool");
  const int64_t pool_slots = num_blocks * block_size;
  if (head_dim % 8 || (k_tok_stride | k_head_stride | v_tok_stride | v_head_stride) % 8 ||
      ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15))
    return set_error(TI_ERR_INVALID_ARGUMENT, "kv_scatter: rows must be 16-byte aligned");
  const int64_t work = (int64_t)num_tokens * num_kv_heads * (head_dim / 8);
  const int blocks = (int)std::min<int64_t>((work + 255) / 256, 148 * 16);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16)
    return launch_kernel("kv_scatter launch", step::kv_scatter_kernel<__nv_bfloat16>,
                         dim3(blocks), dim3(256), 0, s, 1,
        (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, (const __nv_bfloat16*)k, k_tok_stride,
        k_head_stride, (const __nv_bfloat16*)v, v_tok_stride, v_head_stride, slot_mapping,
        pool_slots, num_tokens, num_kv_heads, head_dim, block_size);
  else if (dtype == TI_DTYPE_FP16)
    return launch_kernel("kv_scatter launch", step::kv_scatter_kernel<__half>,
                         dim3(blocks), dim3(256), 0, s, 1,
        (__half*)k_cache, (__half*)v_cache, (const __half*)k, k_tok_stride, k_head_stride,
        (const __half*)v, v_tok_stride, v_head_stride, slot_mapping, pool_slots, num_tokens,
        num_kv_heads, head_dim, block_size);
  else
    return set_error(TI_ERR_UNSUPPORTED, "kv_scatter: dtype must be bf16 or fp16");
}
