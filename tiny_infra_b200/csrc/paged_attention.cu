// Paged decode attention for sm_100a.
//
// Replaces the reference's paged_attention_kernel / launch_paged_attention
// (src/attention.cu:54-154, :156-197) with the same results:
//   * single query per sequence, GQA: query head h reads kv head h / (NH / KVH)  (attention.cu:92)
//   * scale 1/sqrt(D) on the scores                                                (attention.cu:70,184)
//   * ctx == 0: output row left untouched                                          (attention.cu:62)
//   * reading stops at the first negative block-table entry                        (attention.cu:90)
//   * no token read at all -> 0/0 = NaN output                                     (attention.cu:150)
//
// B200 design (the reference is one 64-thread CTA per (head, seq) with a block-reduce per token):
//   * One CTA per (partition, kv head, sequence).  A partition is up to 16 KV blocks (256
//     tokens); long contexts are split across partitions (split-K / flash-decoding) and the last
//     CTA to finish a (sequence, kv head) merges the partials (atomic arrival counter, no spin).
//   * Each KV block of one kv head is a contiguous 16 x D tile in the pool; one elected thread
//     issues all TMA tile loads of the partition up front (SWIZZLE_128B), so the whole partition
//     is in flight at once.  Every K/V byte is read from HBM exactly once per kv head: all
//     query heads of the GQA group are served from the same shared-memory tile.
//   * Scores and P.V run on tensor cores with mma.sync m16n8k16: the GQA group (7 query heads
//     for Qwen2.5-0.5B) forms the M dimension, the 16 tokens of a block the N (or K) dimension.
//     The kernel is HBM-bound (about 7 flop per KV byte), so register-fragment MMAs are ample;
//     tcgen05 would need M >= 64 and add TMEM round trips for the softmax.
//   * Four warps per CTA; each warp owns every fourth block of the partition and keeps its own
//     online-softmax state; the CTA merges the four states in shared memory.
#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "capi_internal.h"
#include "common.cuh"

namespace ti {
namespace attn {

constexpr int kBlock = 16;          // tokens per KV block (the pool's block_size)
constexpr int kMaxPart = 16;        // KV blocks per partition (max)
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxGroup = 16;       // query heads per kv head handled by one 16-row MMA tile
// Split-K arrival counters live at the start of the workspace, one int32 per (sequence, kv
// head), in a fixed region so that calls with different shapes never see scratch data there.
constexpr int kMaxCounters = 16384;
constexpr int64_t kCounterBytes = kMaxCounters * 4;

template <int HD>
struct Smem {
  static constexpr int kChunks = HD / 64;                  // 128-byte column chunks per row
  static constexpr int kTileBytes = kBlock * HD * 2;        // one K (or V) block of one kv head
  static constexpr int kStageBytes = 2 * kTileBytes;        // K + V
  static constexpr int kDataBytes = kMaxPart * kStageBytes;
  // merge area (reuses the data area after the main loop): kWarps x 16 rows x HD floats
  static constexpr int kMergeBytes = kWarps * kMaxGroup * HD * 4 + 2 * kWarps * kMaxGroup * 4;
  static_assert(kMergeBytes <= kDataBytes, "merge area must fit in the data area");
  static constexpr int kBarOffset = kDataBytes;
  static constexpr int kTotal = kDataBytes + kMaxPart * 8 + 64 + 1024;  // + align slack
};

struct Params {
  void* out;
  const void* q;
  int64_t out_stride;       // elements between consecutive sequences of out
  int64_t q_stride;         // elements between consecutive sequences of q
  const int32_t* block_tables;
  int64_t bt_stride;        // int32 elements between block-table rows
  const int32_t* row_index; // optional: block-table row of each sequence (nullptr: row = seq)
  const int32_t* context_lens;
  int num_heads, num_kv_heads, group, max_blocks, part_blocks, max_parts;
  int64_t num_blocks;
  float scale_log2;         // log2(e) / sqrt(D)
  // split-K workspace
  float* ws_o;              // [B, NH, max_parts, HD]
  float* ws_ml;             // [B, NH, max_parts, 2]
  int32_t* ws_stop;         // [B, KVH, max_parts]
  int32_t* ws_count;        // [B, KVH]
};

template <typename T, int HD>
__global__ void __launch_bounds__(kThreads)
decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
              Params p) {
  using S = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ int s_phys[kMaxPart];
  __shared__ int s_nvalid, s_stop, s_last;

  const int part = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int ctx = p.context_lens[seq];
  if (ctx <= 0) return;                                        // attention.cu:62
  int nblk = (ctx + kBlock - 1) / kBlock;
  nblk = min(nblk, p.max_blocks);
  const int nparts = (nblk + p.part_blocks - 1) / p.part_blocks;
  if (part >= nparts) return;
  const int b0 = part * p.part_blocks;
  const int nb = min(p.part_blocks, nblk - b0);
  const int row = p.row_index ? p.row_index[seq] : seq;
  const int32_t* bt = p.block_tables + (int64_t)row * p.bt_stride;
  const uint32_t bar0 = smem_u32(smem + S::kBarOffset);

  // ---- block-table entries of this partition; stop at the first negative (attention.cu:90)
  if (warp == 0) {
    int phys = (lane < nb) ? bt[b0 + lane] : 0;
    bool bad = (lane < nb) && (phys < 0 || (int64_t)phys >= p.num_blocks);
    // out-of-range ids are treated like an unassigned entry: the reference would read outside
    // the pool there; this kernel never does.
    unsigned neg = __ballot_sync(0xffffffffu, bad);
    int nvalid = neg ? (__ffs(neg) - 1) : nb;
    if (lane < kMaxPart) s_phys[lane] = phys;
    __syncwarp();
    if (lane == 0) {
      s_nvalid = nvalid;
      s_stop = neg ? 1 : 0;
      for (int i = 0; i < nvalid; ++i) mbar_init(bar0 + 8 * i, 1);
      fence_mbar_init();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const uint64_t pol = l2_policy_evict_first();
      for (int i = 0; i < nvalid; ++i) {
        const int pb = s_phys[i];
        const uint32_t bar = bar0 + 8 * i;
        const uint32_t dst = smem_u32(smem + i * S::kStageBytes);
        mbar_arrive_expect_tx(bar, S::kStageBytes);
        const int y = (pb * p.num_kv_heads + kvh) * kBlock;
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c) {
          tma_load_2d_hint(dst + c * kBlock * 128, &kmap, bar, c * 64, y, pol);
          tma_load_2d_hint(dst + S::kTileBytes + c * kBlock * 128, &vmap, bar, c * 64, y, pol);
        }
      }
    }
  }
  __syncthreads();
  const int nvalid = s_nvalid;

  // ---- query fragments (A operand, rows = query heads of this group, zero-padded to 16)
  const int g = lane >> 2, t4 = lane & 3;
  const T* qbase = reinterpret_cast<const T*>(p.q) + (int64_t)seq * p.q_stride +
                   (int64_t)kvh * p.group * HD;
  uint32_t qa[HD / 16][4];
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int rowh = g + ((r & 1) ? 8 : 0);
      const int col = ks * 16 + 2 * t4 + ((r & 2) ? 8 : 0);
      uint32_t v = 0;
      if (rowh < p.group) v = *reinterpret_cast<const uint32_t*>(qbase + rowh * HD + col);
      qa[ks][r] = v;
    }
  }

  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (int j = warp; j < nvalid; j += kWarps) {
    uint8_t* kt = smem + j * S::kStageBytes;
    uint8_t* vt = kt + S::kTileBytes;
    mbar_wait(bar0 + 8 * j, 0, TI_DEVERR_ATTN_WAIT);
    const int tok0 = (b0 + j) * kBlock;
    const int valid = min(kBlock, ctx - tok0);
    if (valid < kBlock) {
      // zero the V rows past the context so that 0 * (stale value) cannot produce NaN
      for (int i = lane; i < (kBlock - valid) * S::kChunks * 8; i += 32) {
        const int r = valid + i / (S::kChunks * 8);
        const int ch = i % (S::kChunks * 8);
        *reinterpret_cast<uint4*>(vt + (ch >> 3) * kBlock * 128 + swz128(r, ch & 7)) =
            make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    // S = Q K^T  (16 heads x 16 tokens)
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const uint32_t kb = smem_u32(kt);
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const int mi = lane >> 3;
      const int tok = ((mi & 2) ? 8 : 0) + (lane & 7);
      const int chunk = ks * 2 + (mi & 1);
      const uint32_t addr = kb + (chunk >> 3) * kBlock * 128 + swz128(tok, chunk & 7);
      uint32_t b0r, b1r, b2r, b3r;
      ldsm_x4(addr, b0r, b1r, b2r, b3r);
      Mma<T>::run(s[0], qa[ks], b0r, b1r);
      Mma<T>::run(s[1], qa[ks], b2r, b3r);
    }
    // scale, mask, online softmax (rows g and g+8)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tk = nt * 8 + 2 * t4 + (e & 1);
        s[nt][e] = (tk < valid) ? s[nt][e] * p.scale_log2 : -INFINITY;
      }
    float mx[2];
    mx[0] = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    mx[1] = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float mn = fmaxf(m_r[h], mx[h]);
      alpha[h] = fast_exp2(m_r[h] - mn);
      m_r[h] = mn;
    }
    float pr[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) pr[nt][e] = fast_exp2(s[nt][e] - m_r[e >> 1]);
    l_r[0] = l_r[0] * alpha[0] + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    l_r[1] = l_r[1] * alpha[1] + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0]; o[i][1] *= alpha[0];
      o[i][2] *= alpha[1]; o[i][3] *= alpha[1];
    }
    uint32_t pa[4], pl[4];
    split_p<T>(pr, pa, pl);
    // O += P V  (16 heads x HD)
    const uint32_t vb = smem_u32(vt);
#pragma unroll
    for (int nt = 0; nt < HD / 8; nt += 2) {
      const int mi = lane >> 3;
      const int tok = ((mi & 1) ? 8 : 0) + (lane & 7);
      const int chunk = nt + (mi >> 1);
      const uint32_t addr = vb + (chunk >> 3) * kBlock * 128 + swz128(tok, chunk & 7);
      uint32_t b0r, b1r, b2r, b3r;
      ldsm_x4_t(addr, b0r, b1r, b2r, b3r);
      Mma<T>::run(o[nt], pa, b0r, b1r);
      Mma<T>::run(o[nt + 1], pa, b2r, b3r);
      if constexpr (kSplitP<T>) {
        Mma<T>::run(o[nt], pl, b0r, b1r);
        Mma<T>::run(o[nt + 1], pl, b2r, b3r);
      }
    }
  }
  // full row sums across the 4 lanes that share a row
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
    l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
  }
  __syncthreads();  // all warps done with the KV tiles: reuse the data area for the merge

  float* wo = reinterpret_cast<float*>(smem);                    // [kWarps][16][HD]
  float* wm = wo + kWarps * kMaxGroup * HD;                      // [kWarps][16]
  float* wl = wm + kWarps * kMaxGroup;                           // [kWarps][16]
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int col = i * 8 + 2 * t4;
    wo[(warp * kMaxGroup + g) * HD + col] = o[i][0];
    wo[(warp * kMaxGroup + g) * HD + col + 1] = o[i][1];
    wo[(warp * kMaxGroup + g + 8) * HD + col] = o[i][2];
    wo[(warp * kMaxGroup + g + 8) * HD + col + 1] = o[i][3];
  }
  if (t4 == 0) {
    wm[warp * kMaxGroup + g] = m_r[0];
    wm[warp * kMaxGroup + g + 8] = m_r[1];
    wl[warp * kMaxGroup + g] = l_r[0];
    wl[warp * kMaxGroup + g + 8] = l_r[1];
  }
  __syncthreads();

  const int G = p.group;
  const int h0 = kvh * G;
  T* outp = reinterpret_cast<T*>(p.out) + (int64_t)seq * p.out_stride;
  if (nparts == 1) {
    for (int i = tid; i < G * HD; i += kThreads) {
      const int r = i / HD, d = i % HD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w * kMaxGroup + r]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float f = (wm[w * kMaxGroup + r] == -INFINITY) ? 0.f : fast_exp2(wm[w * kMaxGroup + r] - M);
        L += wl[w * kMaxGroup + r] * f;
        O += wo[(w * kMaxGroup + r) * HD + d] * f;
      }
      outp[(h0 + r) * HD + d] = Elem<T>::from_f(O / L);   // L == 0 -> NaN (attention.cu:150)
    }
    return;
  }

  // ---- split-K: publish this partition's (m, l, o), last arriver merges
  for (int i = tid; i < G * HD; i += kThreads) {
    const int r = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w * kMaxGroup + r]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = (wm[w * kMaxGroup + r] == -INFINITY) ? 0.f : fast_exp2(wm[w * kMaxGroup + r] - M);
      L += wl[w * kMaxGroup + r] * f;
      O += wo[(w * kMaxGroup + r) * HD + d] * f;
    }
    const int64_t slot = ((int64_t)seq * p.num_heads + h0 + r) * p.max_parts + part;
    p.ws_o[slot * HD + d] = O;
    if (d == 0) {
      p.ws_ml[slot * 2 + 0] = M;
      p.ws_ml[slot * 2 + 1] = L;
    }
  }
  if (tid == 0)
    p.ws_stop[((int64_t)seq * p.num_kv_heads + kvh) * p.max_parts + part] = s_stop;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&p.ws_count[seq * p.num_kv_heads + kvh], 1);
    s_last = (prev == nparts - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // partitions after the first one that met a negative entry are ignored (attention.cu:90)
  const int32_t* stops = p.ws_stop + ((int64_t)seq * p.num_kv_heads + kvh) * p.max_parts;
  int use = nparts;
  for (int q = 0; q < nparts; ++q)
    if (__ldcg(stops + q)) { use = q + 1; break; }
  for (int i = tid; i < G * HD; i += kThreads) {
    const int r = i / HD, d = i % HD;
    const int64_t base = ((int64_t)seq * p.num_heads + h0 + r) * p.max_parts;
    float M = -INFINITY;
    for (int q = 0; q < use; ++q) M = fmaxf(M, __ldcg(p.ws_ml + (base + q) * 2));
    float L = 0.f, O = 0.f;
    for (int q = 0; q < use; ++q) {
      const float mq = __ldcg(p.ws_ml + (base + q) * 2);
      const float f = (mq == -INFINITY) ? 0.f : fast_exp2(mq - M);
      L += __ldcg(p.ws_ml + (base + q) * 2 + 1) * f;
      O += __ldcg(p.ws_o + (base + q) * HD + d) * f;
    }
    outp[(h0 + r) * HD + d] = Elem<T>::from_f(O / L);
  }
  if (tid == 0) p.ws_count[seq * p.num_kv_heads + kvh] = 0;   // ready for the next launch
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------
struct MapKey {
  const void* ptr;
  int64_t rows;
  int hd, dtype;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && hd == o.hd && dtype == o.dtype;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) * 31u) ^
           (size_t)(k.hd * 7 + k.dtype);
  }
};

// Tensor map over one layer's pool viewed as a 2-D [rows = NB*KVH*16, HD] matrix, box 64 x 16,
// SWIZZLE_128B.  Cached per (pointer, rows, HD, dtype).
static int kv_tensor_map(CUtensorMap* out, const void* base, int64_t rows, int hd, int dtype) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{base, rows, hd, dtype};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) { *out = it->second; return TI_OK; }
  }
  cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)kBlock};
  cuuint32_t estr[2] = {1, 1};
  int rc = encode_tensor_map_2d(out,
                                dtype == TI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc != TI_OK) return rc;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return TI_OK;
}

template <typename T, int HD>
static int launch(const Params& p, const CUtensorMap& km, const CUtensorMap& vm, int batch,
                  cudaStream_t stream) {
  using S = Smem<HD>;
  static bool attr_set = false;   // per instantiation; set on first use on every device
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set || attr_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel<T, HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(paged attention)");
    attr_set = true;
    attr_dev = dev;
  }
  dim3 grid(p.max_parts, p.num_kv_heads, batch);
  decode_kernel<T, HD><<<grid, kThreads, S::kTotal, stream>>>(km, vm, p);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "paged attention launch");
  return TI_OK;
}

}  // namespace attn
}  // namespace ti

using namespace ti;

extern "C" size_t ti_paged_attention_workspace_bytes(int batch, int num_heads, int num_kv_heads,
                                                      int head_dim, int max_blocks_per_seq,
                                                      int partition_blocks) {
  if (partition_blocks <= 0) partition_blocks = attn::kMaxPart;
  const int64_t parts = (max_blocks_per_seq + partition_blocks - 1) / partition_blocks;
  const int64_t slots = (int64_t)batch * num_heads * parts;
  size_t bytes = attn::kCounterBytes;                           // arrival counters (kept zero)
  bytes += (size_t)slots * head_dim * 4;                        // ws_o
  bytes += (size_t)slots * 2 * 4;                               // ws_ml
  bytes += (size_t)batch * num_kv_heads * parts * 4;            // ws_stop
  return bytes + 256;
}

extern "C" int ti_paged_attention_decode(
    void* out, int64_t out_seq_stride, const void* q, int64_t q_seq_stride, const void* k_cache,
    const void* v_cache, int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
    const int32_t* row_index, const int32_t* context_lens, int batch, int num_heads,
    int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq, int dtype,
    int partition_blocks, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (batch == 0) return TI_OK;
  if (!out || !q || !k_cache || !v_cache || !block_tables || !context_lens)
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: null pointer");
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: num_heads must be a positive multiple of num_kv_heads");
  if (num_heads / num_kv_heads > attn::kMaxGroup)
    return set_error(TI_ERR_UNSUPPORTED, "paged attention: at most 16 query heads per kv head");
  if (head_dim != 64 && head_dim != 128)
    return set_error(TI_ERR_UNSUPPORTED, "paged attention: head_dim must be 64 or 128");
  if (block_size != attn::kBlock)
    return set_error(TI_ERR_UNSUPPORTED, "paged attention: block_size must be 16");
  if (dtype != TI_DTYPE_BF16 && dtype != TI_DTYPE_FP16)
    return set_error(TI_ERR_UNSUPPORTED, "paged attention: dtype must be bf16 or fp16");
  if (max_blocks_per_seq <= 0 || num_blocks <= 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: empty pool or block table");
  if (partition_blocks <= 0) partition_blocks = attn::kMaxPart;
  if (partition_blocks > attn::kMaxPart)
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: partition_blocks must be <= 16");
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: pool base must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (q_seq_stride & 1))
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: q must be 4-byte aligned with an even row stride");
  const int max_parts = (max_blocks_per_seq + partition_blocks - 1) / partition_blocks;
  const size_t need = ti_paged_attention_workspace_bytes(batch, num_heads, num_kv_heads, head_dim,
                                                          max_blocks_per_seq, partition_blocks);
  if (max_parts > 1 && (!workspace || workspace_bytes < need))
    return set_error(TI_ERR_WORKSPACE, "paged attention: workspace too small");
  if (max_parts > 1 && (int64_t)batch * num_kv_heads > attn::kMaxCounters)
    return set_error(TI_ERR_UNSUPPORTED, "paged attention: batch * num_kv_heads must be <= 16384");
  if (max_parts > 65535 || batch > 65535)
    return set_error(TI_ERR_UNSUPPORTED, "paged attention: grid too large");

  attn::Params p{};
  p.out = out; p.q = q; p.out_stride = out_seq_stride; p.q_stride = q_seq_stride;
  p.block_tables = block_tables; p.bt_stride = bt_stride; p.row_index = row_index;
  p.context_lens = context_lens;
  p.num_heads = num_heads; p.num_kv_heads = num_kv_heads; p.group = num_heads / num_kv_heads;
  p.max_blocks = max_blocks_per_seq; p.part_blocks = partition_blocks; p.max_parts = max_parts;
  p.num_blocks = num_blocks;
  p.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  if (max_parts > 1) {
    const int64_t slots = (int64_t)batch * num_heads * max_parts;
    uint8_t* w = reinterpret_cast<uint8_t*>(workspace);
    p.ws_count = reinterpret_cast<int32_t*>(w); w += attn::kCounterBytes;
    p.ws_o = reinterpret_cast<float*>(w); w += slots * head_dim * 4;
    p.ws_ml = reinterpret_cast<float*>(w); w += slots * 2 * 4;
    p.ws_stop = reinterpret_cast<int32_t*>(w);
  }
  const int64_t rows = num_blocks * num_kv_heads * attn::kBlock;
  CUtensorMap km, vm;
  int rc = attn::kv_tensor_map(&km, k_cache, rows, head_dim, dtype);
  if (rc) return rc;
  rc = attn::kv_tensor_map(&vm, v_cache, rows, head_dim, dtype);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16)
    return head_dim == 64 ? attn::launch<__nv_bfloat16, 64>(p, km, vm, batch, s)
                          : attn::launch<__nv_bfloat16, 128>(p, km, vm, batch, s);
  return head_dim == 64 ? attn::launch<__half, 64>(p, km, vm, batch, s)
                        : attn::launch<__half, 128>(p, km, vm, batch, s);
}
