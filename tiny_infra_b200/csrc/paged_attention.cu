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
#include <cstdlib>
#include <cstring>
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
  int32_t* ws_pieces;       // [B, KVH] v4: pieces of each unit (written by its first piece)
  const int32_t* plan;      // v5: the batch's stream resolved once (ti_paged_attention_plan)
  int early;                // v5 planned: plan and all but each unit's last block are final
                            // before the previous kernel (TI_ATTN_EARLY_KV)
  // v5 plan for a call behind another kernel (TI_ATTN_PLAN_AFTER_QKV): CTAs skew_full.. start
  // about skew_lead_us later (their SMs are held by that kernel) and take fewer streams
  int skew_full;
  float skew_lead_us;
};

// SM count of the current device (the persistent kernels' grid), cached per device.
static int sm_count() {
  static int cached_dev = -1, sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0)
      sms = 148;
    cached_dev = dev;
  }
  return sms;
}

template <typename T, int HD>
__global__ void __launch_bounds__(kThreads)
decode_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
              Params p) {
  pdl_wait();
  pdl_launch_dependents();
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
  int hd, dtype, box_rows;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && hd == o.hd && dtype == o.dtype &&
           box_rows == o.box_rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) * 31u) ^
           (size_t)(k.hd * 7 + k.dtype + k.box_rows * 131);
  }
};

// Tensor map over one layer's pool viewed as a 2-D [rows = NB*KVH*16, HD] matrix, box 64 x 16,
// SWIZZLE_128B.  Cached per (pointer, rows, HD, dtype).
static int kv_tensor_map(CUtensorMap* out, const void* base, int64_t rows, int hd, int dtype,
                         int box_rows = kBlock) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{base, rows, hd, dtype, box_rows};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) { *out = it->second; return TI_OK; }
  }
  cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
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
  return launch_kernel("paged attention launch", decode_kernel<T, HD>, grid, dim3(kThreads),
                       S::kTotal, stream, 1, km, vm, p);
}


// ==========================================================================================
// v2: persistent, load-balanced streaming kernel (head_dim 64, batch <= 4096)
//
// Work unit: one sequence and HP consecutive kv heads.  With HP = 2 (GQA groups of <= 8 query
// heads, an even number of kv heads) the 16 MMA rows hold the query heads of both kv heads --
// rows 0..G-1 for the first, 8..8+G-1 for the second -- so no MMA row is padding for
// Qwen2.5-0.5B's 7-head groups, and one 32-row TMA box fetches both heads' K (4 KB contiguous)
// and one fetches their V.  HP = 1 is the general layout (16 rows, G <= 16).
//
// All KV blocks of all units form one stream (unit-major, blocks in logical order); every warp
// of the grid gets an equal contiguous chunk of it.  A chunk covers a few "pieces" (the part
// of one unit inside the chunk); a unit cut by chunk boundaries is split-K merged by the last
// of its pieces to finish (atomic arrival counter, no waiting), other units write their output
// directly.  Each CTA rebuilds the block offsets with a prefix scan over sequences.
//
// Per warp: a STAGES-deep TMA ring that lane 0 keeps full across piece boundaries while the
// warp computes, piece metadata in a 4-entry ring and a 32-entry window of block ids.
// ==========================================================================================
constexpr int kV2Meta = 4;
constexpr int kV2MaxBatch = 4096;
constexpr int kV2MaxPieces = 17;                           // pieces per unit (bounded by the chunk)
// Small decode batches (the v5 kernel): units may be cut into up to this many pieces, so that a
// few sequences still spread over every SM (the merge reads their partials in rounds of 16).
constexpr int kV5MaxPiecesSmall = 65;
// Stream positions of one v5 CTA held in shared memory (pool row and valid tokens of each):
// 4096 cover 256 sequences of up to 32k tokens (the long-context replica workload).
constexpr int kV5IdCap = 4096;
constexpr int kV5SmallBatch = 64;

struct PieceV2 {
  int row, unit, j0, len, ctx, piece, pieces;
  int nvalid;      // blocks to read (len until a negative entry is met)
  int issued;      // blocks issued so far
  int scanned;     // issue cursor is done with this piece (nvalid final)
  int stop;        // met a negative entry
};

template <int HP>
struct CfgV2 {
  static constexpr int kWarps = HP == 2 ? 12 : 6;
  static constexpr int kStages = HP == 2 ? 2 : 8;
  static constexpr int kTile = HP * kBlock * 64 * 2;          // K (or V) of one block, HP heads
  static constexpr int kStage = 2 * kTile;
  static constexpr int kRing = kWarps * kStages * kStage;     // 192 KB
  static constexpr int kBars = kWarps * kStages * 8;
  static constexpr int kMeta = kWarps * kV2Meta * (int)sizeof(PieceV2);
  static constexpr int kWin = kWarps * 32 * 4;
  static constexpr int kOffBytes = (kV2MaxBatch + 1) * 4;
  static constexpr int kTotal = kRing + kBars + kMeta + kWin + kOffBytes + 1024;
  static_assert(kTotal <= 227 * 1024, "v2 shared memory");
};

// chunk of the block stream per warp: balanced, but at least max_blocks / (max_parts - 1) (so
// that a unit is cut into at most max_parts pieces, which bounds the split-K workspace) and at
// least 2 (small batches: 8 sequences of up to 512 tokens take 9.7 us with 2, 11.2 us with 4,
// measured)
__host__ __device__ inline int v2_chunk(int64_t total_blocks, int warps, int max_blocks,
                                        int max_parts) {
  int64_t c = (total_blocks + warps - 1) / warps;
  const int lo = max(2, (max_blocks + max_parts - 2) / (max_parts - 1));
  return (int)(c < lo ? lo : c);
}

// One KV block (16 tokens) of the unit's HP kv heads: S = QK^T, online softmax, O += PV for the
// 16-row tile.  kb / vb: shared addresses of the SWIZZLE_128B K and V tiles (HP * 16 rows).
template <typename T, int HP>
__device__ __forceinline__ void v2_block(uint32_t kb, uint32_t vb, uint8_t* vt, int valid,
                                         int lane, const uint32_t (&qa)[4][4], float scale_log2,
                                         float (&m_r)[2], float (&l_r)[2], float (&o)[8][4]) {
  const int t4 = lane & 3;
  if (valid < kBlock) {
    // zero the V rows past the context so that 0 * (stale value) cannot produce NaN
    for (int i = lane; i < HP * (kBlock - valid) * 8; i += 32) {
      const int h = i / ((kBlock - valid) * 8), r = i % ((kBlock - valid) * 8);
      *reinterpret_cast<uint4*>(vt + swz128(h * kBlock + valid + r / 8, r & 7)) =
          make_uint4(0, 0, 0, 0);
    }
    __syncwarp();
  }
  // scores: rows g from kv sub-head 0, rows g+8 from kv sub-head HP-1
  float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  float sd[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int mi = lane >> 3;
    const int tok = ((mi & 2) ? 8 : 0) + (lane & 7);
    uint32_t b0, b1, b2, b3;
    ldsm_x4(kb + swz128(tok, ks * 2 + (mi & 1)), b0, b1, b2, b3);
    Mma<T>::run(sc[0], qa[ks], b0, b1);
    Mma<T>::run(sc[1], qa[ks], b2, b3);
    if constexpr (HP == 2) {
      ldsm_x4(kb + swz128(kBlock + tok, ks * 2 + (mi & 1)), b0, b1, b2, b3);
      Mma<T>::run(sd[0], qa[ks], b0, b1);
      Mma<T>::run(sd[1], qa[ks], b2, b3);
    }
  }
  if constexpr (HP == 2) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][2] = sd[nt][2];
      sc[nt][3] = sd[nt][3];
    }
  }
  if (valid < kBlock) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tk = nt * 8 + 2 * t4 + (e & 1);
        sc[nt][e] = (tk < valid) ? sc[nt][e] * scale_log2 : -INFINITY;
      }
  } else {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] *= scale_log2;
  }
  float mx[2];
  mx[0] = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
  mx[1] = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
  }
  float alpha[2];
  bool moved = false;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float mn = fmaxf(m_r[h], mx[h]);
    moved |= mn != m_r[h];
    alpha[h] = fast_exp2(m_r[h] - mn);
    m_r[h] = mn;
  }
  float pr[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[nt][e] = fast_exp2(sc[nt][e] - m_r[e >> 1]);
  l_r[0] = l_r[0] * alpha[0] + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
  l_r[1] = l_r[1] * alpha[1] + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
  if (__any_sync(0xffffffffu, moved)) {       // rescale only when some row's max moved
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= alpha[0]; o[i][1] *= alpha[0];
      o[i][2] *= alpha[1]; o[i][3] *= alpha[1];
    }
  }
  uint32_t pa[4], pl[4];
  split_p<T>(pr, pa, pl);
  // A fragments: registers 0/2 hold rows g, 1/3 rows g+8.  With HP == 2 rows g multiply the
  // first kv head's V and rows g+8 the second's, so each product uses half of the fragment.
  const uint32_t mask_lo[4] = {0xffffffffu, 0u, 0xffffffffu, 0u};
#pragma unroll
  for (int sub = 0; sub < HP; ++sub) {
    uint32_t ah[4], al[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t keep = HP == 1 ? 0xffffffffu : (sub == 0 ? mask_lo[i] : ~mask_lo[i]);
      ah[i] = pa[i] & keep;
      al[i] = pl[i] & keep;
    }
#pragma unroll
    for (int nt = 0; nt < 8; nt += 2) {
      const int mi = lane >> 3;
      const int tok = sub * kBlock + ((mi & 1) ? 8 : 0) + (lane & 7);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vb + swz128(tok, nt + (mi >> 1)), b0, b1, b2, b3);
      Mma<T>::run(o[nt], ah, b0, b1);
      Mma<T>::run(o[nt + 1], ah, b2, b3);
      if constexpr (kSplitP<T>) {
        Mma<T>::run(o[nt], al, b0, b1);
        Mma<T>::run(o[nt + 1], al, b2, b3);
      }
    }
  }
}

// Query heads of the 16 MMA rows: row r < 8 -> first kv head of the unit, r >= 8 -> the last
// (HP == 2), or r -> r (HP == 1).  Returns -1 for a padding row.
template <int HP>
__device__ __forceinline__ int v2_row_head(int unit, int r, int G) {
  if constexpr (HP == 2) {
    const int sub = r >> 3, i = r & 7;
    return i < G ? (unit * 2 + sub) * G + i : -1;
  } else {
    return r < G ? unit * G + r : -1;
  }
}

// Merge the published pieces of one unit and write its nheads (<= 16) output rows.  Lane l
// owns head l/2, dims 32*(l%2) .. +31; every load of a lane is independent of the others, so
// the merge costs a few memory round trips instead of one per head.
template <typename T>
__device__ __forceinline__ void v2_merge(const Params& p, int row, int unit, int nheads,
                                         int pieces, int lane, T* outp) {
  const int h0 = unit * nheads;
  const int units = p.num_heads / nheads;
  const int64_t pair = (int64_t)row * units + unit;
  const int32_t* stops = p.ws_stop + pair * p.max_parts;
  int use = pieces;
  {
    const int st = lane < pieces ? __ldcg(stops + lane) : 0;   // pieces <= 17 < 32
    const unsigned b = __ballot_sync(0xffffffffu, st != 0);
    if (b) use = __ffs(b);                                     // up to and including the first stop
  }
  for (int hb = 0; hb < nheads; hb += 16) {
    const int h = hb + (lane >> 1), half = lane & 1;
    const bool live = h < nheads;
    const int64_t base = ((int64_t)row * p.num_heads + h0 + (live ? h : 0)) * p.max_parts;
    float mq[kV2MaxPieces], lq[kV2MaxPieces];
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < kV2MaxPieces; ++q) {
      if (q < use && live) {
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.ws_ml) + base + q);
        mq[q] = ml.x;
        lq[q] = ml.y;
      } else {
        mq[q] = -INFINITY;
        lq[q] = 0.f;
      }
      M = fmaxf(M, mq[q]);
    }
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.f;
    float L = 0.f;
    float f[kV2MaxPieces];
#pragma unroll
    for (int q = 0; q < kV2MaxPieces; ++q) {
      f[q] = (q < use && live && mq[q] != -INFINITY) ? fast_exp2(mq[q] - M) : 0.f;
      L += lq[q] * f[q];
    }
    // two pieces per round: their 16 loads are in flight together (the merge sits on the
    // kernel's critical tail, so its L2 round trips are what it costs)
#pragma unroll
    for (int q = 0; q < kV2MaxPieces; q += 2) {
      if (q < use) {
        const bool two = q + 1 < use && q + 1 < kV2MaxPieces;
        float4 va[8], vb[8];
        const float4* s0 = reinterpret_cast<const float4*>(p.ws_o + (base + q) * 64 + half * 32);
        const float4* s1 = s0 + 16;   // the next piece's slot of this head (64 floats later)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          va[i] = live ? __ldcg(s0 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          vb[i] = (live && two) ? __ldcg(s1 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float f0 = f[q], f1 = two ? f[q + 1 < kV2MaxPieces ? q + 1 : q] : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc[4 * i] += f0 * va[i].x + f1 * vb[i].x;
          acc[4 * i + 1] += f0 * va[i].y + f1 * vb[i].y;
          acc[4 * i + 2] += f0 * va[i].z + f1 * vb[i].z;
          acc[4 * i + 3] += f0 * va[i].w + f1 * vb[i].w;
        }
      }
    }
    if (live) {
      const float inv = 1.f / L;                               // L == 0 -> NaN (attention.cu:150)
      T* dst = outp + (int64_t)(h0 + h) * 64 + half * 32;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 u;
        u.x = Elem<T>::pack2(acc[i] * inv, acc[i + 1] * inv);
        u.y = Elem<T>::pack2(acc[i + 2] * inv, acc[i + 3] * inv);
        u.z = Elem<T>::pack2(acc[i + 4] * inv, acc[i + 5] * inv);
        u.w = Elem<T>::pack2(acc[i + 6] * inv, acc[i + 7] * inv);
        *reinterpret_cast<uint4*>(dst + i) = u;
      }
    }
  }
}

// Split-K arrival: every lane's partial-result stores are ordered before lane 0's acq_rel
// increment (warp barrier + cumulative release); the last arriver acquires the others'.
__device__ __forceinline__ bool arrive_last(int32_t* counter, int expected, int lane) {
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    int prev;
    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
    last = prev == expected - 1;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  __syncwarp();
  return last != 0;
}

template <typename T, int HP>
__global__ void __launch_bounds__(CfgV2<HP>::kWarps * 32, 1)
decode_kernel_v2(const __grid_constant__ CUtensorMap kmap,
                 const __grid_constant__ CUtensorMap vmap, Params p, int batch) {
  pdl_wait();
  pdl_launch_dependents();
  using C = CfgV2<HP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t bar_all = smem_u32(smem + C::kRing);
  PieceV2* meta_all = reinterpret_cast<PieceV2*>(smem + C::kRing + C::kBars);
  int* win_all = reinterpret_cast<int*>(smem + C::kRing + C::kBars + C::kMeta);
  int* s_off = win_all + C::kWarps * 32;      // s_off[r] = KVU * blocks of rows before r
  __shared__ int s_wsum[C::kWarps];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KVH = p.num_kv_heads;
  const int KVU = KVH / HP;                   // units per sequence
  auto nblk_of = [&](int r) {
    const int ctx = p.context_lens[r];
    return ctx > 0 ? min((ctx + kBlock - 1) / kBlock, p.max_blocks) : 0;
  };

  // ---- exclusive prefix sum of KVU * blocks per sequence into s_off[0..batch]
  const int per = (batch + blockDim.x - 1) / blockDim.x;
  const int r0 = min(batch, tid * per), r1 = min(batch, r0 + per);
  int local = 0;
  for (int r = r0; r < r1; ++r) local += KVU * nblk_of(r);
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_wsum[warp] = incl;
  if (tid < C::kWarps * C::kStages) {
    mbar_init(bar_all + 8 * tid, 1);
    fence_mbar_init();
  }
  __syncthreads();
  int run = incl - local;
  for (int w = 0; w < warp; ++w) run += s_wsum[w];
  for (int r = r0; r < r1; ++r) {
    s_off[r] = run;
    run += KVU * nblk_of(r);
  }
  if (tid == 0) {
    int tot = 0;
    for (int w = 0; w < C::kWarps; ++w) tot += s_wsum[w];
    s_off[batch] = tot;
  }
  __syncthreads();
  const int total = s_off[batch];
  const int W = gridDim.x * C::kWarps;
  const int chunk = v2_chunk(total, W, p.max_blocks, p.max_parts);
  const int wid = blockIdx.x * C::kWarps + warp;
  const int begin = wid * chunk;
  if (begin >= total) return;
  const int end = min(total, begin + chunk);

  uint8_t* ring = smem + warp * C::kStages * C::kStage;
  const uint32_t bar = bar_all + warp * C::kStages * 8;
  PieceV2* meta = meta_all + warp * kV2Meta;
  int* win = win_all + warp * 32;
  const int G = p.group;
  const int NHU = HP * G;                     // query heads per unit
  const int g = lane >> 2, t4 = lane & 3;
  const uint64_t pol = l2_policy_evict_first();

  uint32_t phase = 0;                 // expected parity of each stage's barrier
  int issued = 0, consumed = 0;       // blocks of this warp
  int ik = 0, ij = 0, started = 0;    // issue cursor: piece, block within piece; pieces started
  int ipos = begin;                   // stream position of piece ik's first block
  int win_lo = 0, win_hi = 0;         // block-id window [win_lo, win_hi) of piece ik (unit-relative)
  bool idone = false;
  int ck = 0, cj = 0;                 // consume cursor
  bool open = false;                  // softmax state belongs to piece ck
  uint32_t qa[4][4];
  float m_r[2], l_r[2], o[8][4];

  while (true) {
    // ---- issue: keep up to kStages blocks in flight, at most kV2Meta pieces ahead
    __syncwarp();
    while (!idone) {
      if (ik == started) {
        if (ik - ck >= kV2Meta) break;
        int lo = 0, hi = batch;                  // largest row with s_off[row] <= ipos
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (s_off[mid] <= ipos) lo = mid; else hi = mid;
        }
        const int row = lo;
        const int nb = (s_off[row + 1] - s_off[row]) / KVU;
        const int rel = ipos - s_off[row];
        const int unit = rel / nb, j0 = rel - unit * nb;
        const int pstart = s_off[row] + unit * nb;
        const int len = min(nb - j0, end - ipos);
        if (lane == 0) {
          PieceV2& m = meta[ik % kV2Meta];
          m.row = row; m.unit = unit; m.j0 = j0; m.len = len; m.ctx = p.context_lens[row];
          m.piece = ipos / chunk - pstart / chunk;
          m.pieces = (pstart + nb - 1) / chunk - pstart / chunk + 1;
          m.nvalid = len; m.issued = 0; m.scanned = 0; m.stop = 0;
        }
        __syncwarp();
        ++started;
        win_lo = win_hi = j0;
      }
      PieceV2& m = meta[ik % kV2Meta];
      if (ij < m.nvalid) {
        if (issued - consumed >= C::kStages) break;
        const int j = m.j0 + ij;
        if (j >= win_hi) {                       // next 32 block ids of this piece
          const int lim = m.j0 + m.len;
          const int brow = p.row_index ? p.row_index[m.row] : m.row;
          const int jj = j + lane;
          const int phys = jj < lim ? p.block_tables[(int64_t)brow * p.bt_stride + jj] : 0;
          const bool bad = jj < lim && (phys < 0 || (int64_t)phys >= p.num_blocks);
          const unsigned neg = __ballot_sync(0xffffffffu, bad);
          win[lane] = phys;
          if (neg && lane == 0) {                // stop at the first negative (attention.cu:90)
            m.nvalid = (j - m.j0) + __ffs(neg) - 1;
            m.stop = 1;
          }
          win_lo = j;
          win_hi = j + 32;
          __syncwarp();
          if (ij >= m.nvalid) continue;
        }
        if (lane == 0) {
          const int st = issued % C::kStages;
          const uint32_t dst = smem_u32(ring + st * C::kStage);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive_expect_tx(bar + 8 * st, C::kStage);
          const int y = (win[j - win_lo] * KVH + m.unit * HP) * kBlock;
          tma_load_2d_hint(dst, &kmap, bar + 8 * st, 0, y, pol);
          tma_load_2d_hint(dst + C::kTile, &vmap, bar + 8 * st, 0, y, pol);
          m.issued = ij + 1;
        }
        __syncwarp();
        ++ij;
        ++issued;
      } else {
        if (lane == 0) m.scanned = 1;
        __syncwarp();
        ipos += m.len;
        ++ik;
        ij = 0;
        if (ipos >= end) idone = true;
      }
    }
    if (ck == started && idone) break;
    const PieceV2& m = meta[ck % kV2Meta];
    if (!open) {                      // start a piece: its query rows, fresh softmax state
      const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)m.row * p.q_stride;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int head = v2_row_head<HP>(m.unit, g + ((r & 1) ? 8 : 0), G);
          const int col = ks * 16 + 2 * t4 + ((r & 2) ? 8 : 0);
          qa[ks][r] = head >= 0 ? *reinterpret_cast<const uint32_t*>(qb + head * 64 + col) : 0u;
        }
      m_r[0] = m_r[1] = -INFINITY;
      l_r[0] = l_r[1] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      open = true;
    }
    if (cj < m.issued) {
      const int st = consumed % C::kStages;
      if (!mbar_wait(bar + 8 * st, (phase >> st) & 1u, TI_DEVERR_ATTN_WAIT)) return;
      phase ^= 1u << st;
      uint8_t* kt = ring + st * C::kStage;
      const int valid = min(kBlock, m.ctx - (m.j0 + cj) * kBlock);
      v2_block<T, HP>(smem_u32(kt), smem_u32(kt + C::kTile), kt + C::kTile, valid, lane, qa,
                      p.scale_log2, m_r, l_r, o);
      ++cj;
      ++consumed;
      continue;
    }
    if (!m.scanned) continue;         // more blocks of this piece still to issue
    // ---- piece finished
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
      l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
    }
    const int row = m.row;
    const int hA = v2_row_head<HP>(m.unit, g, G), hB = v2_row_head<HP>(m.unit, g + 8, G);
    T* outp = reinterpret_cast<T*>(p.out) + (int64_t)row * p.out_stride;
    if (m.pieces == 1) {
      const float inv0 = 1.f / l_r[0], inv1 = 1.f / l_r[1];   // l == 0 -> NaN (attention.cu:150)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int col = i * 8 + 2 * t4;
        if (hA >= 0)
          *reinterpret_cast<uint32_t*>(outp + hA * 64 + col) =
              Elem<T>::pack2(o[i][0] * inv0, o[i][1] * inv0);
        if (hB >= 0)
          *reinterpret_cast<uint32_t*>(outp + hB * 64 + col) =
              Elem<T>::pack2(o[i][2] * inv1, o[i][3] * inv1);
      }
    } else {
      const int64_t rb = (int64_t)row * p.num_heads;
      const int64_t s0 = (rb + (hA >= 0 ? hA : 0)) * p.max_parts + m.piece;
      const int64_t s1 = (rb + (hB >= 0 ? hB : 0)) * p.max_parts + m.piece;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int col = i * 8 + 2 * t4;
        if (hA >= 0) *reinterpret_cast<float2*>(p.ws_o + s0 * 64 + col) = make_float2(o[i][0], o[i][1]);
        if (hB >= 0) *reinterpret_cast<float2*>(p.ws_o + s1 * 64 + col) = make_float2(o[i][2], o[i][3]);
      }
      if (t4 == 0) {
        if (hA >= 0) *reinterpret_cast<float2*>(p.ws_ml + s0 * 2) = make_float2(m_r[0], l_r[0]);
        if (hB >= 0) *reinterpret_cast<float2*>(p.ws_ml + s1 * 2) = make_float2(m_r[1], l_r[1]);
      }
      const int64_t pair = (int64_t)row * KVU + m.unit;
      if (lane == 0) p.ws_stop[pair * p.max_parts + m.piece] = m.stop;
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(&p.ws_count[pair], 1) == m.pieces - 1;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
        v2_merge<T>(p, row, m.unit, NHU, m.pieces, lane, outp);
        if (lane == 0) p.ws_count[pair] = 0;     // ready for the next launch
      }
    }
    open = false;
    ++ck;
    cj = 0;
  }
}

// One KV block of ONE kv head with the tokens as the MMA M dimension and the (<= 8) query heads
// of its GQA group as N: S^T[16 tokens x 8 heads] = K . Q^T (4 MMAs over head_dim 64), online
// softmax per head (column), O^T[64 dims x 8 heads] += V^T . P^T (4 MMAs; with bf16 P split into
// hi + lo, 8).  No padding rows: 7 of the 8 columns carry a query head for Qwen2.5-0.5B.
//   kb / vb   shared addresses of the 16 x 64 K and V tiles (SWIZZLE_128B rows)
//   qb[ks]    B fragments of Q^T for the four 16-wide head_dim steps
//   m, l      running max / sum of heads 2*t4, 2*t4+1 (this lane's two columns)
//   o[mt]     C fragments of O^T for dims 16*mt .. 16*mt+15
template <typename T>
__device__ __forceinline__ void swapped_block(uint32_t kb, uint32_t vb, uint8_t* vt, int valid,
                                              int lane, const uint32_t (&qb)[4][2],
                                              float scale_log2, float (&m)[2], float (&l)[2],
                                              float (&o)[4][4]) {
  const int g = lane >> 2, t4 = lane & 3;
  if (valid < kBlock) {
    // zero the V rows past the context so that 0 * (stale value) cannot produce NaN; the
    // proxy fence orders these generic-proxy writes before the TMA that later refills the
    // stage (the only generic writes to the ring)
    for (int i = lane; i < (kBlock - valid) * 8; i += 32)
      *reinterpret_cast<uint4*>(vt + swz128(valid + i / 8, i & 7)) = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
  }
  // ---- S^T = K Q^T : rows = tokens g, g+8; columns = heads 2t4, 2t4+1
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const int mi = lane >> 3;
    const int tok = ((mi & 1) ? 8 : 0) + (lane & 7);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t a[4];
      ldsm_x4(kb + swz128(tok, ks * 2 + (mi >> 1)), a[0], a[1], a[2], a[3]);
      Mma<T>::run(s, a, qb[ks][0], qb[ks][1]);
    }
  }
  if (valid < kBlock) {
    s[0] = g < valid ? s[0] * scale_log2 : -INFINITY;
    s[1] = g < valid ? s[1] * scale_log2 : -INFINITY;
    s[2] = g + 8 < valid ? s[2] * scale_log2 : -INFINITY;
    s[3] = g + 8 < valid ? s[3] * scale_log2 : -INFINITY;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) s[e] *= scale_log2;
  }
  // ---- online softmax per column (head): reduce over the 16 tokens = lanes sharing t4
  float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
  const bool moved = (mn0 != m[0]) | (mn1 != m[1]);
  const float al0 = fast_exp2(m[0] - mn0), al1 = fast_exp2(m[1] - mn1);
  m[0] = mn0;
  m[1] = mn1;
  const float p0 = fast_exp2(s[0] - mn0), p1 = fast_exp2(s[1] - mn1);
  const float p2 = fast_exp2(s[2] - mn0), p3 = fast_exp2(s[3] - mn1);
  l[0] = l[0] * al0 + p0 + p2;           // per-lane partial over its tokens; reduced at the end
  l[1] = l[1] * al1 + p1 + p3;
  if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      o[mt][0] *= al0; o[mt][1] *= al1;
      o[mt][2] *= al0; o[mt][3] *= al1;
    }
  }
  // ---- P^T from C layout (token rows, head columns) to the B layout of V^T P^T:
  // lane (g, t4) needs P^T[2t4][g], P^T[2t4+1][g] (b0) and P^T[2t4+8][g], P^T[2t4+9][g] (b1),
  // held by lanes 8t4 + g/2 and 8t4 + 4 + g/2, in the half of their word chosen by g % 2.
  const uint32_t x01 = Elem<T>::pack2(p0, p1), x23 = Elem<T>::pack2(p2, p3);
  const int src0 = 8 * t4 + (g >> 1), src1 = src0 + 4;
  const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
  uint32_t bh[2], bl[2] = {0u, 0u};
  bh[0] = __byte_perm(__shfl_sync(0xffffffffu, x01, src0), __shfl_sync(0xffffffffu, x01, src1), sel);
  bh[1] = __byte_perm(__shfl_sync(0xffffffffu, x23, src0), __shfl_sync(0xffffffffu, x23, src1), sel);
  if constexpr (kSplitP<T>) {
    const float2 h01 = Elem<T>::unpack2(x01), h23 = Elem<T>::unpack2(x23);
    const uint32_t y01 = Elem<T>::pack2(p0 - h01.x, p1 - h01.y);
    const uint32_t y23 = Elem<T>::pack2(p2 - h23.x, p3 - h23.y);
    bl[0] = __byte_perm(__shfl_sync(0xffffffffu, y01, src0), __shfl_sync(0xffffffffu, y01, src1), sel);
    bl[1] = __byte_perm(__shfl_sync(0xffffffffu, y23, src0), __shfl_sync(0xffffffffu, y23, src1), sel);
  }
  // ---- O^T += V^T P^T : A = V^T (rows = dims, k = tokens) via ldmatrix.trans of the V tile
  {
    const int mi = lane >> 3;
    const int tok = ((mi >> 1) ? 8 : 0) + (lane & 7);
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      uint32_t a[4];
      ldsm_x4_t(vb + swz128(tok, mt * 2 + (mi & 1)), a[0], a[1], a[2], a[3]);
      Mma<T>::run(o[mt], a, bh[0], bh[1]);
      if constexpr (kSplitP<T>) Mma<T>::run(o[mt], a, bl[0], bl[1]);
    }
  }
}

// ==========================================================================================
// v4: persistent, load-balanced, self-issuing kernel (head_dim 64, GQA groups <= 8)
//
// The whole batch's KV blocks form one stream (per sequence, per unit of HP kv heads); every
// warp gets an equal contiguous chunk; a unit cut by chunk boundaries is split-K merged by the
// last of its pieces to finish.  In the prologue each CTA resolves its range of the stream to
// TMA row coordinates and valid-token counts in shared memory, so the main loop does no global
// metadata loads.  Each warp then streams its own chunk through a kV4Stages-deep ring (lane 0
// issues the next TMA as soon as a stage is consumed -- issue cost is spread over all warps)
// and computes each KV block with tokens as the MMA M dimension and the group's query heads as
// N (swapped_block).
// ==========================================================================================
constexpr int kV4Warps = 12;
constexpr int kV4Stages = 2;
constexpr int kV4IdCap = 2048;

// Stream prologue of the v4 / v5 kernels (all NT threads of the CTA call it).
//  * s_off[r] = first stream position of sequence r (KVU units of its blocks, unit-major),
//    s_off[batch] = total;
//  * chunk = stream positions per consumer (`streams` consumers per CTA); this CTA's range is
//    [cb, ce), resolved into ids[] (TMA row coordinate of the unit's first kv head, -1 for a
//    negative or out-of-pool block-table entry) and vtok[] (valid tokens of the block).
// Returns false (uniformly) when the CTA has no positions.  The leading __syncthreads also
// publishes barrier initialisation done by the caller before the call.
// Skewed split for a call behind another kernel: CTAs 0 .. skew_full-1 start on the SMs that
// kernel leaves free, the others only when it ends, about skew_lead_us later.  The late CTAs
// then take nl < streams chunks (their last streams stay idle) so that both groups end
// together: nl = streams * (1 - lead / expected loop time), the loop time estimated from the
// stream's KV bytes at the HBM rate (kSkewUsPerPos per position), in [5/8, 1] of streams, and
// only while the early CTAs' larger ranges still fit their id windows.  No skew otherwise.
constexpr float kSkewUsPerPos = 8192.f / 6.4e6f;   // one block of two kv heads at 6.4 TB/s (us)
__device__ __forceinline__ int late_streams(int total, int streams, int ctas, const Params& p) {
  if (p.skew_lead_us <= 0.f || p.skew_full <= 0 || p.skew_full >= ctas) return streams;
  const float loop_us = fmaxf((float)total * kSkewUsPerPos, 1.f);
  int nl = streams - __float2int_rn((float)streams * p.skew_lead_us / loop_us);
  nl = max((streams * 5 + 7) / 8, min(streams, nl));
  if (nl == streams) return streams;
  const int units = p.skew_full * streams + (ctas - p.skew_full) * nl;
  if ((int64_t)v2_chunk(total, units, p.max_blocks, p.max_parts) * streams > kV5IdCap)
    return streams;
  return nl;
}
// Stream range of CTA b: the first `full` CTAs take `streams` chunks each, the rest nl.
__host__ __device__ __forceinline__ void cta_range(int b, int full, int streams, int nl, int chunk,
                                                   int total, int& cb, int& ce) {
  const int first = b < full ? b * streams : full * streams + (b - full) * nl;
  cb = first * chunk;
  ce = min(total, cb + (b < full ? streams : nl) * chunk);
}

template <int HP, int NT>
__device__ __forceinline__ bool resolve_stream(const Params& p, int batch, int streams, int* s_off,
                                               int* ids, uint8_t* vtok, int* s_wsum, int& chunk,
                                               int& cb, int& ce) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KVH = p.num_kv_heads;
  const int KVU = KVH / HP;
  auto nblk_of = [&](int r) {
    const int ctx = p.context_lens[r];
    return ctx > 0 ? min((ctx + kBlock - 1) / kBlock, p.max_blocks) : 0;
  };
  const int per = (batch + NT - 1) / NT;
  const int r0 = min(batch, tid * per), r1 = min(batch, r0 + per);
  int local = 0;
  for (int r = r0; r < r1; ++r) local += KVU * nblk_of(r);
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_wsum[warp] = incl;
  __syncthreads();
  int run = incl - local;
  for (int w = 0; w < warp; ++w) run += s_wsum[w];
  for (int r = r0; r < r1; ++r) {
    s_off[r] = run;
    run += KVU * nblk_of(r);
  }
  if (tid == 0) {
    int tot = 0;
    for (int w = 0; w < NT / 32; ++w) tot += s_wsum[w];
    s_off[batch] = tot;
  }
  __syncthreads();
  const int total = s_off[batch];
  const int nl = late_streams(total, streams, (int)gridDim.x, p);
  const int full = nl < streams ? p.skew_full : (int)gridDim.x;
  chunk = v2_chunk(total, full * streams + ((int)gridDim.x - full) * nl, p.max_blocks,
                   p.max_parts);
  cta_range((int)blockIdx.x, full, streams, nl, chunk, total, cb, ce);
  if (cb >= total) return false;
  for (int q = tid; q < ce - cb; q += NT) {
    const int pos = cb + q;
    int lo = 0, hi = batch;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_off[mid] <= pos) lo = mid; else hi = mid;
    }
    const int nb = (s_off[lo + 1] - s_off[lo]) / KVU;
    const int rel = pos - s_off[lo];
    const int unit = rel / nb, j = rel - unit * nb;
    const int brow = p.row_index ? p.row_index[lo] : lo;
    const int phys = p.block_tables[(int64_t)brow * p.bt_stride + j];
    const bool bad = phys < 0 || (int64_t)phys >= p.num_blocks;
    ids[q] = bad ? -1 : (phys * KVH + unit * HP) * kBlock;
    vtok[q] = (uint8_t)min(kBlock, p.context_lens[lo] - j * kBlock);
  }
  __syncthreads();
  return true;
}

template <int HP>
struct CfgV4 {
  static constexpr int kTile = HP * kBlock * 64 * 2;
  static constexpr int kStage = 2 * kTile;
  static constexpr int kRing = kV4Warps * kV4Stages * kStage;
  static constexpr int kBars = kV4Warps * kV4Stages * 8;
  static constexpr int kIds = kV4IdCap * 4;
  static constexpr int kVtok = kV4IdCap;
  static constexpr int kOffBytes = (kV2MaxBatch + 1) * 4;
  static constexpr int kTotal = kRing + kBars + kIds + kVtok + kOffBytes + 1024;
  static_assert(kTotal <= 227 * 1024, "v4 shared memory");
};

template <typename T, int HP>
__global__ void __launch_bounds__(kV4Warps * 32, 1)
decode_kernel_v4(const __grid_constant__ CUtensorMap kmap,
                 const __grid_constant__ CUtensorMap vmap, Params p, int batch) {
  if (threadIdx.x == 0) {   // descriptors are kernel parameters: independent of earlier kernels
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  pdl_wait();
  pdl_launch_dependents();
  using C = CfgV4<HP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t bar_all = smem_u32(smem + C::kRing);
  int* ids = reinterpret_cast<int*>(smem + C::kRing + C::kBars);
  uint8_t* vtok = smem + C::kRing + C::kBars + C::kIds;
  int* s_off = reinterpret_cast<int*>(smem + C::kRing + C::kBars + C::kIds + C::kVtok);
  constexpr int kThreads = kV4Warps * 32;
  __shared__ int s_wsum[kThreads / 32];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KVH = p.num_kv_heads;
  const int KVU = KVH / HP;
  if (tid < kV4Warps * kV4Stages) {
    mbar_init(bar_all + 8 * tid, 1);
    fence_mbar_init();
  }
  int chunk, cb, ce;
  if (!resolve_stream<HP, kThreads>(p, batch, kV4Warps, s_off, ids, vtok, s_wsum, chunk, cb, ce))
    return;

  int pos = min(ce, cb + warp * chunk);
  const int end = min(ce, pos + chunk);
  if (pos >= end) return;
  uint8_t* ring = smem + warp * kV4Stages * C::kStage;
  const uint32_t bar = bar_all + warp * kV4Stages * 8;
  const uint64_t pol = l2_policy_evict_first();
  const int G = p.group;
  const int g = lane >> 2, t4 = lane & 3;

  // issue cursor: the next stream position with a readable block (after a negative entry the
  // rest of its unit is skipped, exactly as the consume cursor below does)
  auto unit_end = [&](int pp) {
    int lo = 0, hi = batch;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_off[mid] <= pp) lo = mid; else hi = mid;
    }
    const int nb = (s_off[lo + 1] - s_off[lo]) / KVU;
    return s_off[lo] + ((pp - s_off[lo]) / nb + 1) * nb;
  };
  int ip = pos, issued = 0, consumed = 0;
  auto skip_stops = [&]() {
    while (ip < end && ids[ip - cb] < 0) ip = min(end, unit_end(ip));
  };
  auto issue = [&]() {
    if (lane == 0) {
      const int st = issued % kV4Stages;
      const uint32_t dst = smem_u32(ring + st * C::kStage);
      // Reads of the stage by ldmatrix completed before the MMAs that consume them issued;
      // the zeroing writes fenced themselves (swapped_block).
      mbar_arrive_expect_tx(bar + 8 * st, C::kStage);
      const int y = ids[ip - cb];
      tma_load_2d_hint(dst, &kmap, bar + 8 * st, 0, y, pol);
      tma_load_2d_hint(dst + C::kTile, &vmap, bar + 8 * st, 0, y, pol);
    }
    ++issued;
    ++ip;
    skip_stops();
  };
  skip_stops();
  while (issued < kV4Stages && ip < end) issue();

  uint32_t phase = 0;
  uint32_t qb[HP][4][2];
  float m[HP][2], l[HP][2], o[HP][4][4];

  while (pos < end) {
    // ---- a piece: positions of one unit inside [pos, end)
    int lo = 0, hi = batch;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_off[mid] <= pos) lo = mid; else hi = mid;
    }
    const int row = lo;
    const int nb = (s_off[row + 1] - s_off[row]) / KVU;
    const int unit = (pos - s_off[row]) / nb;
    const int pstart = s_off[row] + unit * nb;
    const int pend = min(end, pstart + nb);
    const int piece = pos / chunk - pstart / chunk;
    const int pieces = (pstart + nb - 1) / chunk - pstart / chunk + 1;
    {
      const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)row * p.q_stride;
#pragma unroll
      for (int sub = 0; sub < HP; ++sub) {
        const T* qh = qrow + (int64_t)((unit * HP + sub) * G + g) * 64;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          qb[sub][ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 2 * t4) : 0u;
          qb[sub][ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 8 + 2 * t4) : 0u;
        }
        m[sub][0] = m[sub][1] = -INFINITY;
        l[sub][0] = l[sub][1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) o[sub][mt][0] = o[sub][mt][1] = o[sub][mt][2] = o[sub][mt][3] = 0.f;
      }
    }
    int stop = 0;
    for (; pos < pend; ++pos) {
      if (ids[pos - cb] < 0) { stop = 1; pos = pend; break; }
      const int st = consumed % kV4Stages;
      if (!mbar_wait(bar + 8 * st, (phase >> st) & 1u, TI_DEVERR_ATTN_WAIT)) return;
      phase ^= 1u << st;
      uint8_t* kt = ring + st * C::kStage;
      const int valid = vtok[pos - cb];
#pragma unroll
      for (int sub = 0; sub < HP; ++sub) {
        uint8_t* ksub = kt + sub * kBlock * 128;
        uint8_t* vsub = kt + C::kTile + sub * kBlock * 128;
        swapped_block<T>(smem_u32(ksub), smem_u32(vsub), vsub, valid, lane, qb[sub], p.scale_log2,
                         m[sub], l[sub], o[sub]);
      }
      ++consumed;
      __syncwarp();                    // every lane is done with the stage before it is reused
      if (ip < end) issue();
    }
    // ---- finish the piece: lane holds heads (2t4, 2t4+1) x dims (16mt+g, 16mt+g+8)
    T* outp = reinterpret_cast<T*>(p.out) + (int64_t)row * p.out_stride;
    const int64_t pair = (int64_t)row * KVU + unit;
#pragma unroll
    for (int sub = 0; sub < HP; ++sub)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1)
          l[sub][j] += __shfl_xor_sync(0xffffffffu, l[sub][j], off);
    if (piece == 0 && lane == 0) p.ws_pieces[pair] = pieces;   // read by merge_pieces_kernel
    if (pieces == 1) {
#pragma unroll
      for (int sub = 0; sub < HP; ++sub)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int hl = 2 * t4 + j;
          if (hl >= G) continue;
          const float inv = 1.f / l[sub][j];           // l == 0 -> NaN (attention.cu:150)
          T* oh = outp + (int64_t)((unit * HP + sub) * G + hl) * 64;
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            oh[mt * 16 + g] = Elem<T>::from_f(o[sub][mt][j] * inv);
            oh[mt * 16 + g + 8] = Elem<T>::from_f(o[sub][mt][2 + j] * inv);
          }
        }
    } else {
#pragma unroll
      for (int sub = 0; sub < HP; ++sub)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int hl = 2 * t4 + j;
          if (hl >= G) continue;
          const int64_t sl = ((int64_t)row * p.num_heads + (unit * HP + sub) * G + hl) * p.max_parts + piece;
          float* wo = p.ws_o + sl * 64;
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            wo[mt * 16 + g] = o[sub][mt][j];
            wo[mt * 16 + g + 8] = o[sub][mt][2 + j];
          }
          if (g == 0) *reinterpret_cast<float2*>(p.ws_ml + sl * 2) = make_float2(m[sub][j], l[sub][j]);
        }
      if (lane == 0) p.ws_stop[pair * p.max_parts + piece] = stop;
    }
  }
}

// v4 split-K merge: one CTA per (sequence, unit of HP kv heads), one thread per (query head of
// the unit, 4 dims).  Units that v4 did not split (pieces == 1) or that have no blocks are left
// as they are.  Two rounds of loads (context length and piece count, then all of the unit's
// partials): this runs right after the attention kernel (programmatic dependent launch).
template <typename T>
__global__ void __launch_bounds__(256)
merge_pieces_kernel(Params p, int units, int nheads) {
  pdl_wait();
  pdl_launch_dependents();
  const int pair = blockIdx.x;
  const int row = pair / units, unit = pair % units;
  const int h = threadIdx.x >> 4, d4 = threadIdx.x & 15;
  if (h >= nheads) return;
  const int32_t* stops = p.ws_stop + (int64_t)pair * p.max_parts;
  const int64_t base = ((int64_t)row * p.num_heads + unit * nheads + h) * p.max_parts;
  // Rounds of kRound pieces, all of a round's partials loaded together (one round for the
  // pieces a decode step's unit usually has); pieces are used up to and including the first
  // that stopped at a negative block-table entry, and each round's maximum rescales the running
  // sums (online softmax over the pieces).  The first round's slots (within the unit's
  // max_parts slots, whatever the piece count) are loaded together with the context length and
  // the piece count: one round trip; slots past the count are dropped.  (8 slots a round keep
  // the kernel at two CTAs per SM: 256 sequences' merges in one wave.)
  constexpr int kRound = 8;
  int st[kRound];
  float2 ml[kRound];
  float4 v[kRound];
#pragma unroll
  for (int i = 0; i < kRound; ++i) {
    if (i < p.max_parts) {
      st[i] = stops[i];
      ml[i] = reinterpret_cast<const float2*>(p.ws_ml)[base + i];
      v[i] = reinterpret_cast<const float4*>(p.ws_o + (base + i) * 64)[d4];
    }
  }
  const int ctx = p.context_lens[row];
  const int pieces = min(p.ws_pieces[pair], p.max_parts);
  if (ctx <= 0 || pieces <= 1) return;   // no blocks (row left untouched) or not split
  int use = pieces;
  float M = -INFINITY, L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q0 = 0; q0 < use; q0 += kRound) {
#pragma unroll
    for (int i = 0; i < kRound; ++i) {
      const int q = q0 + i;
      if (q0 > 0 && q < use) {
        st[i] = stops[q];
        ml[i] = reinterpret_cast<const float2*>(p.ws_ml)[base + q];
        v[i] = reinterpret_cast<const float4*>(p.ws_o + (base + q) * 64)[d4];
      } else if (q >= use) {
        st[i] = 0;
        ml[i] = make_float2(-INFINITY, 0.f);
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    int n = min(kRound, use - q0);          // this round's pieces, up to the first stop
    bool stopped = false;
#pragma unroll
    for (int i = kRound - 1; i >= 0; --i)
      if (i < n && st[i]) { n = i + 1; stopped = true; }
    if (stopped) use = q0 + n;              // no later round: the stop ends the unit's pieces
    float Mr = M;
#pragma unroll
    for (int i = 0; i < kRound; ++i)
      if (i < n) Mr = fmaxf(Mr, ml[i].x);
    const float fo = M == -INFINITY ? 0.f : fast_exp2(M - Mr);   // rescale the earlier rounds
    L *= fo;
    acc.x *= fo; acc.y *= fo; acc.z *= fo; acc.w *= fo;
#pragma unroll
    for (int i = 0; i < kRound; ++i) {
      if (i < n) {
        const float f = ml[i].x == -INFINITY ? 0.f : fast_exp2(ml[i].x - Mr);
        L += ml[i].y * f;
        acc.x += f * v[i].x; acc.y += f * v[i].y; acc.z += f * v[i].z; acc.w += f * v[i].w;
      }
    }
    M = Mr;
  }
  const float inv = 1.f / L;               // L == 0 -> NaN (attention.cu:150)
  T* dst = reinterpret_cast<T*>(p.out) + (int64_t)row * p.out_stride +
           (int64_t)(unit * nheads + h) * 64 + d4 * 4;
  uint2 u;
  u.x = Elem<T>::pack2(acc.x * inv, acc.y * inv);
  u.y = Elem<T>::pack2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(dst) = u;
}

// Merge for units cut into more than 16 pieces (small batches): one CTA of 128 threads per
// (sequence, unit, query head of the unit), 8 threads per 4 dims, each taking every 8th piece,
// so that all of a unit's partials (up to kV5MaxPiecesSmall) arrive in one round of loads
// instead of rounds of 16, and small CTAs put every merge of a small batch on the SMs in one
// wave.  Pieces are used up to and including the first that stopped at a negative block-table
// entry; each thread folds its pieces into (max, sum, O) and the 8 are combined by shuffles in
// a fixed tree (deterministic).
constexpr int kWideLanes = 8;
constexpr int kWideThreads = 16 * kWideLanes;
constexpr int kWidePer = (kV5MaxPiecesSmall + kWideLanes - 1) / kWideLanes;   // pieces / thread
template <typename T>
__global__ void __launch_bounds__(kWideThreads)
merge_pieces_wide_kernel(Params p, int units, int nheads) {
  pdl_wait();
  pdl_launch_dependents();
  const int pair = blockIdx.x, h = blockIdx.y;
  const int row = pair / units, unit = pair % units;
  const int d4 = threadIdx.x / kWideLanes, j = threadIdx.x % kWideLanes;   // piece lanes adjacent
  const int32_t* stops = p.ws_stop + (int64_t)pair * p.max_parts;
  const int64_t base = ((int64_t)row * p.num_heads + unit * nheads + h) * p.max_parts;
  int st[kWidePer];
  float2 ml[kWidePer];
  float4 v[kWidePer];
  // every slot of the unit (max_parts of them) loaded with the context length and the piece
  // count in one round trip; slots past the count are dropped
#pragma unroll
  for (int i = 0; i < kWidePer; ++i) {
    const int q = j + kWideLanes * i;
    if (q < p.max_parts) {
      st[i] = stops[q];
      ml[i] = reinterpret_cast<const float2*>(p.ws_ml)[base + q];
      v[i] = reinterpret_cast<const float4*>(p.ws_o + (base + q) * 64)[d4];
    }
  }
  const int ctx = p.context_lens[row];
  const int pieces = min(p.ws_pieces[pair], p.max_parts);
  if (ctx <= 0 || pieces <= 1) return;   // whole CTA: no blocks, or the unit was not split
  int first_stop = pieces;               // index of this thread's first stopped piece
#pragma unroll
  for (int i = 0; i < kWidePer; ++i) {
    if (j + kWideLanes * i >= pieces) {
      st[i] = 0;
      ml[i] = make_float2(-INFINITY, 0.f);
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
#pragma unroll
  for (int i = kWidePer - 1; i >= 0; --i)
    if (st[i] && j + kWideLanes * i < first_stop) first_stop = j + kWideLanes * i;
#pragma unroll
  for (int o = 1; o < kWideLanes; o <<= 1)
    first_stop = min(first_stop, __shfl_xor_sync(0xffffffffu, first_stop, o));
  float M = -INFINITY;
#pragma unroll
  for (int i = 0; i < kWidePer; ++i)
    if (j + kWideLanes * i <= first_stop) M = fmaxf(M, ml[i].x);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kWidePer; ++i) {
    if (j + kWideLanes * i <= first_stop && ml[i].x != -INFINITY) {
      const float f = fast_exp2(ml[i].x - M);
      L += ml[i].y * f;
      acc.x += f * v[i].x; acc.y += f * v[i].y; acc.z += f * v[i].z; acc.w += f * v[i].w;
    }
  }
#pragma unroll
  for (int o = 1; o < kWideLanes; o <<= 1) {   // combine the lanes' (M, L, acc)
    const float Mo = __shfl_xor_sync(0xffffffffu, M, o);
    const float Lo = __shfl_xor_sync(0xffffffffu, L, o);
    const float ax = __shfl_xor_sync(0xffffffffu, acc.x, o);
    const float ay = __shfl_xor_sync(0xffffffffu, acc.y, o);
    const float az = __shfl_xor_sync(0xffffffffu, acc.z, o);
    const float aw = __shfl_xor_sync(0xffffffffu, acc.w, o);
    const float Mn = fmaxf(M, Mo);
    const float fa = M == -INFINITY ? 0.f : fast_exp2(M - Mn);
    const float fb = Mo == -INFINITY ? 0.f : fast_exp2(Mo - Mn);
    L = L * fa + Lo * fb;
    acc.x = acc.x * fa + ax * fb; acc.y = acc.y * fa + ay * fb;
    acc.z = acc.z * fa + az * fb; acc.w = acc.w * fa + aw * fb;
    M = Mn;
  }
  if (j != 0) return;
  const float inv = 1.f / L;               // L == 0 -> NaN (attention.cu:150)
  T* dst = reinterpret_cast<T*>(p.out) + (int64_t)row * p.out_stride +
           (int64_t)(unit * nheads + h) * 64 + d4 * 4;
  uint2 u;
  u.x = Elem<T>::pack2(acc.x * inv, acc.y * inv);
  u.y = Elem<T>::pack2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(dst) = u;
}

// ==========================================================================================
// v5: one producer warp and pairs of consumer warps (head_dim 64, units of two kv heads,
// GQA groups <= 8)
//
// Same block stream, chunking (one chunk per warp PAIR), pieces, split-K workspace and merge
// as v4.  Warp 0 (lane 0) issues every TMA load of the CTA: per pair a kV5Stages-deep ring,
// each stage the K and V tiles of one block for both kv heads of the unit (two 4 KB boxes).
// The two warps of a pair read the same stage, warp 2i+1 computing the first kv head and warp
// 2i+2 the second (swapped_block), and release it through an empty barrier of count 2.  With
// the issue off the consumers and one head per consumer, a pair finishes a block in about the
// time v4 spends on one of its two heads.
// ==========================================================================================
constexpr int kV5Pairs = 8;
constexpr int kV5Stages = 3;
constexpr int kV5Threads = (1 + 2 * kV5Pairs) * 32;

// Positions the planned call loads with the plan header in its first round (the whole range of
// a 256-sequence batch of contexts up to ~2k tokens); longer ranges take a second round.
constexpr int kV5FirstRound = 2048;

struct CfgV5 {
  static constexpr int kTile = 2 * kBlock * 64 * 2;          // K (or V) of one block, 2 heads
  static constexpr int kStage = 2 * kTile;
  static constexpr int kRing = kV5Pairs * kV5Stages * kStage;   // 192 KB
  static constexpr int kBars = 2 * kV5Pairs * kV5Stages * 8;    // full, then empty
  static constexpr int kIds = kV5IdCap * 4;
  static constexpr int kVtok = kV5IdCap;
  // then s_off[batch + 1] (padded to 16 bytes): the dynamic part, sized per launch
  static constexpr int kFixed = kRing + kBars + kIds + kVtok + 1024;   // + alignment slack
  static constexpr int kMaxSmem = 227 * 1024 - 256;   // 256 bytes for the static s_wsum / s_hdr
  static constexpr int kMaxBatch = (kMaxSmem - kFixed) / 16 * 16 / 4 - 1;
  static int total(int batch) { return kFixed + ((batch + 1) * 4 + 15) / 16 * 16; }
  static_assert(kMaxBatch >= 1024, "v5 serves batches of at least 1024 sequences");
  static_assert((kRing + kBars) % 16 == 0 && kIds % 16 == 0 && kVtok % 16 == 0, "int4 copies");
};

// Plan layout (int32 words; base 16-byte aligned), written by plan_kernel for the v5 chunking:
//   [0] total positions  [1] chunk  [2] consumers (CTAs x kV5Pairs)  [3] batch
//   [4] ids word offset  [5] vtok byte offset  [6] CTAs with kV5Pairs streams (the rest: late)
//   [7] streams of a late CTA (kV5Pairs: no skew)
//   [8 ..) s_off[0 .. batch] (padded to 4 words), then per CTA a kV5IdCap slot of ids (int32)
//   and, after all id slots, per CTA a kV5IdCap slot of vtok (bytes).
__host__ __device__ inline int64_t plan_ids_word(int batch) { return 8 + (batch + 1 + 3) / 4 * 4; }
__host__ __device__ inline int64_t plan_vtok_byte(int batch, int ctas) {
  return (plan_ids_word(batch) + (int64_t)ctas * kV5IdCap) * 4;
}
inline size_t plan_bytes(int batch, int ctas) {
  return (size_t)((plan_vtok_byte(batch, ctas) + (int64_t)ctas * kV5IdCap + 15) / 16 * 16);
}

// One CTA per v5 CTA: the v5 prologue (resolve_stream), its ids / vtok kept in the plan's slot.
template <int NT>
__global__ void __launch_bounds__(NT)
plan_kernel(Params p, int batch, int32_t* plan) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int s_off[kV2MaxBatch + 1];
  __shared__ int s_wsum[NT / 32];
  int32_t* ids = plan + plan_ids_word(batch) + (int64_t)blockIdx.x * kV5IdCap;
  uint8_t* vtok = reinterpret_cast<uint8_t*>(plan) + plan_vtok_byte(batch, gridDim.x) +
                  (int64_t)blockIdx.x * kV5IdCap;
  int chunk = 0, cb = 0, ce = 0;
  resolve_stream<2, NT>(p, batch, kV5Pairs, s_off, ids, vtok, s_wsum, chunk, cb, ce);
  if (blockIdx.x == 0) {
    const int nl = late_streams(s_off[batch], kV5Pairs, (int)gridDim.x, p);
    for (int r = threadIdx.x; r <= batch; r += NT) plan[8 + r] = s_off[r];
    if (threadIdx.x == 0) {
      plan[0] = s_off[batch];
      plan[1] = chunk;
      plan[2] = gridDim.x * kV5Pairs;
      plan[3] = batch;
      plan[4] = (int)plan_ids_word(batch);
      plan[5] = (int)plan_vtok_byte(batch, gridDim.x);
      plan[6] = nl < kV5Pairs ? p.skew_full : (int)gridDim.x;
      plan[7] = nl;
    }
  }
}

template <typename T, bool PLANNED>
__global__ void __launch_bounds__(kV5Threads, 1)
decode_kernel_v5(const __grid_constant__ CUtensorMap kmap,
                 const __grid_constant__ CUtensorMap vmap, Params p, int batch) {
  if (threadIdx.x == 0) {   // descriptors are kernel parameters: independent of earlier kernels
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  // early (TI_ATTN_EARLY_KV): the plan and all blocks but each unit's last are final before
  // the previous kernel started, so the plan load and the producer's first loads run before the
  // wait for it; every thread waits before it reads q or a unit's last block, or writes.
  const bool early = PLANNED && p.early;
  if (!early) {
    pdl_wait();
    pdl_launch_dependents();
  }
  using C = CfgV5;
  constexpr int kSlots = kV5Pairs * kV5Stages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t full0 = smem_u32(smem + C::kRing);     // [pair][stage]
  const uint32_t empty0 = full0 + kSlots * 8;
  int* ids = reinterpret_cast<int*>(smem + C::kRing + C::kBars);
  uint8_t* vtok = smem + C::kRing + C::kBars + C::kIds;
  int* s_off = reinterpret_cast<int*>(smem + C::kRing + C::kBars + C::kIds + C::kVtok);
  __shared__ int s_wsum[kV5Threads / 32];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KVU = p.num_kv_heads / 2;
  if (tid < kSlots) {
    mbar_init(full0 + 8 * tid, 1);    // the producer's arrive + the two tiles' bytes
    mbar_init(empty0 + 8 * tid, 2);   // one arrive per consumer warp of the pair
    fence_mbar_init();
  }
  int chunk, cb, ce;
  if constexpr (PLANNED) {
    // one round of loads: header, s_off and the first kV5FirstRound positions of this CTA's id
    // and vtok slots; a longer range loads the rest in a second round once the header is known
    __shared__ int s_hdr[4];
    const int32_t* pl = p.plan;
    const int n_off = (batch + 1 + 3) / 4;
    const int4* g_off = reinterpret_cast<const int4*>(pl + 8);
    const int4* g_ids = reinterpret_cast<const int4*>(pl + plan_ids_word(batch) +
                                                      (int64_t)blockIdx.x * kV5IdCap);
    const int4* g_vt = reinterpret_cast<const int4*>(
        reinterpret_cast<const uint8_t*>(pl) + plan_vtok_byte(batch, gridDim.x) +
        (int64_t)blockIdx.x * kV5IdCap);
    constexpr int n_ids = kV5FirstRound / 4, n_vt = kV5FirstRound / 16;
    // L2-coherent loads (ld.global.cg): an early call reads the plan before its wait
    for (int i = tid; i < n_off + n_ids + n_vt; i += kV5Threads) {
      if (i < n_off) reinterpret_cast<int4*>(s_off)[i] = __ldcg(g_off + i);
      else if (i < n_off + n_ids) reinterpret_cast<int4*>(ids)[i - n_off] = __ldcg(g_ids + i - n_off);
      else reinterpret_cast<int4*>(vtok)[i - n_off - n_ids] = __ldcg(g_vt + i - n_off - n_ids);
    }
    if (tid == 0) {
      const int4 h = __ldcg(reinterpret_cast<const int4*>(pl));
      const int4 h2 = __ldcg(reinterpret_cast<const int4*>(pl) + 1);
      const bool ok = h.w == batch && h.z == (int)gridDim.x * kV5Pairs &&
                      h.y > 0 && (int64_t)h.y * kV5Pairs <= kV5IdCap && h2.z >= 0 &&
                      h2.z <= (int)gridDim.x && h2.w >= 1 && h2.w <= kV5Pairs;
      if (!ok) raise_device_error(TI_DEVERR_ATTN_PLAN);   // a plan of another batch / grid
      s_hdr[0] = ok ? h.x : 0;
      s_hdr[1] = ok ? h.y : 1;
      s_hdr[2] = ok ? h2.z : (int)gridDim.x;
      s_hdr[3] = ok ? h2.w : kV5Pairs;
    }
    __syncthreads();
    chunk = s_hdr[1];
    cta_range((int)blockIdx.x, s_hdr[2], kV5Pairs, s_hdr[3], chunk, s_hdr[0], cb, ce);
    if (cb >= s_hdr[0]) return;
    if (ce - cb > kV5FirstRound) {   // the same for every thread of the CTA; ce - cb <= kV5IdCap
      const int n_ids2 = (ce - cb + 3) / 4, n_vt2 = (ce - cb + 15) / 16;
      for (int i = n_ids + tid; i < n_ids2; i += kV5Threads)
        reinterpret_cast<int4*>(ids)[i] = __ldcg(g_ids + i);
      for (int i = n_vt + tid; i < n_vt2; i += kV5Threads)
        reinterpret_cast<int4*>(vtok)[i] = __ldcg(g_vt + i);
      __syncthreads();
    }
  } else {
    if (!resolve_stream<2, kV5Threads>(p, batch, kV5Pairs, s_off, ids, vtok, s_wsum, chunk, cb,
                                       ce))
      return;
  }
  // end of the unit that contains stream position pp
  auto unit_end = [&](int pp) {
    int lo = 0, hi = batch;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_off[mid] <= pp) lo = mid; else hi = mid;
    }
    const int nb = (s_off[lo + 1] - s_off[lo]) / KVU;
    return s_off[lo] + ((pp - s_off[lo]) / nb + 1) * nb;
  };

  if (warp == 0) {
    // ---- producer: lane i issues the loads of pair i, a load whenever the pair's next stage
    // is free (one SIMT test of all pairs' barriers per round).  The issue cursor skips the rest
    // of a unit after a negative entry, as the consumers do.
    if (lane >= kV5Pairs) return;
    const uint64_t pol = l2_policy_evict_first();
    int ip = min(ce, cb + lane * chunk);
    const int iend = min(ce, ip + chunk);
    while (ip < iend && ids[ip - cb] < 0) ip = min(iend, unit_end(ip));
    int issued = 0, idle = 0;
    if (early) {
      // first uses of the pair's stages, up to the first block that is the last of its unit
      // (it holds the token the previous kernel appended)
      while (ip < iend && issued < kV5Stages && ip + 1 < unit_end(ip)) {
        const int slot = lane * kV5Stages + issued;
        const uint32_t fb = full0 + 8 * slot;
        const uint32_t dst = smem_u32(smem + slot * C::kStage);
        mbar_arrive_expect_tx(fb, C::kStage);
        const int y = ids[ip - cb];
        tma_load_2d_hint(dst, &kmap, fb, 0, y, pol);
        tma_load_2d_hint(dst + C::kTile, &vmap, fb, 0, y, pol);
        ++issued;
        ++ip;
        while (ip < iend && ids[ip - cb] < 0) ip = min(iend, unit_end(ip));
      }
      pdl_wait();
      pdl_launch_dependents();
    }
    long long t0 = clock64();
    while (ip < iend) {
      const int st = issued % kV5Stages;
      const int use = issued / kV5Stages;
      const int slot = lane * kV5Stages + st;
      // stage reuse: wait for the consumption of its previous use (phase use - 1)
      if (use == 0 || mbar_test_wait(empty0 + 8 * slot, (use - 1) & 1)) {
        const uint32_t fb = full0 + 8 * slot;
        const uint32_t dst = smem_u32(smem + slot * C::kStage);
        mbar_arrive_expect_tx(fb, C::kStage);
        const int y = ids[ip - cb];
        tma_load_2d_hint(dst, &kmap, fb, 0, y, pol);
        tma_load_2d_hint(dst + C::kTile, &vmap, fb, 0, y, pol);
        ++issued;
        ++ip;
        while (ip < iend && ids[ip - cb] < 0) ip = min(iend, unit_end(ip));
        t0 = clock64();
        idle = 0;
      } else if (clock64() - t0 > kWaitCycles) {
        raise_device_error(TI_DEVERR_ATTN_WAIT);   // the pair's consumers time out as well
        break;
      } else if (++idle > 64) {
        __nanosleep(32);   // long waits only: a sleeping lane would miss the free stage
      }
    }
    return;
  }

  // ---- consumers
  if (early) {
    pdl_wait();
    pdl_launch_dependents();
  }
  const int cw = warp - 1, pr = cw >> 1, sub = cw & 1;
  int pos = min(ce, cb + pr * chunk);
  const int end = min(ce, pos + chunk);
  if (pos >= end) return;
  uint8_t* ring = smem + pr * kV5Stages * C::kStage;
  const uint32_t fullp = full0 + pr * kV5Stages * 8, emptyp = empty0 + pr * kV5Stages * 8;
  const int G = p.group;
  const int g = lane >> 2, t4 = lane & 3;
  int consumed = 0;
  uint32_t phase = 0;
  uint32_t qb[4][2];
  float m[2], l[2], o[4][4];

  while (pos < end) {
    // ---- a piece: positions of one unit inside [pos, end)
    int lo = 0, hi = batch;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_off[mid] <= pos) lo = mid; else hi = mid;
    }
    const int row = lo;
    const int nb = (s_off[row + 1] - s_off[row]) / KVU;
    const int unit = (pos - s_off[row]) / nb;
    const int pstart = s_off[row] + unit * nb;
    const int pend = min(end, pstart + nb);
    const int piece = pos / chunk - pstart / chunk;
    const int pieces = (pstart + nb - 1) / chunk - pstart / chunk + 1;
    if (pieces > p.max_parts) {                // only a mismatched plan gets here
      raise_device_error(TI_DEVERR_ATTN_PLAN);
      return;
    }
    const int head0 = (unit * 2 + sub) * G;   // first query head of this warp's kv head
    {
      const T* qh = reinterpret_cast<const T*>(p.q) + (int64_t)row * p.q_stride +
                    (int64_t)(head0 + g) * 64;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        qb[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 2 * t4) : 0u;
        qb[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 8 + 2 * t4) : 0u;
      }
      m[0] = m[1] = -INFINITY;
      l[0] = l[1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    }
    int stop = 0;
    for (; pos < pend; ++pos) {
      if (ids[pos - cb] < 0) { stop = 1; pos = pend; break; }
      const int st = consumed % kV5Stages;
      if (!mbar_wait(fullp + 8 * st, (phase >> st) & 1u, TI_DEVERR_ATTN_WAIT)) return;
      phase ^= 1u << st;
      uint8_t* kt = ring + st * C::kStage + sub * kBlock * 128;
      uint8_t* vt = ring + st * C::kStage + C::kTile + sub * kBlock * 128;
      swapped_block<T>(smem_u32(kt), smem_u32(vt), vt, vtok[pos - cb], lane, qb, p.scale_log2, m, l,
                       o);
      __syncwarp();                    // every lane is done with the stage before it is released
      if (lane == 0) mbar_arrive(emptyp + 8 * st);
      ++consumed;
    }
    // ---- finish the piece: lane holds heads (2t4, 2t4+1) x dims (16mt+g, 16mt+g+8)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) l[j] += __shfl_xor_sync(0xffffffffu, l[j], off);
    const int64_t pair = (int64_t)row * KVU + unit;
    if (piece == 0 && sub == 0 && lane == 0) p.ws_pieces[pair] = pieces;   // merge_pieces_kernel
    if (pieces == 1) {
      T* outp = reinterpret_cast<T*>(p.out) + (int64_t)row * p.out_stride;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int hl = 2 * t4 + j;
        if (hl >= G) continue;
        const float inv = 1.f / l[j];                 // l == 0 -> NaN (attention.cu:150)
        T* oh = outp + (int64_t)(head0 + hl) * 64;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          oh[mt * 16 + g] = Elem<T>::from_f(o[mt][j] * inv);
          oh[mt * 16 + g + 8] = Elem<T>::from_f(o[mt][2 + j] * inv);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int hl = 2 * t4 + j;
        if (hl >= G) continue;
        const int64_t sl = ((int64_t)row * p.num_heads + head0 + hl) * p.max_parts + piece;
        float* wo = p.ws_o + sl * 64;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          wo[mt * 16 + g] = o[mt][j];
          wo[mt * 16 + g + 8] = o[mt][2 + j];
        }
        if (g == 0) *reinterpret_cast<float2*>(p.ws_ml + sl * 2) = make_float2(m[j], l[j]);
      }
      if (sub == 0 && lane == 0) p.ws_stop[pair * p.max_parts + piece] = stop;
    }
  }
}

// ==========================================================================================
// Unit kernel: one CTA per unit (a sequence's pair of kv heads) for calls whose sequences are
// all short (at most kUnitMaxBlocks blocks) and whose units fit one wave of CTAs.  The producer
// warp and the 8 warp pairs stream the unit's blocks as v5's do (the pairs split the blocks into
// 8 contiguous chunks); the pairs' partials (max, sum, O) are combined in shared memory in a
// fixed order and normalised by the CTA itself: one launch, no split-K workspace, no merge
// kernel.  head_dim 64, even numbers of kv heads, GQA groups <= 8.  Reference semantics as v5
// (attention.cu:54-154): ctx 0 leaves the row untouched, reading stops at the first negative
// (or out-of-pool) block-table entry, a sequence without a readable token gets NaN.
// ==========================================================================================
constexpr int kUnitMaxBlocks = 32;   // context length <= 512 tokens

struct CfgUnit {
  static constexpr int kIds = kUnitMaxBlocks * 4;
  static constexpr int kSmem = CfgV5::kRing + CfgV5::kBars + kIds + kUnitMaxBlocks + 1024;
  // a pair's partial over its drained ring: O [sub][head][dim], then (m, l) [sub][head]
  static constexpr int kPartO = 2 * 8 * 64;
  static constexpr int kPartBytes = (kPartO + 2 * 8 * 2) * 4;
  static_assert(kPartBytes <= kV5Stages * CfgV5::kStage, "a pair's partial fits its ring");
  static_assert(kSmem <= 227 * 1024, "shared memory");
  static_assert(kUnitMaxBlocks <= kV5Threads, "one thread per table entry");
};

template <typename T>
__global__ void __launch_bounds__(kV5Threads, 1)
decode_kernel_unit(const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, Params p) {
  using C = CfgV5;
  constexpr int kSlots = kV5Pairs * kV5Stages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t full0 = smem_u32(smem + C::kRing);   // [pair][stage]
  const uint32_t empty0 = full0 + kSlots * 8;
  int* ids = reinterpret_cast<int*>(smem + C::kRing + C::kBars);
  uint8_t* vtok = smem + C::kRing + C::kBars + CfgUnit::kIds;
  __shared__ int s_nb, s_stop, s_ctx;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KVU = p.num_kv_heads / 2;
  const int row = (int)blockIdx.x / KVU, unit = (int)blockIdx.x % KVU;
  const int G = p.group;
  // set-up that reads nothing an earlier kernel writes, before the wait for it
  if (tid == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    s_stop = 1 << 30;
  }
  if (tid < kSlots) {
    mbar_init(full0 + 8 * tid, 1);    // the producer's arrive + the two tiles' bytes
    mbar_init(empty0 + 8 * tid, 2);   // one arrive per consumer warp of the pair
    fence_mbar_init();
  }
  pdl_wait();
  pdl_launch_dependents();
  // one round of loads: the context length and the whole table row (at most kUnitMaxBlocks
  // entries, one per thread), read together rather than the row after the length
  const int brow = p.row_index ? p.row_index[row] : row;
  const int32_t* bt = p.block_tables + (int64_t)brow * p.bt_stride;
  const int phys = tid < p.max_blocks ? bt[tid] : -1;
  if (tid == 0) {
    const int ctx = p.context_lens[row];
    s_ctx = ctx;
    s_nb = ctx > 0 ? min((ctx + kBlock - 1) / kBlock, p.max_blocks) : 0;
  }
  __syncthreads();
  const int nb = s_nb;
  // reading stops at the first bad entry (negative or past the pool)
  if (tid < nb && (phys < 0 || (int64_t)phys >= p.num_blocks)) atomicMin(&s_stop, tid);
  __syncthreads();
  const int nbe = min(nb, s_stop);
  if (tid < nbe) {
    ids[tid] = (phys * p.num_kv_heads + unit * 2) * kBlock;
    vtok[tid] = (uint8_t)min(kBlock, s_ctx - tid * kBlock);
  }
  __syncthreads();
  const int chunk = (nbe + kV5Pairs - 1) / kV5Pairs;
  // consumer state (pair pr, warp sub: kv head 2 unit + sub), kept across the barriers below
  const int cw = warp - 1, pr = cw >> 1, sub = cw & 1;
  const int g = lane >> 2, t4 = lane & 3;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, o[4][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  if (warp == 0) {
    // ---- producer: lane i issues pair i's loads, a load whenever the pair's next stage is free
    if (lane < kV5Pairs) {
      const uint64_t pol = l2_policy_evict_first();
      int ip = min(nbe, lane * chunk);
      const int iend = min(nbe, ip + chunk);
      int issued = 0, idle = 0;
      long long t0 = clock64();
      while (ip < iend) {
        const int st = issued % kV5Stages;
        const int use = issued / kV5Stages;
        const int slot = lane * kV5Stages + st;
        if (use == 0 || mbar_test_wait(empty0 + 8 * slot, (use - 1) & 1)) {
          const uint32_t fb = full0 + 8 * slot;
          const uint32_t dst = smem_u32(smem + slot * C::kStage);
          mbar_arrive_expect_tx(fb, C::kStage);
          tma_load_2d_hint(dst, &kmap, fb, 0, ids[ip], pol);
          tma_load_2d_hint(dst + C::kTile, &vmap, fb, 0, ids[ip], pol);
          ++issued;
          ++ip;
          t0 = clock64();
          idle = 0;
        } else if (clock64() - t0 > kWaitCycles) {
          raise_device_error(TI_DEVERR_ATTN_WAIT);   // the pair's consumers time out as well
          break;
        } else if (++idle > 64) {
          __nanosleep(32);
        }
      }
    }
  } else {
    // ---- consumers: pair pr, warp sub computes kv head 2 unit + sub over the pair's chunk
    int pos = min(nbe, pr * chunk);
    const int end = min(nbe, pos + chunk);
    if (pos < end) {
      const int head0 = (unit * 2 + sub) * G;
      uint32_t qb[4][2];
      const T* qh = reinterpret_cast<const T*>(p.q) + (int64_t)row * p.q_stride +
                    (int64_t)(head0 + g) * 64;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        qb[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 2 * t4) : 0u;
        qb[ks][1] = g < G ? *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 8 + 2 * t4) : 0u;
      }
      uint8_t* ring = smem + pr * kV5Stages * C::kStage;
      const uint32_t fullp = full0 + pr * kV5Stages * 8, emptyp = empty0 + pr * kV5Stages * 8;
      uint32_t phase = 0;
      for (int consumed = 0; pos < end; ++pos, ++consumed) {
        const int st = consumed % kV5Stages;
        if (!mbar_wait(fullp + 8 * st, (phase >> st) & 1u, TI_DEVERR_ATTN_WAIT)) break;
        phase ^= 1u << st;
        uint8_t* kt = ring + st * C::kStage + sub * kBlock * 128;
        uint8_t* vt = ring + st * C::kStage + C::kTile + sub * kBlock * 128;
        swapped_block<T>(smem_u32(kt), smem_u32(vt), vt, vtok[pos], lane, qb, p.scale_log2, m, l,
                         o);
        __syncwarp();                    // every lane is done with the stage before it is released
        if (lane == 0) mbar_arrive(emptyp + 8 * st);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) l[j] += __shfl_xor_sync(0xffffffffu, l[j], off);
    }
  }
  __syncthreads();   // every warp is done with the rings (all loads were consumed)
  if (warp > 0) {
    // the pair's partial over its drained ring (an empty pair: (-inf, 0) and zeros)
    float* po = reinterpret_cast<float*>(smem + pr * kV5Stages * C::kStage);
    float* pml = po + CfgUnit::kPartO;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int hl = 2 * t4 + j;
      if (hl >= G) continue;
      float* oh = po + (sub * 8 + hl) * 64;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        oh[mt * 16 + g] = o[mt][j];
        oh[mt * 16 + g + 8] = o[mt][2 + j];
      }
      if (g == 0) {
        pml[(sub * 8 + hl) * 2] = m[j];
        pml[(sub * 8 + hl) * 2 + 1] = l[j];
      }
    }
  }
  __syncthreads();   // every pair's partial is in shared memory
  if (s_ctx <= 0) return;   // ctx 0: the row is left as it was
  // ---- combine the 8 pairs in a fixed order, normalise, store: task = (sub, head, dim)
  T* outp = reinterpret_cast<T*>(p.out) + (int64_t)row * p.out_stride;
  for (int t = tid; t < 2 * G * 64; t += kV5Threads) {
    const int sb = t / (G * 64), hl = (t / 64) % G, d = t % 64;
    const int hi = sb * 8 + hl;
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < kV5Pairs; ++q) {
      const float* pq = reinterpret_cast<const float*>(smem + q * kV5Stages * C::kStage);
      M = fmaxf(M, pq[CfgUnit::kPartO + hi * 2]);
    }
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int q = 0; q < kV5Pairs; ++q) {
      const float* pq = reinterpret_cast<const float*>(smem + q * kV5Stages * C::kStage);
      const float mq = pq[CfgUnit::kPartO + hi * 2];
      if (mq == -INFINITY) continue;
      const float f = fast_exp2(mq - M);
      L += pq[CfgUnit::kPartO + hi * 2 + 1] * f;
      O += pq[hi * 64 + d] * f;
    }
    outp[(int64_t)((unit * 2 + sb) * G + hl) * 64 + d] = Elem<T>::from_f(O / L);   // L 0: NaN
  }
}

template <typename T>
static int launch_unit(const Params& p, const CUtensorMap& km, const CUtensorMap& vm, int units,
                       cudaStream_t stream) {
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel_unit<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, CfgUnit::kSmem);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(paged attention unit)");
    set_dev = dev;
  }
  return launch_kernel("paged attention unit launch", decode_kernel_unit<T>, dim3(units),
                       dim3(kV5Threads), CfgUnit::kSmem, stream, 1, km, vm, p);
}

template <typename T, bool PLANNED>
static int launch_v5(const Params& p, const CUtensorMap& km, const CUtensorMap& vm, int batch,
                     int ctas, cudaStream_t stream) {
  using C = CfgV5;
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel_v5<T, PLANNED>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::total(C::kMaxBatch));
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(paged attention v5)");
    set_dev = dev;
  }
  if (batch > C::kMaxBatch) return set_error(TI_ERR_UNSUPPORTED, "paged attention v5: batch too large");
  int rc = launch_kernel("paged attention v5 launch", decode_kernel_v5<T, PLANNED>,
                         dim3(ctas), dim3(kV5Threads), C::total(batch), stream, 1, km, vm, p,
                         batch);
  if (rc) return rc;
  const int units = p.num_kv_heads / 2;
  if (p.max_parts > kV2MaxPieces)   // small batches: up to kV5MaxPiecesSmall pieces per unit
    return launch_kernel("paged attention merge launch", merge_pieces_wide_kernel<T>,
                         dim3(batch * units, 2 * p.group), dim3(kWideThreads), 0, stream, 1, p,
                         units, 2 * p.group);
  return launch_kernel("paged attention merge launch", merge_pieces_kernel<T>,
                       dim3(batch * units), dim3(256), 0, stream, 1, p, units, 2 * p.group);
}

template <typename T, int HP>
static int launch_v4(const Params& p, const CUtensorMap& km, const CUtensorMap& vm, int batch,
                     cudaStream_t stream) {
  using C = CfgV4<HP>;
  static int set_dev = -1;
  static int sms = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel_v4<T, HP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kTotal);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(paged attention v4)");
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    set_dev = dev;
  }
  int rc = launch_kernel("paged attention v4 launch", decode_kernel_v4<T, HP>, dim3(sms),
                         dim3(kV4Warps * 32), C::kTotal, stream, 1, km, vm, p, batch);
  if (rc) return rc;
  const int units = p.num_kv_heads / HP;
  return launch_kernel("paged attention merge launch", merge_pieces_kernel<T>,
                       dim3(batch * units), dim3(256), 0, stream, 1, p, units, HP * p.group);
}

template <typename T, int HP>
static int launch_v2(const Params& p, const CUtensorMap& km, const CUtensorMap& vm, int batch,
                     cudaStream_t stream) {
  using C = CfgV2<HP>;
  static int set_dev = -1;
  static int sms = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel_v2<T, HP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kTotal);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(paged attention v2)");
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    set_dev = dev;
  }
  return launch_kernel("paged attention v2 launch", decode_kernel_v2<T, HP>, dim3(sms),
                       dim3(C::kWarps * 32), C::kTotal, stream, 1, km, vm, p, batch);
}

// TI_PAGED_ATTN_KERNEL=v2|v4|v5|unit restricts the choice among the equivalent head_dim-64
// kernels (for comparisons and tests; a kernel that cannot serve the call is still skipped).
static int forced_kernel() {
  const char* e = getenv("TI_PAGED_ATTN_KERNEL");
  return !e ? 0
            : !strcmp(e, "v2") ? 2
            : !strcmp(e, "v4") ? 4
            : !strcmp(e, "v5") ? 5
            : !strcmp(e, "unit") ? 6
                                 : 0;
}

// Partition size (KV blocks per split-K CTA of the v1 kernel) used when the caller passes 0.
static int default_partition(int /*max_blocks*/) { return kMaxPart; }

// The v2 kernel serves head_dim 64 and batches up to kV2MaxBatch.
static bool use_v2(int head_dim, int batch) { return head_dim == 64 && batch <= kV2MaxBatch; }
}  // namespace attn
}  // namespace ti

using namespace ti;

// Split-K slots per sequence: the v2 kernel cuts a (sequence, kv head) into at most
// kV2MaxPieces pieces; the v1 kernel into ceil(max_blocks / partition_blocks) partitions.
static int64_t attn_parts(int batch, int head_dim, int max_blocks, int partition_blocks) {
  if (attn::use_v2(head_dim, batch)) return attn::kV2MaxPieces;
  if (partition_blocks <= 0) partition_blocks = attn::default_partition(max_blocks);
  return (max_blocks + partition_blocks - 1) / partition_blocks;
}

static bool v5_path(int batch, int num_heads, int num_kv_heads, int head_dim, int max_blocks);

// Whether a decode call of this shape runs the unit kernel: head_dim 64, pairs of kv heads with
// GQA groups <= 8, every sequence at most kUnitMaxBlocks blocks and one CTA per unit fitting one
// wave.  Such a call splits no sequence: one launch, no workspace, no plan.
static bool unit_path(int batch, int num_heads, int num_kv_heads, int head_dim, int max_blocks) {
  if (!attn::use_v2(head_dim, batch) || num_kv_heads <= 0 || num_heads % num_kv_heads) return false;
  if (num_kv_heads % 2 || num_heads / num_kv_heads > 8 || max_blocks <= 0) return false;
  const int forced = attn::forced_kernel();
  if (forced != 0 && forced != 6) return false;
  return max_blocks <= attn::kUnitMaxBlocks &&
         (int64_t)batch * (num_kv_heads / 2) <= attn::sm_count();
}

// Split-K slots per (sequence, query head) of a call: 1 for the unit kernel; the v5 kernel at
// <= kV5SmallBatch sequences cuts units finer (kV5MaxPiecesSmall pieces at most), so a small
// batch's blocks spread over every SM; otherwise as attn_parts.
static int64_t split_parts(int batch, int num_heads, int num_kv_heads, int head_dim,
                           int max_blocks, int partition_blocks) {
  if (partition_blocks <= 0 && unit_path(batch, num_heads, num_kv_heads, head_dim, max_blocks))
    return 1;
  if (batch <= attn::kV5SmallBatch && partition_blocks <= 0 &&
      v5_path(batch, num_heads, num_kv_heads, head_dim, max_blocks))
    return attn::kV5MaxPiecesSmall;
  return attn_parts(batch, head_dim, max_blocks, partition_blocks);
}

namespace ti {
int64_t attn_split_parts(int batch, int num_heads, int num_kv_heads, int head_dim,
                         int max_blocks) {
  return split_parts(batch, num_heads, num_kv_heads, head_dim, max_blocks, 0);
}
}  // namespace ti

extern "C" size_t ti_paged_attention_workspace_bytes(int batch, int num_heads, int num_kv_heads,
                                                      int head_dim, int max_blocks_per_seq,
                                                      int partition_blocks) {
  const int64_t parts =
      split_parts(batch, num_heads, num_kv_heads, head_dim, max_blocks_per_seq, partition_blocks);
  const int64_t slots = (int64_t)batch * num_heads * parts;
  size_t bytes = attn::kCounterBytes;                           // arrival counters (kept zero)
  bytes += (size_t)slots * head_dim * 4;                        // ws_o
  bytes += (size_t)slots * 2 * 4;                               // ws_ml
  bytes += (size_t)batch * num_kv_heads * parts * 4;            // ws_stop
  bytes += (size_t)batch * num_kv_heads * 4;                    // ws_pieces
  return bytes + 256;
}

// CTAs of the v5 kernel and of its plan for a batch of this shape, 0 when v5 cannot take it:
// the largest chunk any batch of the shape can get (the piece floor at 17 pieces is the larger
// one) must fit a CTA's id window.  Batches of at most kV5SmallBatch sequences run on half the
// SMs when that still fits: in a decode step the QKV GEMM before the attention holds the other
// half (72 CTAs at these batch sizes), so every attention CTA becomes resident while the GEMM
// runs and streams its first blocks early (TI_ATTN_EARLY_KV), instead of the half behind the
// GEMM starting only when it ends and setting the launch's length.
static int v5_ctas(int batch, int num_kv_heads, int max_blocks) {
  const int64_t worst = (int64_t)batch * (num_kv_heads / 2) * max_blocks;
  auto fits = [&](int ctas) {
    return (int64_t)attn::v2_chunk(worst, ctas * attn::kV5Pairs, max_blocks, attn::kV2MaxPieces) *
               attn::kV5Pairs <= attn::kV5IdCap;
  };
  const int sms = attn::sm_count();
#ifndef TI_V5_HALF_MAX_BATCH
#define TI_V5_HALF_MAX_BATCH attn::kV5SmallBatch
#endif
  if (batch <= TI_V5_HALF_MAX_BATCH && fits(sms / 2)) return sms / 2;
  return fits(sms) ? sms : 0;
}

// Whether a decode call of this shape runs the v5 kernel (and can use a plan).
static bool v5_path(int batch, int num_heads, int num_kv_heads, int head_dim, int max_blocks) {
  if (!attn::use_v2(head_dim, batch) || num_kv_heads <= 0 || num_heads % num_kv_heads) return false;
  if (unit_path(batch, num_heads, num_kv_heads, head_dim, max_blocks)) return false;
  if (num_kv_heads % 2 || num_heads / num_kv_heads > 8 || max_blocks <= 0) return false;
  const int forced = attn::forced_kernel();
  if (forced != 0 && forced != 5) return false;
  if (batch > attn::CfgV5::kMaxBatch) return false;
  return v5_ctas(batch, num_kv_heads, max_blocks) > 0;
}

static int decode_impl(
    void* out, int64_t out_seq_stride, const void* q, int64_t q_seq_stride, const void* k_cache,
    const void* v_cache, int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
    const int32_t* row_index, const int32_t* context_lens, int batch, int num_heads,
    int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq, int dtype,
    int partition_blocks, void* workspace, size_t workspace_bytes, void* stream,
    const int32_t* plan, int flags = 0) {
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
  // the split limit and the workspace follow the caller's partition argument (0: the default,
  // under which small v5 batches are cut finer), exactly as ti_paged_attention_workspace_bytes
  // and ti_paged_attention_plan see it
  const int req_partition = partition_blocks;
  if (partition_blocks <= 0) partition_blocks = attn::default_partition(max_blocks_per_seq);
  if (partition_blocks > attn::kMaxPart)
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: partition_blocks must be <= 16");
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: pool base must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (q_seq_stride & 1) ||
      (reinterpret_cast<uintptr_t>(out) & 3) || (out_seq_stride & 1))
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: q/out must be 4-byte aligned with even row strides");
  const bool v2 = attn::use_v2(head_dim, batch);
  const int max_parts = (int)split_parts(batch, num_heads, num_kv_heads, head_dim,
                                         max_blocks_per_seq, req_partition);
  const size_t need = ti_paged_attention_workspace_bytes(batch, num_heads, num_kv_heads, head_dim,
                                                          max_blocks_per_seq, req_partition);
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
    p.ws_pieces = p.ws_stop + (int64_t)batch * num_kv_heads * max_parts;
  }
  const int64_t rows = num_blocks * num_kv_heads * attn::kBlock;
  // two kv heads per MMA tile when both GQA groups fit the 16 rows
  const int hp = (v2 && num_kv_heads % 2 == 0 && p.group <= 8) ? 2 : 1;
  CUtensorMap km, vm;
  int rc = attn::kv_tensor_map(&km, k_cache, rows, head_dim, dtype, hp * attn::kBlock);
  if (rc) return rc;
  rc = attn::kv_tensor_map(&vm, v_cache, rows, head_dim, dtype, hp * attn::kBlock);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (req_partition <= 0 &&
      unit_path(batch, num_heads, num_kv_heads, head_dim, max_blocks_per_seq)) {
    // short sequences: one CTA per unit, no split (a plan, if given, is not read)
    const int units = batch * (num_kv_heads / 2);
    return dtype == TI_DTYPE_BF16 ? attn::launch_unit<__nv_bfloat16>(p, km, vm, units, s)
                                  : attn::launch_unit<__half>(p, km, vm, units, s);
  }
  if (v2) {
    // v4 needs its CTA's whole stream range in shared memory: check the worst case here
    static int sms = 0;
    if (!sms) {
      int dev = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (sms <= 0) sms = 148;
    }
    const int64_t worst = (int64_t)batch * (num_kv_heads / hp) * max_blocks_per_seq;
    const int forced = attn::forced_kernel();
    if (v5_path(batch, num_heads, num_kv_heads, head_dim, max_blocks_per_seq)) {
      p.plan = plan;
      p.early = plan && (flags & TI_ATTN_EARLY_KV) ? 1 : 0;
      const int ctas = v5_ctas(batch, num_kv_heads, max_blocks_per_seq);
      if (plan)
        return dtype == TI_DTYPE_BF16
                   ? attn::launch_v5<__nv_bfloat16, true>(p, km, vm, batch, ctas, s)
                   : attn::launch_v5<__half, true>(p, km, vm, batch, ctas, s);
      return dtype == TI_DTYPE_BF16 ? attn::launch_v5<__nv_bfloat16, false>(p, km, vm, batch, ctas, s)
                                    : attn::launch_v5<__half, false>(p, km, vm, batch, ctas, s);
    }
    const int64_t chunk_ub = attn::v2_chunk(worst, sms * attn::kV4Warps, max_blocks_per_seq,
                                            max_parts);
    if (p.group <= 8 && forced != 2 && chunk_ub * attn::kV4Warps <= attn::kV4IdCap) {
      if (hp == 2)
        return dtype == TI_DTYPE_BF16 ? attn::launch_v4<__nv_bfloat16, 2>(p, km, vm, batch, s)
                                      : attn::launch_v4<__half, 2>(p, km, vm, batch, s);
      return dtype == TI_DTYPE_BF16 ? attn::launch_v4<__nv_bfloat16, 1>(p, km, vm, batch, s)
                                    : attn::launch_v4<__half, 1>(p, km, vm, batch, s);
    }
  }
  if (v2 && hp == 2)
    return dtype == TI_DTYPE_BF16 ? attn::launch_v2<__nv_bfloat16, 2>(p, km, vm, batch, s)
                                  : attn::launch_v2<__half, 2>(p, km, vm, batch, s);
  if (v2)
    return dtype == TI_DTYPE_BF16 ? attn::launch_v2<__nv_bfloat16, 1>(p, km, vm, batch, s)
                                  : attn::launch_v2<__half, 1>(p, km, vm, batch, s);
  if (dtype == TI_DTYPE_BF16)
    return head_dim == 64 ? attn::launch<__nv_bfloat16, 64>(p, km, vm, batch, s)
                          : attn::launch<__nv_bfloat16, 128>(p, km, vm, batch, s);
  return head_dim == 64 ? attn::launch<__half, 64>(p, km, vm, batch, s)
                        : attn::launch<__half, 128>(p, km, vm, batch, s);
}

extern "C" int ti_paged_attention_decode(
    void* out, int64_t out_seq_stride, const void* q, int64_t q_seq_stride, const void* k_cache,
    const void* v_cache, int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
    const int32_t* row_index, const int32_t* context_lens, int batch, int num_heads,
    int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq, int dtype,
    int partition_blocks, void* workspace, size_t workspace_bytes, void* stream) {
  return decode_impl(out, out_seq_stride, q, q_seq_stride, k_cache, v_cache, num_blocks,
                     block_tables, bt_stride, row_index, context_lens, batch, num_heads,
                     num_kv_heads, head_dim, block_size, max_blocks_per_seq, dtype,
                     partition_blocks, workspace, workspace_bytes, stream, nullptr);
}

extern "C" size_t ti_paged_attention_plan_bytes(int batch) {
  return batch < 0 ? 0 : attn::plan_bytes(batch, attn::sm_count());
}

// How long the QKV GEMM before a decode step's attention keeps its SMs after the attention
// grid launched (in-kernel traces at 32-256 rows: ~6 us); the skewed plan uses it.
#ifndef TI_QKV_LEAD_US
#define TI_QKV_LEAD_US 6.f
#endif
constexpr float kQkvLeadUs = TI_QKV_LEAD_US;

static int plan_impl(const int32_t* block_tables, int64_t bt_stride, const int32_t* row_index,
                     const int32_t* context_lens, int batch, int num_heads, int num_kv_heads,
                     int head_dim, int max_blocks_per_seq, int64_t num_blocks, void* plan,
                     size_t plan_bytes, int flags, int qkv_hidden, int dtype, void* stream) {
  clear_error();
  if (batch == 0) return TI_OK;
  if (!block_tables || !context_lens || !plan)
    return set_error(TI_ERR_INVALID_ARGUMENT, "attention plan: null pointer");
  if (batch < 0 || num_blocks <= 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "attention plan: negative batch or empty pool");
  if (reinterpret_cast<uintptr_t>(plan) & 15)
    return set_error(TI_ERR_INVALID_ARGUMENT, "attention plan: buffer must be 16-byte aligned");
  if (flags & ~TI_ATTN_PLAN_AFTER_QKV)
    return set_error(TI_ERR_INVALID_ARGUMENT, "attention plan: unknown flags");
  if (!v5_path(batch, num_heads, num_kv_heads, head_dim, max_blocks_per_seq)) {
    // the planned decode takes the unplanned path for this shape (a zero header: chunk 0)
    if (plan_bytes < 32)
      return set_error(TI_ERR_WORKSPACE, "attention plan: buffer too small");
    cudaError_t e = cudaMemsetAsync(plan, 0, 32, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TI_OK : set_cuda_error(e, "attention plan header");
  }
  if (plan_bytes < ti_paged_attention_plan_bytes(batch))
    return set_error(TI_ERR_WORKSPACE, "attention plan: buffer too small");
  attn::Params p{};
  p.block_tables = block_tables; p.bt_stride = bt_stride; p.row_index = row_index;
  p.context_lens = context_lens;
  p.num_heads = num_heads; p.num_kv_heads = num_kv_heads; p.group = num_heads / num_kv_heads;
  p.max_blocks = max_blocks_per_seq; p.num_blocks = num_blocks;
  p.max_parts = (int)split_parts(batch, num_heads, num_kv_heads, head_dim, max_blocks_per_seq, 0);
  const int ctas = v5_ctas(batch, num_kv_heads, max_blocks_per_seq);
  if ((flags & TI_ATTN_PLAN_AFTER_QKV) && qkv_hidden > 0 && ctas == attn::sm_count()) {
    // the QKV GEMM of these rows holds gemm_qkv_ctas SMs when the attention grid launches
    const int held = gemm_qkv_ctas(batch, (num_heads + 2 * num_kv_heads) * head_dim, qkv_hidden,
                                   dtype);
    if (held > 0 && held < ctas) {
      p.skew_full = ctas - held;
      p.skew_lead_us = kQkvLeadUs;
    }
  }
  return launch_kernel("attention plan launch", attn::plan_kernel<512>, dim3(ctas), dim3(512), 0,
                       reinterpret_cast<cudaStream_t>(stream), 1, p, batch,
                       reinterpret_cast<int32_t*>(plan));
}

extern "C" int ti_paged_attention_plan(const int32_t* block_tables, int64_t bt_stride,
                                       const int32_t* row_index, const int32_t* context_lens,
                                       int batch, int num_heads, int num_kv_heads, int head_dim,
                                       int max_blocks_per_seq, int64_t num_blocks, void* plan,
                                       size_t plan_bytes, void* stream) {
  return plan_impl(block_tables, bt_stride, row_index, context_lens, batch, num_heads,
                   num_kv_heads, head_dim, max_blocks_per_seq, num_blocks, plan, plan_bytes, 0, 0,
                   TI_DTYPE_BF16, stream);
}

extern "C" int ti_paged_attention_plan_ex(const int32_t* block_tables, int64_t bt_stride,
                                          const int32_t* row_index, const int32_t* context_lens,
                                          int batch, int num_heads, int num_kv_heads,
                                          int head_dim, int max_blocks_per_seq,
                                          int64_t num_blocks, void* plan, size_t plan_bytes,
                                          int flags, int qkv_hidden, int dtype, void* stream) {
  return plan_impl(block_tables, bt_stride, row_index, context_lens, batch, num_heads,
                   num_kv_heads, head_dim, max_blocks_per_seq, num_blocks, plan, plan_bytes, flags,
                   qkv_hidden, dtype, stream);
}

extern "C" int ti_paged_attention_decode_planned_ex(
    void* out, int64_t out_seq_stride, const void* q, int64_t q_seq_stride, const void* k_cache,
    const void* v_cache, int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
    const int32_t* row_index, const int32_t* context_lens, int batch, int num_heads,
    int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq, int dtype,
    void* workspace, size_t workspace_bytes, const void* plan, int flags, void* stream) {
  if (!plan) {
    clear_error();
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: null plan");
  }
  if (reinterpret_cast<uintptr_t>(plan) & 15) {
    clear_error();
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: plan must be 16-byte aligned");
  }
  if (flags & ~TI_ATTN_EARLY_KV) {
    clear_error();
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention: unknown flags");
  }
  return decode_impl(out, out_seq_stride, q, q_seq_stride, k_cache, v_cache, num_blocks,
                     block_tables, bt_stride, row_index, context_lens, batch, num_heads,
                     num_kv_heads, head_dim, block_size, max_blocks_per_seq, dtype, 0, workspace,
                     workspace_bytes, stream, reinterpret_cast<const int32_t*>(plan), flags);
}

extern "C" int ti_paged_attention_decode_planned(
    void* out, int64_t out_seq_stride, const void* q, int64_t q_seq_stride, const void* k_cache,
    const void* v_cache, int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
    const int32_t* row_index, const int32_t* context_lens, int batch, int num_heads,
    int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq, int dtype,
    void* workspace, size_t workspace_bytes, const void* plan, void* stream) {
  return ti_paged_attention_decode_planned_ex(
      out, out_seq_stride, q, q_seq_stride, k_cache, v_cache, num_blocks, block_tables, bt_stride,
      row_index, context_lens, batch, num_heads, num_kv_heads, head_dim, block_size,
      max_blocks_per_seq, dtype, workspace, workspace_bytes, plan, 0, stream);
}
