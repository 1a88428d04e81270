// Device sampler: temperature, top-k, top-p and the draw of the reference's
// ContinuousBatcher._sample_next_token (engine/scheduler.py:104-156), one CTA per row, with no
// sort of the vocabulary.
//
// The reference divides the row by its temperature (0 -> 1; here: multiplies by 1/t in fp32),
// keeps values >= a cutoff that is the max_k-th largest value for rows whose top_k equals the
// batch's largest top_k and -inf for the others (:119-130), then -- when any row has p < 1 --
// removes the tail of the descending order after the first token whose cumulative softmax
// probability exceeds p (:133-146), and finally draws from the softmax of what is left, or
// takes the argmax for temperature 0 (:149-155).  The batch-level rules are resolved on the
// host into a per-row cut rank (0: no cut) and p (>= 1: no top-p).
//
// Here every "position in the descending order" question is answered by a radix select over
// order-preserving 32-bit keys of the fp32 values (4 passes of 8-bit digits over the row):
//   * top-k cutoff: the max_k-th largest key (counts);
//   * top-p boundary and the draw: the first element of the descending order whose cumulative
//     weight exceeds a target, weights exp(x - max) in 32.32 fixed point (integer sums: the
//     result does not depend on the order of the additions); elements with equal values are
//     ordered by ascending index (a final pass scans the tied elements in index order).
// The draw uses a caller-provided uniform u in [0, 1): the token is the first one, in
// descending order, whose cumulative kept weight exceeds u * (total kept weight).
//
// Rows with a top-k cut of at most 512 (the common case) take a faster route to the same
// answers: the k-th largest of the 512 threads' maxima bounds the row's k-th largest value from
// below (those k maxima are k elements at least that large), so one more pass compacts every
// element at or above it into shared memory; the candidates are sorted (value descending, index
// ascending) and the cutoff, the top-p boundary and the draw are read off their prefix sums of
// the same fixed-point weights.  When more than kCand elements reach the bound (ties), the row
// falls back to the radix selects, whose histograms are per warp.
#include <algorithm>
#include <type_traits>

#include "capi_internal.h"
#include "common.cuh"

namespace ti {
namespace smp {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 256;
constexpr int kCand = 4096;        // compacted top-k candidates (power of two)

__device__ __forceinline__ uint32_t f2key(float x) {   // order-preserving: larger x, larger key
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct Shared {
  union {
    unsigned long long hist[kWarps][kBins];   // radix selects: one histogram per warp
    unsigned long long cand[kCand];           // fast path: (key << 32) | ~index, then weights
  };
  unsigned long long bin_sum[kBins];
  float tmax[kThreads];
  int cand_n;
  unsigned long long scan[kWarps];
  float red_v[kWarps];
  int red_i[kWarps];
  uint32_t sel_key;
  unsigned long long sel_acc;    // weight of the elements above the selected bucket
  int sel_found;
  int sel_index;
  unsigned long long sel_cum;    // cumulative weight up to and including the selected element
};

// A row of logits scaled by 1 / temperature (temperature 0 -> 1): the value every pass sees.
template <typename T>
struct Row {
  const T* p;
  float inv_t;
  __device__ __forceinline__ float x(int j) const {
    float v;
    if constexpr (std::is_same<T, float>::value) v = p[j];
    else v = Elem<T>::to_f(p[j]);
    return v * inv_t;
  }
};

// f(x, j) for every element j of the row, in no particular order: 16-byte loads, U of them in
// flight per thread (the scalar strided loop was load-latency bound); rows whose start is not
// 16-byte aligned, and the tail, go element by element.
template <typename T, typename F>
__device__ __forceinline__ void row_scan(const Row<T>& row, int V, F&& f) {
  constexpr int kVec = 16 / (int)sizeof(T);
  constexpr int U = 8;
  const int nvec = (reinterpret_cast<uintptr_t>(row.p) & 15) == 0 ? V / kVec : 0;
  const uint4* pv = reinterpret_cast<const uint4*>(row.p);
  int v = threadIdx.x;
  for (; v + (U - 1) * kThreads < nvec; v += U * kThreads) {
    uint4 buf[U];
#pragma unroll
    for (int u = 0; u < U; ++u) buf[u] = __ldg(pv + v + u * kThreads);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const T* e = reinterpret_cast<const T*>(&buf[u]);
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        float x;
        if constexpr (std::is_same<T, float>::value) x = e[i];
        else x = Elem<T>::to_f(e[i]);
        f(x * row.inv_t, (v + u * kThreads) * kVec + i);
      }
    }
  }
  for (; v < nvec; v += kThreads) {
    const uint4 b = __ldg(pv + v);
    const T* e = reinterpret_cast<const T*>(&b);
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      float x;
      if constexpr (std::is_same<T, float>::value) x = e[i];
      else x = Elem<T>::to_f(e[i]);
      f(x * row.inv_t, v * kVec + i);
    }
  }
  for (int j = nvec * kVec + (int)threadIdx.x; j < V; j += kThreads) f(row.x(j), j);
}

// The same walk over 16-bit rows a vector at a time: fv(b, j0) gets each aligned 16-byte vector
// (8 raw elements, first index j0), fs(x, j) the raw elements of an unaligned row and of the
// tail; a thread sees its vectors in increasing index order, then its tail elements.  The passes use it to test a whole
// vector with a few packed instructions (its maximum) and look at single elements only in the
// rare vectors that can matter: the per-element work was what bounded them.
template <typename T, typename FV, typename FS>
__device__ __forceinline__ void row_scan_vec(const Row<T>& row, int V, FV&& fv, FS&& fs) {
  static_assert(sizeof(T) == 2, "16-bit rows");
  constexpr int U = 8;
  const int nvec = (reinterpret_cast<uintptr_t>(row.p) & 15) == 0 ? V / 8 : 0;
  const uint4* pv = reinterpret_cast<const uint4*>(row.p);
  int v = threadIdx.x;
  for (; v + (U - 1) * kThreads < nvec; v += U * kThreads) {
    uint4 buf[U];
#pragma unroll
    for (int u = 0; u < U; ++u) buf[u] = __ldg(pv + v + u * kThreads);
#pragma unroll
    for (int u = 0; u < U; ++u) fv(buf[u], (v + u * kThreads) * 8);
  }
  for (; v < nvec; v += kThreads) fv(__ldg(pv + v), v * 8);
  for (int j = nvec * 8 + (int)threadIdx.x; j < V; j += kThreads) fs(Elem<T>::to_f(row.p[j]), j);
}

// Largest of a 16-byte vector's 8 elements: NaN-ignoring (a number wins over NaN) or, with
// PROPAGATE = true, NaN when any element is NaN.
template <typename T, bool PROPAGATE>
__device__ __forceinline__ float vec_max(const uint4& b) {
  using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
  const T2* h = reinterpret_cast<const T2*>(&b);
  T2 a, c;
  if constexpr (PROPAGATE) {
    a = __hmax2_nan(h[0], h[1]);
    c = __hmax2_nan(h[2], h[3]);
    a = __hmax2_nan(a, c);
  } else {
    a = __hmax2(h[0], h[1]);
    c = __hmax2(h[2], h[3]);
    a = __hmax2(a, c);
  }
  const float lo = Elem<T>::to_f(a.x), hi = Elem<T>::to_f(a.y);
  if constexpr (PROPAGATE) return (lo != lo || hi != hi) ? lo + hi : fmaxf(lo, hi);
  else return fmaxf(lo, hi);
}

// Weight of element with value x in 32.32 fixed point (exp(x - m), x <= m), 0 when not a
// candidate.
__device__ __forceinline__ unsigned long long weight(float x, float m) {
  const float w = __expf(x - m);
  return (unsigned long long)(w * 4294967296.0f);
}

// Find, among the elements with key >= lowkey, the first element of the descending order
// (ties: ascending index) whose cumulative weight exceeds `target` (COUNT: every weight is 1).
// Results in sh.sel_*: sel_found, sel_key, sel_index, sel_cum.  With SKIP_TIES only the key
// is resolved (sel_index = -1).
template <typename T, bool COUNT, bool SKIP_TIES>
__device__ void select_first_exceeding(Shared& sh, const Row<T>& row, int V, uint32_t lowkey,
                                       float m, unsigned long long target) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, pmask = 0;
  unsigned long long acc = 0;
  bool found = true;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < kWarps * kBins; b += kThreads) (&sh.hist[0][0])[b] = 0ull;
    __syncthreads();
    row_scan(row, V, [&](float x, int) {
      const uint32_t k = f2key(x);
      if (k < lowkey || (k & pmask) != prefix) return;
      atomicAdd(&sh.hist[warp][(k >> shift) & 255u], COUNT ? 1ull : weight(x, m));
    });
    __syncthreads();
    for (int b = tid; b < kBins; b += kThreads) {
      unsigned long long t = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += sh.hist[w][b];
      sh.bin_sum[b] = t;
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255 - 8l ... 248 - 8l (descending); suffix sums in that order
      unsigned long long own[8], s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) { own[i] = sh.bin_sum[255 - 8 * lane - i]; s += own[i]; }
      unsigned long long before = s;                 // inclusive scan over lanes
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(0xffffffffu, before, o);
        if (lane >= o) before += v;
      }
      before -= s;                                   // exclusive: weight of higher bins
      const bool here = acc + before <= target && acc + before + s > target;
      const unsigned ball = __ballot_sync(0xffffffffu, here);
      if (ball == 0) {
        if (lane == 0) sh.sel_found = 0;
      } else if (lane == __ffs(ball) - 1) {
        unsigned long long run = acc + before;
        int bin = 255 - 8 * lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (run + own[i] > target) { bin = 255 - 8 * lane - i; break; }
          run += own[i];
        }
        sh.sel_found = 1;
        sh.sel_key = (uint32_t)bin;
        sh.sel_acc = run;
      }
    }
    __syncthreads();
    if (!sh.sel_found) { found = false; break; }
    prefix |= sh.sel_key << shift;
    pmask |= 255u << shift;
    acc = sh.sel_acc;
    __syncthreads();
  }
  if (!found) {
    if (tid == 0) sh.sel_found = 0;
    __syncthreads();
    return;
  }
  if (SKIP_TIES) {
    if (tid == 0) { sh.sel_found = 1; sh.sel_key = prefix; sh.sel_index = -1; sh.sel_acc = acc; }
    __syncthreads();
    return;
  }
  // elements with key == prefix, in index order: thread t owns a contiguous index range
  if (tid == 0) sh.sel_index = -1;
  __syncthreads();
  const int chunk = (V + kThreads - 1) / kThreads;
  const int j0 = min(V, tid * chunk), j1 = min(V, j0 + chunk);
  unsigned long long mine = 0;
  for (int j = j0; j < j1; ++j) {
    const float x = row.x(j);
    if (f2key(x) == prefix) mine += COUNT ? 1ull : weight(x, m);
  }
  unsigned long long incl = mine;   // block-wide inclusive scan in thread order
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) sh.scan[warp] = incl;
  __syncthreads();
  unsigned long long wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += sh.scan[w];
  const unsigned long long excl = acc + wbase + incl - mine;
  if (excl <= target && excl + mine > target) {
    unsigned long long run = excl;
    for (int j = j0; j < j1; ++j) {
      const float x = row.x(j);
      if (f2key(x) != prefix) continue;
      run += COUNT ? 1ull : weight(x, m);
      if (run > target) {
        sh.sel_index = j;
        sh.sel_cum = run;
        break;
      }
    }
    sh.sel_key = prefix;
    sh.sel_found = 1;
  }
  __syncthreads();
}


// Bitonic sort of sh.cand[0 .. n2) in descending order (n2 a power of two, at most kCand); all
// threads of the CTA take part.
__device__ void sort_desc(Shared& sh, int n2) {
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n2 / 2; i += kThreads) {
        const int a = 2 * i - (i & (stride - 1)), b = a + stride;
        const bool desc = (a & size) == 0;
        const unsigned long long x = sh.cand[a], y = sh.cand[b];
        if ((x < y) == desc) { sh.cand[a] = y; sh.cand[b] = x; }
      }
      __syncthreads();
    }
  }
}

// Top-k fast path (1 <= k <= kThreads): returns false (uniformly) when more than kCand elements
// reach the bound, leaving the row to the radix selects; otherwise sets `token` exactly as they
// would.  sh.tmax holds each thread's maximum of the scaled row.
template <typename T>
__device__ bool topk_fast(Shared& sh, const Row<T>& row, int V, int k, float m, float p, float u,
                          int& token) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the k-th largest thread maximum: a lower bound of the row's k-th largest value
  sh.cand[tid] = ((unsigned long long)f2key(sh.tmax[tid]) << 32) | (uint32_t)tid;
  if (tid == 0) sh.cand_n = 0;
  __syncthreads();
  sort_desc(sh, kThreads);
  const uint32_t bound = (uint32_t)(sh.cand[k - 1] >> 32);
  __syncthreads();
  // compact the elements at or above the bound: (key << 32) | ~index
  auto keep = [&](float x, int j) {   // few elements pass: one shared atomic each
    const uint32_t key = f2key(x);
    if (key < bound) return;
    const int slot = atomicAdd(&sh.cand_n, 1);
    if (slot < kCand) sh.cand[slot] = ((unsigned long long)key << 32) | (uint32_t)~(uint32_t)j;
  };
  bool scanned = false;
  if constexpr (sizeof(T) == 2) {
    if (row.inv_t > 0.f) {
      // an element's key reaches the bound only if its scaled value is not below the bound's
      // value, so a vector whose scaled maximum is below it holds none (the maximum propagates
      // NaN: such vectors take the exact per-element test)
      const float thr = key2f(bound);
      row_scan_vec(row, V, [&](const uint4& b, int j0) {
        if (vec_max<T, true>(b) * row.inv_t < thr) return;
        const T* e = reinterpret_cast<const T*>(&b);
#pragma unroll
        for (int i = 0; i < 8; ++i) keep(Elem<T>::to_f(e[i]) * row.inv_t, j0 + i);
      }, [&](float x, int j) { keep(x * row.inv_t, j); });
      scanned = true;
    }
  }
  if (!scanned) row_scan(row, V, keep);
  __syncthreads();
  const int n = sh.cand_n;
  if (n > kCand) return false;
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int i = n + tid; i < n2; i += kThreads) sh.cand[i] = 0ull;   // sorts last
  __syncthreads();
  sort_desc(sh, n2);
  // kept: the leading entries with key >= the k-th largest key (k <= n)
  const uint32_t cut = (uint32_t)(sh.cand[k - 1] >> 32);
  constexpr int E = kCand / kThreads;
  unsigned long long w[E], mine = 0;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = tid * E + e;
    w[e] = 0ull;
    if (i < n) {
      const uint32_t key = (uint32_t)(sh.cand[i] >> 32);
      if (key >= cut) w[e] = weight(key2f(key), m);
    }
    mine += w[e];
  }
  unsigned long long incl = mine;   // block-wide scan in thread (= descending) order
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) sh.scan[warp] = incl;
  __syncthreads();
  unsigned long long wbase = 0, Z = 0;
  for (int q = 0; q < kWarps; ++q) {
    if (q < warp) wbase += sh.scan[q];
    Z += sh.scan[q];
  }
  const unsigned long long excl = wbase + incl - mine;
  // first kept entry whose cumulative weight exceeds `target` -> its cumulative weight / index
  auto find = [&](unsigned long long target, bool want_index) {
    if (tid == 0) sh.sel_found = 0;
    __syncthreads();
    if (excl <= target && excl + mine > target) {
      unsigned long long run = excl;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        run += w[e];
        if (run > target) {
          sh.sel_found = 1;
          sh.sel_cum = run;
          sh.sel_index = want_index ? (int)~(uint32_t)(sh.cand[tid * E + e] & 0xffffffffull) : -1;
          break;
        }
      }
    }
    __syncthreads();
  };
  unsigned long long zk = Z;
  if (p < 1.f) {
    const double tgt = (double)p * (double)Z;
    if (tgt < (double)Z) {
      find(tgt <= 0.0 ? 0ull : (unsigned long long)tgt, false);
      if (sh.sel_found) zk = sh.sel_cum;
    }
  }
  find((unsigned long long)((double)u * (double)zk), true);
  if (sh.sel_found && sh.sel_index >= 0) token = sh.sel_index;
  return true;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
sample_kernel(const T* __restrict__ logits, int64_t ld, int V, const float* __restrict__ temps,
              const int32_t* __restrict__ cut_ks, const float* __restrict__ top_ps,
              const float* __restrict__ uniforms, int32_t* __restrict__ out,
              const int32_t* __restrict__ slots, int32_t* seq_len, int inc) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ Shared sh;
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float temp = temps[r];
  Row<T> row;
  row.p = logits + (int64_t)r * ld;
  row.inv_t = temp == 0.f ? 1.f : 1.f / temp;

  // ---- max and first argmax
  float best = -INFINITY;
  int bi = 0x7fffffff;
  auto take = [&](float x, int j) {
    if (x > best || (x == best && j < bi)) { best = x; bi = j; }
  };
  if constexpr (sizeof(T) == 2) {
    if (row.inv_t > 0.f) {
      // raw values: a positive scale keeps the order (and rounds monotonically), so the scaled
      // maximum is the raw one scaled and the first index of either is the same for scale 1
      // (greedy rows, the only ones that use it); a thread's vectors come in increasing index
      // order, so a vector whose maximum only ties the thread's best holds no earlier index
      float braw = -INFINITY;
      row_scan_vec(row, V, [&](const uint4& b, int j0) {
        const float vm = vec_max<T, false>(b);
        if (vm > braw) {
          const T* e = reinterpret_cast<const T*>(&b);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (Elem<T>::to_f(e[i]) == vm) { braw = vm; bi = j0 + i; break; }
        }
      }, [&](float x, int j) {
        if (x > braw) { braw = x; bi = j; }
      });
      best = braw * row.inv_t;
    } else {
      row_scan(row, V, take);
    }
  } else {
    row_scan(row, V, take);
  }
  sh.tmax[tid] = best;   // this thread's maximum (top-k fast path)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, best, o);
    const int i = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
  if (lane == 0) { sh.red_v[warp] = best; sh.red_i[warp] = bi; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kWarps; ++w)
      if (sh.red_v[w] > sh.red_v[0] || (sh.red_v[w] == sh.red_v[0] && sh.red_i[w] < sh.red_i[0])) {
        sh.red_v[0] = sh.red_v[w];
        sh.red_i[0] = sh.red_i[w];
      }
  }
  __syncthreads();
  const float m = sh.red_v[0];
  int token = sh.red_i[0] == 0x7fffffff ? 0 : sh.red_i[0];   // an all-NaN row yields 0

  const int k = temp != 0.f && m > -INFINITY ? cut_ks[r] : 0;
  const float u = fminf(fmaxf(uniforms[r], 0.f), 0.99999994f);
  bool fast = false;
  if (k > 0 && k <= kThreads && k < V) fast = topk_fast<T>(sh, row, V, k, m, top_ps[r], u, token);
  if (temp != 0.f && m > -INFINITY && !fast) {
    // ---- top-k cutoff: keep x >= the k-th largest value (k = 0: keep everything)
    uint32_t lowkey = 0;
    if (k > 0 && k < V) {
      select_first_exceeding<T, true, true>(sh, row, V, 0u, m, (unsigned long long)(k - 1));
      if (sh.sel_found) lowkey = sh.sel_key;       // keep x >= the k-th largest value
    }
    // ---- total weight of the candidates
    unsigned long long z = 0;
    row_scan(row, V, [&](float x, int) {
      if (f2key(x) >= lowkey) z += weight(x, m);
    });
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    if (lane == 0) sh.scan[warp] = z;
    __syncthreads();
    unsigned long long Z = 0;
    for (int w = 0; w < kWarps; ++w) Z += sh.scan[w];
    __syncthreads();
    // ---- top-p: kept = the descending prefix up to the first element whose cumulative
    //      weight exceeds p * Z (the first element is always kept)
    unsigned long long zk = Z;
    const float p = top_ps[r];
    if (p < 1.f) {
      const double tgt = (double)p * (double)Z;
      if (tgt < (double)Z) {
        const unsigned long long target = tgt <= 0.0 ? 0ull : (unsigned long long)tgt;
        select_first_exceeding<T, false, false>(sh, row, V, lowkey, m, target);
        if (sh.sel_found) zk = sh.sel_cum;
      }
    }
    // ---- the draw: first element whose cumulative weight exceeds u * zk
    const unsigned long long t2 = (unsigned long long)((double)u * (double)zk);
    select_first_exceeding<T, false, false>(sh, row, V, lowkey, m, t2);
    if (sh.sel_found && sh.sel_index >= 0) token = sh.sel_index;
  }
  if (tid == 0) {
    out[r] = token;
    if (slots && seq_len) {
      const int s = slots[r];
      if (s >= 0) seq_len[s] += inc;
    }
  }
}

}  // namespace smp
}  // namespace ti

using namespace ti;

extern "C" int ti_sample(const void* logits, int64_t ld, int dtype, int rows, int vocab,
                         const float* temperatures, const int32_t* cut_ks, const float* top_ps,
                         const float* uniforms, int32_t* out_tokens, const int32_t* slots,
                         int32_t* seq_len, int seq_inc, void* stream) {
  clear_error();
  if (rows == 0) return TI_OK;
  if (!logits || !temperatures || !cut_ks || !top_ps || !uniforms || !out_tokens || rows < 0 ||
      vocab <= 0 || ld < vocab)
    return set_error(TI_ERR_INVALID_ARGUMENT, "sample: null pointer or bad size");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == TI_DTYPE_BF16)
    return launch_kernel("sample launch", smp::sample_kernel<__nv_bfloat16>, dim3(rows),
                         dim3(smp::kThreads), 0, s, 1, (const __nv_bfloat16*)logits, ld, vocab,
                         temperatures, cut_ks, top_ps, uniforms, out_tokens, slots, seq_len,
                         seq_inc);
  if (dtype == TI_DTYPE_FP16)
    return launch_kernel("sample launch", smp::sample_kernel<__half>, dim3(rows),
                         dim3(smp::kThreads), 0, s, 1, (const __half*)logits, ld, vocab,
                         temperatures, cut_ks, top_ps, uniforms, out_tokens, slots, seq_len,
                         seq_inc);
  if (dtype == TI_DTYPE_FP32)
    return launch_kernel("sample launch", smp::sample_kernel<float>, dim3(rows),
                         dim3(smp::kThreads), 0, s, 1, (const float*)logits, ld, vocab,
                         temperatures, cut_ks, top_ps, uniforms, out_tokens, slots, seq_len,
                         seq_inc);
  return set_error(TI_ERR_UNSUPPORTED, "sample: dtype must be bf16, fp16 or fp32");
}
