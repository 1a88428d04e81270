// Exact int8 -> bf16 / fp16 conversion of weight tiles, for the weight-only int8 lm_head
// kernels: a whole tile into a 16-bit shared-memory tile (lmhead_i8.cu), or one row per thread
// into registers for tensor memory (gemv.cu).
//
// convert_int8_tile -- input: a 128-row x 64-byte int8 tile as TMA writes it without swizzle
// (row pitch 64 bytes); output: the same 128 x 64 values as 16-bit elements in the canonical
// SWIZZLE_128B K-major layout the tcgen05 shared-memory descriptors read (128-byte rows,
// 1024-byte aligned base).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"

namespace ti {

// 8 int8 values (two 32-bit words) -> 8 elements of T packed as four 32-bit words, exactly and
// with full-rate integer / float ops only (a per-element int -> float conversion instruction runs
// on the slow conversion unit and made the converters the bottleneck).  u = byte ^ 0x80 is the
// value + 128; bf16: the float32 with bits 0x4B000000 | u is 2^23 + u, minus 2^23 + 128 it is the
// value, and a small integer's float32 has zero low 16 bits, so its high half is the bf16;
// fp16: the half with bits 0x6400 | u is 1024 + u, minus 1152 (one packed subtraction).
template <typename T>
__device__ __forceinline__ uint4 convert8(uint32_t lo, uint32_t hi) {
  uint32_t o[4];
  const uint32_t w[2] = {lo ^ 0x80808080u, hi ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      float f[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        f[j] = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7540u | j)) - 8388736.0f;
      o[2 * i] = __byte_perm(__float_as_uint(f[0]), __float_as_uint(f[1]), 0x7632u);
      o[2 * i + 1] = __byte_perm(__float_as_uint(f[2]), __float_as_uint(f[3]), 0x7632u);
    } else {
      const __half2 bias = __halves2half2(__float2half(1152.f), __float2half(1152.f));
      const uint32_t a = __byte_perm(w[i], 0x64646464u, 0x5140u);
      const uint32_t b = __byte_perm(w[i], 0x64646464u, 0x5342u);
      __half2 ha = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
      __half2 hb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
      o[2 * i] = *reinterpret_cast<uint32_t*>(&ha);
      o[2 * i + 1] = *reinterpret_cast<uint32_t*>(&hb);
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Converts the int8 tile at shared address q into the 16-bit tile at c; called by 128 threads
// (t = 0..127), each converting four 16-byte pieces (piece i = row i / 4, bytes 16 (i % 4) ..).
// All four loads are issued before the first conversion, so their latencies overlap and the
// conversions of the four pieces are independent chains.  Loads: a warp reads 512 contiguous
// bytes.  Stores: the 8 threads of a store phase cover two rows x four pieces, i.e. the even and
// the odd 16-byte chunks of two rows of different parity, eight distinct bank groups after the
// swizzle.  The caller fences the writes to the async proxy before the MMA reads the tile.
template <typename T>
__device__ __forceinline__ void convert_int8_tile(uint32_t q, uint32_t c, int t) {
  uint32_t v[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[j][0]), "=r"(v[j][1]), "=r"(v[j][2]), "=r"(v[j][3])
                 : "r"(q + (uint32_t)(t + 128 * j) * 16u));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t i = (uint32_t)(t + 128 * j), row = i >> 2, p = i & 3u;
    const uint4 a = convert8<T>(v[j][0], v[j][1]);
    const uint4 b = convert8<T>(v[j][2], v[j][3]);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(c + swz128(row, 2 * p)),
                 "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w)
                 : "memory");
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(c + swz128(row, 2 * p + 1)),
                 "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                 : "memory");
  }
}

// One row of a 128-row x 64-byte int8 tile that TMA wrote with the 64-byte swizzle (16-byte
// chunk c of row r at chunk c ^ ((r >> 1) & 3)) -> its 64 values as 32 words of two 16-bit
// elements, lower K index in the low half (the layout of a K-major A tile in tensor memory).
// Eight consecutive rows read eight distinct 16-byte bank groups: conflict-free.
template <typename T>
__device__ __forceinline__ void convert_int8_row(uint32_t tile, int r, uint32_t (&out)[32]) {
  uint32_t v[4][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[c][0]), "=r"(v[c][1]), "=r"(v[c][2]), "=r"(v[c][3])
                 : "r"(tile + (uint32_t)r * 64u + ((uint32_t)(c ^ ((r >> 1) & 3)) << 4)));
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 a = convert8<T>(v[c][0], v[c][1]);
    const uint4 b = convert8<T>(v[c][2], v[c][3]);
    out[8 * c + 0] = a.x; out[8 * c + 1] = a.y; out[8 * c + 2] = a.z; out[8 * c + 3] = a.w;
    out[8 * c + 4] = b.x; out[8 * c + 5] = b.y; out[8 * c + 6] = b.z; out[8 * c + 7] = b.w;
  }
}

}  // namespace ti
