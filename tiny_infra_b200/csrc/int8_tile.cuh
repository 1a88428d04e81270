// Exact int8 -> bf16 / fp16 conversion of a weight tile in shared memory, for the weight-only int8
// lm_head kernels (lmhead_i8.cu, gemv.cu).
//
// Input: a 128-row x 64-byte int8 tile as TMA writes it without swizzle (row pitch 64 bytes).
// Output: the same 128 x 64 values as 16-bit elements in the canonical SWIZZLE_128B K-major
// layout the tcgen05 shared-memory descriptors read (128-byte rows, 1024-byte aligned base).
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

}  // namespace ti
