// One RMSNorm row per warp, shared by the standalone kernel (elementwise.cu) and the GEMM
// prologue that normalises its own activation rows (gemm.cu): both produce the same bits.
//
// Rounding as the reference (models/qwen_25.py:34-36): out = bf16(w * bf16(x * rstd)),
// rstd = rsqrtf(mean(x^2) + eps), the sum of squares taken per lane over its 8-element chunks
// and then across the warp by shuffles.  The row is held in registers: each lane owns NC
// chunks of 8 elements (hidden <= NC * 256), so x is read once.
#pragma once

#include "common.cuh"

namespace ti {
namespace ew {

template <typename T>
struct Vec8 {   // 8 elements of a 16-bit type in one 16-byte register group
  uint4 raw;
  __device__ __forceinline__ void load(const T* p) { raw = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void store(T* p) const { *reinterpret_cast<uint4*>(p) = raw; }
  __device__ __forceinline__ void to_float(float* f) const {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 v = Elem<T>::unpack2(u[i]);
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
  __device__ __forceinline__ void from_float(const float* f) {
    uint32_t* u = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) u[i] = Elem<T>::pack2(f[2 * i], f[2 * i + 1]);
  }
};

__device__ __forceinline__ void load8f(const float* p, float* f) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// The norm weight as this lane's NC chunks of 8 floats (static: loadable before any wait).
template <typename T, int NC>
__device__ __forceinline__ void rms_load_weight(const T* __restrict__ w, int H, int lane,
                                                float (&wf)[NC][8]) {
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int c = lane * 8 + k * 256;
    if (c < H) {
      Vec8<T> wv;
      wv.load(w + c);
      wv.to_float(wf[k]);
    }
  }
}

// Normalise row xr (H elements of TX) into out (H elements of T); called by all 32 lanes.
template <typename TX, typename T, int NC>
__device__ __forceinline__ void rms_row(T* __restrict__ out, const TX* __restrict__ xr,
                                        const float (&wf)[NC][8], float eps, int H, int lane) {
  float f[NC][8];
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int c = lane * 8 + k * 256;
    if (c < H) {
      if constexpr (sizeof(TX) == 4) load8f(reinterpret_cast<const float*>(xr) + c, f[k]);
      else { Vec8<TX> v; v.load(xr + c); v.to_float(f[k]); }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    if (lane * 8 + k * 256 < H) {
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[k][j] * f[k][j];
    }
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int c = lane * 8 + k * 256;
    if (c < H) {
      float o8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o8[j] = wf[k][j] * Elem<T>::to_f(Elem<T>::from_f(f[k][j] * rstd));
      Vec8<T> o;
      o.from_float(o8);
      o.store(out + c);
    }
  }
}

}  // namespace ew
}  // namespace ti
