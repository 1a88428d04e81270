// Library-level C ABI: error reporting, launch accounting, device status word, tensor maps.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "capi_internal.h"
#include "common.cuh"

namespace ti {

__device__ unsigned int g_device_status = 0;

static thread_local std::string t_last_error;
static std::atomic<uint64_t> g_launches{0};

int set_error(int code, const char* msg) {
  t_last_error = msg ? msg : "";
  return code;
}
int set_cuda_error(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return TI_ERR_CUDA;
}
void clear_error() { t_last_error.clear(); }
void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("TI_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_tensor_map_2d(CUtensorMap* out, CUtensorMapDataType type, void* base,
                         const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                         const cuuint32_t* box, const cuuint32_t* elem_strides,
                         CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return set_error(TI_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  CUresult r = fn(out, type, 2, base, dims, strides_bytes, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "cuTensorMapEncodeTiled failed (%d): dims=%llu,%llu stride=%llu box=%u,%u",
             (int)r, (unsigned long long)dims[0], (unsigned long long)dims[1],
             (unsigned long long)strides_bytes[0], box[0], box[1]);
    return set_error(TI_ERR_CUDA, buf);
  }
  return TI_OK;
}

}  // namespace ti

extern "C" const char* ti_last_error(void) { return ti::t_last_error.c_str(); }
extern "C" int ti_version(void) { return 1; }
extern "C" uint64_t ti_launch_count(void) { return ti::g_launches.load(); }

extern "C" int ti_device_status(unsigned int* bits, int clear, void* stream) {
  ti::clear_error();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return ti::set_cuda_error(e, "ti_device_status: stream sync");
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, ti::g_device_status, sizeof(v));
  if (e != cudaSuccess) return ti::set_cuda_error(e, "ti_device_status: read");
  if (bits) *bits = v;
  if (clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(ti::g_device_status, &z, sizeof(z));
    if (e != cudaSuccess) return ti::set_cuda_error(e, "ti_device_status: clear");
  }
  return TI_OK;
}
