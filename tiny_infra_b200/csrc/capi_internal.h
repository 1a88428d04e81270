// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace ti {

// Record an error message for ti_last_error() and return `code`.
int set_error(int code, const char* msg);
int set_cuda_error(cudaError_t e, const char* what);
void clear_error();
void count_launch(unsigned n = 1);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link needed).
int encode_tensor_map_2d(CUtensorMap* out, CUtensorMapDataType type, void* base,
                         const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                         const cuuint32_t* box, const cuuint32_t* elem_strides,
                         CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo);

}  // namespace ti
