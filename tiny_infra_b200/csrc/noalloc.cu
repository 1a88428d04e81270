// Paged decode attention that needs no caller-provided scratch: the split-K workspace lives in
// a static device array of this library (TI_NOALLOC_SCRATCH_BYTES per GPU that loads it, held
// until the process exits).  For callers that cannot allocate device memory themselves.
//
// The array's name is a host-side stand-in, not a device address, so the host never passes it
// to a kernel: on first use on each device (with that device current) the address is looked
// up once with cudaGetSymbolAddress and cached per device.  That first call therefore also
// loads this library's device code on the device and should happen before any stream capture.
// Every call shares the one array, whose contents persist between calls: the split-K arrival
// counters at its start are cleared on the call's stream before each launch, and calls that
// overlap on the GPU (other streams, other threads) race on the array.  The cached address
// belongs to the device's current context: after cudaDeviceReset (or any teardown of that
// context) the entry point must not be called again in the same process.
#include <cstdio>
#include <mutex>

#include "capi_internal.h"
#include "common.cuh"

namespace ti {
namespace noalloc {

constexpr size_t kScratchBytes = TI_NOALLOC_SCRATCH_BYTES;
constexpr size_t kCounterBytes = 64 * 1024;     // the split-K arrival counters (zero on entry)
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

static std::mutex g_mu;
static void* g_addr[kMaxDevices];

static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, "paged attention (no-alloc): cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(TI_ERR_UNSUPPORTED, "paged attention (no-alloc): device ordinal >= 64");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess)
      return set_cuda_error(e, "paged attention (no-alloc): cudaGetSymbolAddress of the scratch array");
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return TI_OK;
}

}  // namespace noalloc
}  // namespace ti

using namespace ti;

extern "C" int ti_paged_attention_decode_noalloc(
    void* out, int64_t out_seq_stride, const void* q, int64_t q_seq_stride, const void* k_cache,
    const void* v_cache, int64_t num_blocks, const int32_t* block_tables, int64_t bt_stride,
    const int32_t* row_index, const int32_t* context_lens, int batch, int num_heads,
    int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq, int dtype,
    void* stream) {
  clear_error();
  if (batch == 0) return TI_OK;
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_blocks_per_seq <= 0)
    return set_error(TI_ERR_INVALID_ARGUMENT, "paged attention (no-alloc): bad sizes");
  // a call whose sequences are never split (head_dim 128 with at most one partition of
  // blocks) needs no scratch at all, whatever its batch size
  if (attn_split_parts(batch, num_heads, num_kv_heads, head_dim, max_blocks_per_seq) <= 1)
    return ti_paged_attention_decode(out, out_seq_stride, q, q_seq_stride, k_cache, v_cache,
                                     num_blocks, block_tables, bt_stride, row_index, context_lens,
                                     batch, num_heads, num_kv_heads, head_dim, block_size,
                                     max_blocks_per_seq, dtype, 0, nullptr, 0, stream);
  const size_t need = ti_paged_attention_workspace_bytes(batch, num_heads, num_kv_heads, head_dim,
                                                          max_blocks_per_seq, 0);
  if (need > noalloc::kScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "paged attention (no-alloc): this batch needs %zu bytes of split-K scratch but the "
             "static scratch holds %zu; use ti_paged_attention_decode with a workspace",
             need, noalloc::kScratchBytes);
    return set_error(TI_ERR_WORKSPACE, msg);
  }
  void* ws = nullptr;
  int rc = noalloc::scratch_address(&ws);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(ws, 0, noalloc::kCounterBytes, s);
  if (e != cudaSuccess) return set_cuda_error(e, "paged attention (no-alloc): clearing the counters");
  return ti_paged_attention_decode(out, out_seq_stride, q, q_seq_stride, k_cache, v_cache,
                                   num_blocks, block_tables, bt_stride, row_index, context_lens,
                                   batch, num_heads, num_kv_heads, head_dim, block_size,
                                   max_blocks_per_seq, dtype, 0, ws, noalloc::kScratchBytes,
                                   stream);
}
