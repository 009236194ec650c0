// Allocation-free paged decode: psb_paged_decode with its split-K scratch in
// a fixed, statically sized device array instead of a caller workspace.
//
// For callers that cannot allocate device memory at the point where they
// launch decode: an engine step running under a memory pool that is already
// carved up, a host without a device allocator, or an FFI caller (cgo/JNI
// style) that owns no CUDA memory of its own.  The scratch is reserved when
// the module that holds it loads, so nothing is allocated per call.
//
// The array lives in this translation unit only, so its module (and the
// reservation) is loaded on the first call to this entry point and never by
// psb_paged_decode.

#include <cuda_runtime.h>

#include <mutex>

#include "host_util.h"
#include "pagedserve_b200.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

// Split-K scratch for one call at a time per device: on the bf16/f16 fast
// path the fixed table of per-warp partial slots (written before it is read
// in every call, so it needs no clearing), on the CUDA-core path the
// per-(sequence, kv head) arrival counters, which that path zeroes itself at
// the start of every call, and the per-chunk partials.
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's copy of the scratch array, looked up once
// per device with that device current.
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return psb::record_cuda_error(e);
  if (dev < 0 || dev >= kMaxDevices) return PSB_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return psb::record_cuda_error(e);
    if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 256 != 0) return PSB_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return PSB_OK;
}

}  // namespace

extern "C" size_t psb_paged_decode_static_capacity(void) { return kStaticScratchBytes; }

extern "C" int psb_paged_decode_static(const void* query, int64_t q_stride_b, int64_t q_stride_h, void* out,
                                       int64_t o_stride_b, int64_t o_stride_h, const void* k_cache,
                                       const void* v_cache, const int32_t* block_tables, int64_t table_stride,
                                       const int32_t* context_lens, int32_t batch, int32_t q_heads, int32_t layer,
                                       int32_t num_layers, int64_t num_blocks, int32_t num_kv_heads,
                                       int32_t block_size, int32_t head_dim, int32_t dtype, int32_t max_context,
                                       float scale, int32_t* error_flag, psb_stream_t stream) {
  if (!query || !out || !k_cache || !v_cache || !block_tables || !context_lens) return PSB_ERR_INVALID;
  // only the scratch of the path this call takes counts: the fast path's is a
  // fixed ~10.8 MB whatever the batch, so serving batches fit that the
  // CUDA-core path's per-chunk partials would not
  const size_t need = psb::decode_scratch_for_call(query, q_stride_b, q_stride_h, out, o_stride_b, o_stride_h,
                                                   k_cache, v_cache, batch, q_heads, num_kv_heads, block_size,
                                                   head_dim, dtype, max_context);
  if (need == 0) return PSB_ERR_INVALID;
  if (need > kStaticScratchBytes) return PSB_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != PSB_OK) return st;
  return psb_paged_decode(query, q_stride_b, q_stride_h, out, o_stride_b, o_stride_h, k_cache, v_cache,
                          block_tables, table_stride, context_lens, batch, q_heads, layer, num_layers, num_blocks,
                          num_kv_heads, block_size, head_dim, dtype, max_context, scale, scratch,
                          kStaticScratchBytes, error_flag, stream);
}
