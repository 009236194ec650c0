// reshape_and_cache: one launch scatters every new token's K and V rows into
// the paged pools through an int64 slot mapping.
//
// Same addressing and bytes as PagedKVCache.write_token
// (pagedserve/engine/paged_kv_cache.py:187-200):
//     block = slot / block_size, offset = slot % block_size,
//     cache[layer, block, h, offset, :] = src[t, h, :]
// which the reference issues as two tiny copy kernels per token per layer
// (pagedserve/attention/batched_paged_attention.py:115-124).  Each thread
// moves one 16-byte vector of K and the matching vector of V when rows are
// 16-byte aligned, else single elements; the copy is bit-exact.  A negative
// slot is a padding row and writes nothing; a slot past the pool is skipped
// and flagged (PSB_DEVERR_SLOT_RANGE).
#include <algorithm>

#include "common.cuh"
#include "host_util.h"

namespace psb {
namespace {

template <typename V>
__global__ void __launch_bounds__(256) reshape_and_cache_kernel(
    const char* __restrict__ key, int64_t kst, int64_t ksh, const char* __restrict__ value, int64_t vst,
    int64_t vsh, char* __restrict__ k_cache, char* __restrict__ v_cache, const int64_t* __restrict__ slots,
    int32_t num_tokens, int64_t layer_base_tiles, int32_t hkv, int32_t block_size, int32_t row_bytes,
    int64_t pool_slots, int32_t* err) {
  // A decode launched right after may start now: its prologue reads only
  // lengths and block tables, and it waits for this grid before reading the
  // pool.  This grid itself is a programmatic dependent: it waits for its
  // stream predecessor (which may produce key, value or the slots, or read
  // the pool) before touching anything.
  pdl_launch_dependents();
  pdl_wait();
  const int nvec = row_bytes / static_cast<int>(sizeof(V));
  const int64_t per_token = static_cast<int64_t>(hkv) * nvec;
  const int64_t total = per_token * num_tokens;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / per_token;
    const int r = static_cast<int>(i - t * per_token);
    const int h = r / nvec, v = r - h * nvec;
    const int64_t s = __ldg(slots + t);
    if (s < 0) continue;
    if (s >= pool_slots) {
      if (v == 0 && h == 0) flag_error(err, PSB_DEVERR_SLOT_RANGE);
      continue;
    }
    const int64_t blk = s / block_size, off = s - blk * block_size;
    const int64_t dst = (((layer_base_tiles + blk * hkv + h) * block_size + off) * row_bytes) + v * sizeof(V);
    *reinterpret_cast<V*>(k_cache + dst) = __ldg(reinterpret_cast<const V*>(key + t * kst + h * ksh) + v);
    *reinterpret_cast<V*>(v_cache + dst) = __ldg(reinterpret_cast<const V*>(value + t * vst + h * vsh) + v);
  }
}

}  // namespace
}  // namespace psb

using namespace psb;

extern "C" int psb_reshape_and_cache(const void* key, int64_t key_stride_t, int64_t key_stride_h, const void* value,
                                     int64_t value_stride_t, int64_t value_stride_h, void* k_cache, void* v_cache,
                                     const int64_t* slot_mapping, int32_t num_tokens, int32_t layer,
                                     int32_t num_layers, int64_t num_blocks, int32_t num_kv_heads,
                                     int32_t block_size, int32_t head_dim, int32_t dtype, int32_t* error_flag,
                                     psb_stream_t stream) {
  if (num_tokens < 0 || num_layers <= 0 || layer < 0 || layer >= num_layers || num_blocks <= 0 ||
      num_kv_heads <= 0 || block_size <= 0 || head_dim <= 0)
    return PSB_ERR_INVALID;
  if (dtype != PSB_F32 && dtype != PSB_F16 && dtype != PSB_BF16) return PSB_ERR_INVALID;
  if (num_tokens == 0) return PSB_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping) return PSB_ERR_INVALID;
  const int esz = elem_bytes(dtype);
  const int row_bytes = head_dim * esz;
  const int64_t kst = key_stride_t * esz, ksh = key_stride_h * esz;
  const int64_t vst = value_stride_t * esz, vsh = value_stride_h * esz;
  const bool vec16 = row_bytes % 16 == 0 && kst % 16 == 0 && ksh % 16 == 0 && vst % 16 == 0 && vsh % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(key) % 16 == 0 && reinterpret_cast<uintptr_t>(value) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(k_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(v_cache) % 16 == 0;
  const int sms = device_sm_count();
  if (sms <= 0) return PSB_ERR_CUDA;
  const int64_t layer_base_tiles = static_cast<int64_t>(layer) * num_blocks * num_kv_heads;
  const int64_t pool_slots = num_blocks * block_size;
  const int threads = 256;
  const int64_t units = static_cast<int64_t>(num_tokens) * num_kv_heads * (vec16 ? row_bytes / 16 : head_dim);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((units + threads - 1) / threads, sms * 8));
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const char* kp = static_cast<const char*>(key);
  const char* vp = static_cast<const char*>(value);
  char* kc = static_cast<char*>(k_cache);
  char* vc = static_cast<char*>(v_cache);
  cudaError_t e = cudaSuccess;
  if (vec16) {
    discard_stale_error();
    if (!prefer_max_shared(reinterpret_cast<const void*>(reshape_and_cache_kernel<uint4>))) return PSB_ERR_CUDA;
    e = launch_pdl(reshape_and_cache_kernel<uint4>, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0, s, kp, kst,
                   ksh, vp, vst, vsh, kc, vc, slot_mapping, num_tokens, layer_base_tiles, num_kv_heads, block_size,
                   row_bytes, pool_slots, error_flag);
  } else if (esz == 4) {
    discard_stale_error();
    if (!prefer_max_shared(reinterpret_cast<const void*>(reshape_and_cache_kernel<uint32_t>))) return PSB_ERR_CUDA;
    e = launch_pdl(reshape_and_cache_kernel<uint32_t>, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0, s, kp, kst,
                   ksh, vp, vst, vsh, kc, vc, slot_mapping, num_tokens, layer_base_tiles, num_kv_heads, block_size,
                   row_bytes, pool_slots, error_flag);
  } else {
    discard_stale_error();
    if (!prefer_max_shared(reinterpret_cast<const void*>(reshape_and_cache_kernel<uint16_t>))) return PSB_ERR_CUDA;
    e = launch_pdl(reshape_and_cache_kernel<uint16_t>, dim3(static_cast<unsigned>(blocks)), dim3(threads), 0, s, kp, kst,
                   ksh, vp, vst, vsh, kc, vc, slot_mapping, num_tokens, layer_base_tiles, num_kv_heads, block_size,
                   row_bytes, pool_slots, error_flag);
  }
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}
