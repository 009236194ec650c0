// Host-side helpers: device properties, occupancy, error bookkeeping and TMA
// tensor-map encoding through the driver entry point (no -lcuda needed).
#include <algorithm>
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <set>
#include <tuple>
#include <unordered_map>
#include <utility>

#include "../../include/pagedserve_b200.h"
#include "host_util.h"

namespace psb {
namespace {
thread_local int g_last_cuda_error = 0;
std::mutex g_mu;
std::unordered_map<int, int> g_sm_count;
std::map<std::tuple<int, uintptr_t, size_t, int>, int> g_occ;  // (device, func, smem, threads) -> CTAs/SM
std::set<std::pair<int, uintptr_t>> g_smem_raised;             // (device, func) with the smem ceiling raised
std::set<std::pair<int, uintptr_t>> g_carveout_set;      // (device, func) preferring the full smem carve-out
std::set<std::pair<int, uintptr_t>> g_l1_set;            // (device, func) preferring the full L1 carve-out

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}
}  // namespace

int record_cuda_error(cudaError_t e) {
  g_last_cuda_error = static_cast<int>(e);
  return PSB_ERR_CUDA;
}

int check_launch() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PSB_OK : record_cuda_error(e);
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_sm_count.find(dev);
  if (it != g_sm_count.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  g_sm_count[dev] = n;
  return n;
}

bool prefer_max_shared(const void* func) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const auto key = std::make_pair(dev, reinterpret_cast<uintptr_t>(func));
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_carveout_set.insert(key).second) return true;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) {
    g_carveout_set.erase(key);
    return record_cuda_error(e), false;
  }
  return true;
}

bool prefer_max_l1(const void* func) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const auto key = std::make_pair(dev, reinterpret_cast<uintptr_t>(func));
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_l1_set.insert(key).second) return true;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxL1);
  if (e != cudaSuccess) {
    g_l1_set.erase(key);
    return record_cuda_error(e), false;
  }
  return true;
}

int resident_ctas(const void* func, int threads, size_t smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  cudaFuncAttributes fa;
  int regs_sm = 0, smem_sm = 0, reserved = 0, threads_sm = 0, blocks_sm = 0;
  if (cudaFuncGetAttributes(&fa, func) != cudaSuccess ||
      cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&blocks_sm, cudaDevAttrMaxBlocksPerMultiprocessor, dev) != cudaSuccess)
    return 0;
  const int warps = (threads + 31) / 32;
  // registers are allocated per warp in units of 256
  const int regs_warp = ((fa.numRegs * 32 + 255) / 256) * 256;
  int n = std::min(blocks_sm, threads_sm / std::max(threads, 1));
  if (regs_warp > 0) n = std::min(n, regs_sm / (regs_warp * warps));
  const size_t per_block = smem + fa.sharedSizeBytes + static_cast<size_t>(reserved);
  n = std::min<int>(n, static_cast<int>(smem_sm / std::max<size_t>(per_block, 1)));
  return n;
}

bool kernel_occupancy(const void* func, int threads, size_t smem, int* blocks_per_sm) {
  if (!prefer_max_shared(func)) return false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const auto fkey = std::make_pair(dev, reinterpret_cast<uintptr_t>(func));
  const auto okey = std::make_tuple(dev, reinterpret_cast<uintptr_t>(func), smem, threads);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_occ.find(okey);
  if (it != g_occ.end()) {
    *blocks_per_sm = it->second;
    return true;
  }
  // Raise the kernel's dynamic shared-memory ceiling once, to the device
  // maximum, so launches with any smaller size stay valid afterwards.
  if (g_smem_raised.insert(fkey).second) {
    int optin = 0;
    cudaFuncAttributes fa;
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, func);
    // the ceiling is the opt-in maximum less the kernel's static shared memory
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               optin - static_cast<int>(fa.sharedSizeBytes));
    if (e != cudaSuccess) {
      g_smem_raised.erase(fkey);
      return record_cuda_error(e), false;
    }
  }
  int n = 0;
  const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, threads, smem);
  if (e != cudaSuccess) return record_cuda_error(e), false;
  // The runtime's answer assumes the default shared-memory carve-out, not
  // the full carve-out these kernels ask for (measured on B200: 1 CTA per SM
  // for the 100 KB prefill kernel, which runs 2 per SM); count the SM's
  // registers, shared memory, threads and CTA slots instead when that allows more.
  n = std::max(n, resident_ctas(func, threads, smem));
  g_occ[okey] = n;
  *blocks_per_sm = n;
  return true;
}

CUtensorMapDataType dtype_to_tmap(int dtype) {
  switch (dtype) {
    case PSB_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case PSB_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  }
}

bool encode_pool_tile_map(CUtensorMap* map, const void* pool, int64_t tiles, int block_size, int head_dim,
                          int box_tiles, CUtensorMapDataType dt) {
  auto fn = encode_fn();
  if (!fn) return false;
  const size_t esz = dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(block_size),
                              static_cast<cuuint64_t>(tiles)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim * esz),
                                 static_cast<cuuint64_t>(head_dim * esz * block_size)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(head_dim), static_cast<cuuint32_t>(block_size),
                             static_cast<cuuint32_t>(box_tiles)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, dt, 3, const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_cuda_error = 10000 + static_cast<int>(r);
    return false;
  }
  return true;
}

bool encode_matrix_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride_elems,
                       int box_rows, int box_cols, CUtensorMapDataType dt) {
  auto fn = encode_fn();
  if (!fn) return false;
  const size_t esz = dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems * esz)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_cuda_error = 10000 + static_cast<int>(r);
    return false;
  }
  return true;
}

bool encode_rows_map(CUtensorMap* map, const void* base, int64_t rows, int heads, int head_dim, int64_t row_stride,
                     int64_t head_stride, int box_rows, CUtensorMapDataType dt) {
  auto fn = encode_fn();
  if (!fn) return false;
  const size_t esz = dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_stride * esz), static_cast<cuuint64_t>(row_stride * esz)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(head_dim), 1u, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_cuda_error = 10000 + static_cast<int>(r);
    return false;
  }
  return true;
}

bool encode_pool_map(CUtensorMap* map, const void* base, int64_t tiles, int block_size, int head_dim,
                     CUtensorMapDataType dt) {
  auto fn = encode_fn();
  if (!fn) return false;
  const size_t esz = dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(block_size),
                              static_cast<cuuint64_t>(tiles)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim * esz),
                                 static_cast<cuuint64_t>(block_size) * head_dim * esz};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(head_dim), static_cast<cuuint32_t>(block_size), 1u};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_cuda_error = 10000 + static_cast<int>(r);
    return false;
  }
  return true;
}

}  // namespace psb

extern "C" const char* psb_version(void) { return "pagedserve_b200 0.1.0 sm_100a"; }

extern "C" const char* psb_status_string(int status) {
  switch (status) {
    case PSB_OK: return "ok";
    case PSB_ERR_INVALID: return "invalid argument";
    case PSB_ERR_WORKSPACE: return "workspace too small";
    case PSB_ERR_UNSUPPORTED: return "unsupported geometry or dtype";
    case PSB_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

extern "C" int psb_last_cuda_error(void) { return psb::g_last_cuda_error; }

extern "C" int psb_device_sm_count(void) { return psb::device_sm_count(); }
