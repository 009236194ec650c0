// Host-side helpers shared by the pagedserve_b200 translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

namespace psb {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// SM count of the current device (cached per device).
int device_sm_count();

// Ask for the largest shared-memory carve-out for ``func`` (once per device).
// Every kernel of this library does, so a decode CTA (188 KB of shared
// memory) can start on an SM where a small kernel of the same stream - the
// split-K combine, reshape_and_cache - still runs: an SM changes its L1 /
// shared split only when idle, so differing preferences would serialise
// them.
bool prefer_max_shared(const void* func);

// Ask for the largest L1 (smallest shared-memory) carve-out for ``func``
// (once per device; overrides prefer_max_shared).  For kernels that stream
// with plain global loads and use no shared memory: every load in flight
// holds L1 space until its data returns, so L1 capacity bounds an SM's
// bytes in flight.
bool prefer_max_l1(const void* func);

// CTAs of ``func`` that fit on one SM at ``threads`` threads and ``smem``
// dynamic shared bytes under the full carve-out: registers (per warp, in
// units of 256), shared memory (plus static and the per-CTA reservation),
// threads and CTA slots.
int resident_ctas(const void* func, int threads, size_t smem);

// Max resident CTAs per SM for ``func`` at ``threads`` and ``smem`` dynamic
// bytes; raises the kernel's dynamic shared-memory limit when needed (and
// sets the carve-out preference above).
bool kernel_occupancy(const void* func, int threads, size_t smem, int* blocks_per_sm);

// Remember a CUDA error for psb_last_cuda_error(); returns PSB_ERR_CUDA.
int record_cuda_error(cudaError_t e);

// PSB_OK, or PSB_ERR_CUDA when the last launch failed.
int check_launch();

// Drop a non-sticky error another library left in this thread's runtime
// state, so check_launch() reports only our own launch.
inline void discard_stale_error() { (void)cudaGetLastError(); }

CUtensorMapDataType dtype_to_tmap(int dtype);

// Scratch bytes one psb_paged_decode call with these arguments needs on the
// path it will take (fast: the fixed split-K slot table; generic: counters
// and per-chunk partials), 0 for an invalid geometry.  Unlike
// psb_paged_decode_workspace_size, which covers either path because it does
// not see the pointers, this is exact for the call.
size_t decode_scratch_for_call(const void* query, int64_t q_stride_b, int64_t q_stride_h, const void* out,
                               int64_t o_stride_b, int64_t o_stride_h, const void* k_cache, const void* v_cache,
                               int32_t batch, int32_t q_heads, int32_t num_kv_heads, int32_t block_size,
                               int32_t head_dim, int32_t dtype, int32_t max_context);

// Launch with programmatic stream serialization (the kernel may begin while
// its stream predecessor is still running; see pdl_wait in common.cuh).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// 3-D tiled map over a paged pool viewed as [tiles, block_size, head_dim]
// (one tile per (layer, block, kv head)), box = ``box_tiles`` whole
// consecutive tiles, 128-byte swizzle.  head_dim * element size must be 128 bytes.
bool encode_pool_tile_map(CUtensorMap* map, const void* pool, int64_t tiles, int block_size, int head_dim,
                          int box_tiles, CUtensorMapDataType dt);

// 3-D tiled map over [rows, heads, head_dim] rows of a packed token batch
// (element strides row_stride, head_stride; unit stride along head_dim):
// box = box_rows rows of one head, 128-byte swizzle.  head_dim * element
// size must be 128 bytes, both strides multiples of 16 bytes.
bool encode_rows_map(CUtensorMap* map, const void* base, int64_t rows, int heads, int head_dim, int64_t row_stride,
                     int64_t head_stride, int box_rows, CUtensorMapDataType dt);

// 3D tensor map over a paged K or V pool [layers * blocks * kv heads tiles,
// block_size rows, head_dim]: one box is one (layer, block, kv head) tile of
// block_size x head_dim, 128-byte swizzled.
bool encode_pool_map(CUtensorMap* map, const void* base, int64_t tiles, int block_size, int head_dim,
                     CUtensorMapDataType dt);

// 2-D tiled map over a row-major [rows, cols] matrix with row pitch
// ``row_stride_elems``; box = box_rows x box_cols, 128-byte swizzle.
bool encode_matrix_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride_elems,
                       int box_rows, int box_cols, CUtensorMapDataType dt);

}  // namespace psb
