// pack_step: GPU-side ragged-batch packer.
//
// From the scheduler's step plan (per request: its row in the device-resident
// block-table store, the position of its first new token, and how many new
// tokens it has) build, in one launch, everything the step's kernels read:
// cu_seqlens, context_lens, the int64 slot of every new token, the absolute
// position of every new token and the zero-padded [B, width] block table.
//
// Replaces the host loop of pagedserve/attention/triton_paged_decode.py:134-154
// (one torch.tensor H2D copy per row per layer) and the per-token slot
// arithmetic of pagedserve/engine/paged_kv_cache.py:187-192.  Every CTA scans
// query_lens into shared memory itself (no second launch, no grid sync), then
// the grid strides over tokens and table entries.
#include <algorithm>

#include "common.cuh"
#include "host_util.h"

namespace psb {
namespace {

constexpr int kPackThreads = 256;

__global__ void __launch_bounds__(kPackThreads) pack_step_kernel(
    const int32_t* __restrict__ store, int64_t store_width, int32_t store_rows, const int32_t* __restrict__ req_rows,
    const int32_t* __restrict__ starts, const int32_t* __restrict__ qlens, int32_t batch, int32_t total,
    int32_t block_size, int32_t* __restrict__ cu, int32_t* __restrict__ ctx_out, int64_t* __restrict__ slots,
    int64_t* __restrict__ positions, int32_t* __restrict__ tables, int32_t out_width, int32_t* err) {
  extern __shared__ int32_t s_cu[];  // [batch + 1]
  __shared__ int32_t warp_sums[kPackThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (batch + kPackThreads - 1) / kPackThreads;
  const int begin = min(tid * per, batch), end = min(begin + per, batch);
  int local = 0;
  for (int b = begin; b < end; ++b) local += max(qlens[b], 0);
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  int run = incl - local;
  for (int w = 0; w < warp; ++w) run += warp_sums[w];
  for (int b = begin; b < end; ++b) {
    s_cu[b] = run;
    run += max(qlens[b], 0);
  }
  if (tid == 0) {
    int tot = 0;
    for (int w = 0; w < kPackThreads / 32; ++w) tot += warp_sums[w];
    s_cu[batch] = tot;
  }
  __syncthreads();

  const int64_t gtid = blockIdx.x * static_cast<int64_t>(kPackThreads) + tid;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * kPackThreads;
  if (blockIdx.x == 0) {
    if (tid == 0 && s_cu[batch] != total) flag_error(err, PSB_DEVERR_SEQLENS);
    for (int b = tid; b <= batch; b += kPackThreads) cu[b] = s_cu[b];
    for (int b = tid; b < batch; b += kPackThreads) {
      const int q = qlens[b];
      if (q < 0 || starts[b] < 0) flag_error(err, PSB_DEVERR_CONTEXT);
      ctx_out[b] = starts[b] + max(q, 0);
    }
  }
  // padded block tables: entries past the blocks the context needs are zero
  for (int64_t i = gtid; i < static_cast<int64_t>(batch) * out_width; i += gstride) {
    const int b = static_cast<int>(i / out_width), j = static_cast<int>(i - static_cast<int64_t>(b) * out_width);
    const int row = req_rows[b];
    const int ctx = starts[b] + max(qlens[b], 0);
    const int need = (ctx + block_size - 1) / block_size;
    int32_t v = 0;
    if (row < 0 || row >= store_rows || need > store_width || need > out_width) {
      if (j == 0) flag_error(err, PSB_DEVERR_CONTEXT);
    } else if (j < need) {
      v = store[row * store_width + j];
      if (v < 0) flag_error(err, PSB_DEVERR_BLOCK_RANGE);
    }
    tables[i] = v;
  }
  // per-token slot and position
  const int ntok = min(total, s_cu[batch]);
  for (int64_t i = gtid; i < ntok; i += gstride) {
    int lo = 0, hi = batch - 1;  // largest b with s_cu[b] <= i
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_cu[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    const int64_t pos = static_cast<int64_t>(starts[b]) + (i - s_cu[b]);
    const int row = req_rows[b];
    const int64_t logical = pos / block_size;
    int64_t slot = -1;
    if (row >= 0 && row < store_rows && logical < store_width && pos >= 0) {
      const int32_t blk = store[row * store_width + logical];
      if (blk >= 0) slot = static_cast<int64_t>(blk) * block_size + (pos - logical * block_size);
      else flag_error(err, PSB_DEVERR_BLOCK_RANGE);
    } else {
      flag_error(err, PSB_DEVERR_CONTEXT);
    }
    slots[i] = slot;
    positions[i] = pos;
  }
}

}  // namespace
}  // namespace psb

using namespace psb;

extern "C" int psb_pack_step(const int32_t* table_store, int64_t store_width, int32_t store_rows,
                             const int32_t* req_rows, const int32_t* starts, const int32_t* query_lens, int32_t batch,
                             int32_t total, int32_t block_size, int32_t* cu_seqlens, int32_t* context_lens,
                             int64_t* slot_mapping, int64_t* positions, int32_t* block_tables, int32_t out_width,
                             int32_t* error_flag, psb_stream_t stream) {
  if (batch < 0 || total < 0 || block_size <= 0 || store_width <= 0 || store_rows <= 0 || out_width <= 0)
    return PSB_ERR_INVALID;
  if (batch == 0) return total == 0 ? PSB_OK : PSB_ERR_INVALID;
  if (!table_store || !req_rows || !starts || !query_lens || !cu_seqlens || !context_lens || !block_tables ||
      (total > 0 && (!slot_mapping || !positions)))
    return PSB_ERR_INVALID;
  const size_t smem = sizeof(int32_t) * (static_cast<size_t>(batch) + 1);
  if (smem > 200 * 1024) return PSB_ERR_UNSUPPORTED;
  const int sms = device_sm_count();
  if (sms <= 0) return PSB_ERR_CUDA;
  int occ = 0;
  if (!kernel_occupancy(reinterpret_cast<const void*>(pack_step_kernel), kPackThreads, smem, &occ)) return PSB_ERR_CUDA;
  const int64_t work = std::max<int64_t>(total, static_cast<int64_t>(batch) * out_width);
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((work + kPackThreads - 1) / kPackThreads, sms));
  discard_stale_error();
  pack_step_kernel<<<static_cast<unsigned>(grid), kPackThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      table_store, store_width, store_rows, req_rows, starts, query_lens, batch, total, block_size, cu_seqlens,
      context_lens, slot_mapping, positions, block_tables, out_width, error_flag);
  return check_launch();
}
