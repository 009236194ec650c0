// Shared declarations of the packed-prefill translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace psb {

struct PrefillParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int64_t qst, qsh, kst, ksh, vst, vsh, ost, osh;  // element strides (token, head)
  const int32_t* cu;
  int32_t num_seqs, total, max_seqlen, hq, hkv, head_dim;
  float scale_log2;
  int32_t* err;
  // paged prefill (psb_paged_prefill): k and v are the pools
  // [num_layers, num_blocks, hkv, block_size, head_dim]; sequence i's keys are
  // positions 0 .. ctx[i] - 1 read through tables[i, :], and its cu-rows are
  // the last (cu[i+1] - cu[i]) of them
  bool paged = false;
  const int32_t* tables = nullptr;
  int64_t table_stride = 0;
  const int32_t* ctx = nullptr;
  int32_t layer = 0, num_layers_total = 0, block_size = 0, max_context = 0;
  int64_t num_blocks = 0;
  // tcgen05 kernel: room in shared memory for this many tiles per CTA (set
  // by the launch from an upper bound of the tiles and the grid)
  int32_t max_cta_tiles = 0;
};

// tcgen05 / TMEM kernel (varlen_prefill_tc.cu): bf16/f16, head_dim 64,
// 16-byte aligned rows.
bool prefill_tc_supported(const PrefillParams& p, int dtype);
int prefill_tc_launch(const PrefillParams& p, int dtype, cudaStream_t s);

}  // namespace psb
