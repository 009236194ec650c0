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
};

// tcgen05 / TMEM kernel (varlen_prefill_tc.cu): bf16/f16, head_dim 64,
// 16-byte aligned rows.
bool prefill_tc_supported(const PrefillParams& p, int dtype);
int prefill_tc_launch(const PrefillParams& p, int dtype, cudaStream_t s);

}  // namespace psb
