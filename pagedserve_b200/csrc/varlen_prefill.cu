// Packed ragged causal prefill attention.
//
// Replaces the reference's per-request prefill attention
// (pagedserve/attention/qwen_paged_attention.py:121-128 -> paged_attention.py:94-145,
// O(S^2) Python gathers per request) with one launch over a packed batch:
// q [T, Hq, D], k/v [T, Hkv, D], sequence i = rows cu_seqlens[i]..cu_seqlens[i+1],
// causal within each sequence, GQA (q head h reads kv head h / (Hq/Hkv)).
//
// This file holds the CUDA-core kernel used for fp32 and for geometries the
// tensor-core kernel (varlen_prefill_tc.cu) does not cover: one warp per
// (query row, q head), 32 keys per step (one key per lane for Q.K, lanes
// over head_dim for P.V), online softmax in fp32, probabilities rounded to
// the input dtype before P.V as paged_attention.py:133-137 does.
#include <algorithm>

#include "common.cuh"
#include "host_util.h"
#include "varlen_prefill.h"

namespace psb {
namespace {

constexpr int kGenThreads = 128;
constexpr int kMaxDimPerLane = 8;  // head_dim <= 256

// Context length of sequence s of a paged batch: at least its query rows and
// at most max_context (anything else is flagged and clamped).
__device__ __forceinline__ int paged_ctx(const PrefillParams& p, int s, int n) {
  int c = p.ctx[s];
  if (c < n || c > p.max_context) {
    flag_error(p.err, PSB_DEVERR_CONTEXT);
    c = c < n ? n : p.max_context;
  }
  return c;
}

// PAGED: keys and values come from the pools through the block table
// (psb_paged_prefill), the query rows being the last positions of each
// sequence's context.
template <typename T, bool PAGED>
__global__ void __launch_bounds__(kGenThreads) prefill_generic_kernel(const PrefillParams p) {
  extern __shared__ float s_q[];  // [warps][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = p.head_dim;
  const int64_t task = blockIdx.x * static_cast<int64_t>(kGenThreads / 32) + warp;
  if (task >= static_cast<int64_t>(p.total) * p.hq) return;
  const int row = static_cast<int>(task / p.hq), qh = static_cast<int>(task - static_cast<int64_t>(row) * p.hq);
  const int kh = qh / (p.hq / p.hkv);
  // sequence of this row
  int lo = 0, hi = p.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.cu[mid] <= row) lo = mid; else hi = mid - 1;
  }
  const int kbeg = max(p.cu[lo], 0);
  // key positions 0 .. last (within the sequence when PAGED, packed rows otherwise)
  int first = kbeg, last = row;
  int32_t const* table = nullptr;
  int64_t layer_base = 0;
  if constexpr (PAGED) {
    const int n = p.cu[lo + 1] - kbeg;
    const int ctx = paged_ctx(p, lo, n);
    first = 0;
    last = ctx - n + (row - kbeg);
    table = p.tables + static_cast<int64_t>(lo) * p.table_stride;
    layer_base = static_cast<int64_t>(p.layer) * p.num_blocks;
  }
  // row pointer of key position j (nullptr for a block outside the pool)
  auto key_row = [&](const void* base, int64_t st, int64_t sh, int j) -> const T* {
    if constexpr (PAGED) {
      const int blk = table[j / p.block_size];
      if (blk < 0 || blk >= p.num_blocks) return nullptr;
      return reinterpret_cast<const T*>(base) +
             (((layer_base + blk) * p.hkv + kh) * p.block_size + j % p.block_size) * static_cast<int64_t>(D);
    } else {
      return reinterpret_cast<const T*>(base) + kh * sh + static_cast<int64_t>(j) * st;
    }
  };
  float* q = s_q + warp * D;
  const T* qp = reinterpret_cast<const T*>(p.q) + row * p.qst + qh * p.qsh;
  for (int d = lane; d < D; d += 32) q[d] = Elem<T>::to_float(qp[d]);
  __syncwarp();
  float m = -INFINITY, l = 0.f, acc[kMaxDimPerLane];
#pragma unroll
  for (int i = 0; i < kMaxDimPerLane; ++i) acc[i] = 0.f;
  for (int k0 = first; k0 <= last; k0 += 32) {
    const int key = k0 + lane;
    float s = -INFINITY;
    bool live = key <= last;
    if (live) {
      const T* kr = key_row(p.k, p.kst, p.ksh, key);
      if (kr == nullptr) {
        flag_error(p.err, PSB_DEVERR_BLOCK_RANGE);
        live = false;
      } else {
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot = fmaf(q[d], Elem<T>::to_float(kr[d]), dot);
        s = dot * p.scale_log2;
      }
    }
    float mx = s;
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float m_new = fmaxf(m, mx);
    const float alpha = m == -INFINITY ? 0.f : exp2f(m - m_new);
    const float pr = live && m_new != -INFINITY ? exp2f(s - m_new) : 0.f;
    float psum = pr;
#pragma unroll
    for (int o = 16; o; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l = l * alpha + psum;
    const float prr = Elem<T>::to_float(Elem<T>::from_float(pr));
#pragma unroll
    for (int i = 0; i < kMaxDimPerLane; ++i) acc[i] *= alpha;
    const int nk = min(32, last - k0 + 1);
    for (int j = 0; j < nk; ++j) {
      const float pj = __shfl_sync(0xffffffffu, prr, j);
      const T* vr = key_row(p.v, p.vst, p.vsh, k0 + j);
      if (vr == nullptr) continue;  // a block outside the pool (flagged above)
#pragma unroll
      for (int i = 0; i < kMaxDimPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc[i] = fmaf(pj, Elem<T>::to_float(vr[d]), acc[i]);
      }
    }
    m = m_new;
  }
  T* op = reinterpret_cast<T*>(p.out) + row * p.ost + qh * p.osh;
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int i = 0; i < kMaxDimPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < D) op[d] = Elem<T>::from_float(acc[i] * inv);
  }
}

template <typename T, bool PAGED>
int launch_generic(const PrefillParams& p, cudaStream_t s) {
  const int64_t tasks = static_cast<int64_t>(p.total) * p.hq;
  const int64_t blocks = (tasks + kGenThreads / 32 - 1) / (kGenThreads / 32);
  if (blocks == 0) return PSB_OK;
  if (blocks >= (int64_t(1) << 31)) return PSB_ERR_UNSUPPORTED;
  const size_t smem = sizeof(float) * (kGenThreads / 32) * p.head_dim;
  discard_stale_error();
  prefill_generic_kernel<T, PAGED><<<static_cast<unsigned>(blocks), kGenThreads, smem, s>>>(p);
  return check_launch();
}

// cu_seqlens sanity (non-decreasing, within [0, total]) on the device, so a
// malformed batch is reported instead of read out of bounds.
__global__ void check_seqlens_kernel(const int32_t* cu, int32_t n, int32_t total, int32_t* err) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int a = cu[i], b = cu[i + 1];
    if (a < 0 || b < a || b > total || (i == 0 && a != 0)) flag_error(err, PSB_DEVERR_SEQLENS);
  }
}

}  // namespace
}  // namespace psb

using namespace psb;

extern "C" int psb_varlen_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                                  int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                                  int64_t v_stride_h, void* out, int64_t o_stride_t, int64_t o_stride_h,
                                  const int32_t* cu_seqlens, int32_t num_seqs, int32_t total_tokens,
                                  int32_t max_seqlen, int32_t q_heads, int32_t num_kv_heads, int32_t head_dim,
                                  int32_t dtype, float scale, int32_t* error_flag, psb_stream_t stream) {
  if (num_seqs < 0 || total_tokens < 0 || max_seqlen < 0 || q_heads <= 0 || num_kv_heads <= 0 ||
      q_heads % num_kv_heads || head_dim <= 0 || head_dim > 32 * kMaxDimPerLane)
    return PSB_ERR_INVALID;
  if (dtype != PSB_F32 && dtype != PSB_F16 && dtype != PSB_BF16) return PSB_ERR_INVALID;
  if (num_seqs == 0 || total_tokens == 0) return PSB_OK;
  if (!q || !k || !v || !out || !cu_seqlens) return PSB_ERR_INVALID;
  PrefillParams p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.qst = q_stride_t;
  p.qsh = q_stride_h;
  p.kst = k_stride_t;
  p.ksh = k_stride_h;
  p.vst = v_stride_t;
  p.vsh = v_stride_h;
  p.ost = o_stride_t;
  p.osh = o_stride_h;
  p.cu = cu_seqlens;
  p.num_seqs = num_seqs;
  p.total = total_tokens;
  p.max_seqlen = max_seqlen;
  p.hq = q_heads;
  p.hkv = num_kv_heads;
  p.head_dim = head_dim;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = error_flag;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (error_flag != nullptr) {
    discard_stale_error();
    check_seqlens_kernel<<<1, 256, 0, s>>>(cu_seqlens, num_seqs, total_tokens, error_flag);
  }
  if (prefill_tc_supported(p, dtype)) return prefill_tc_launch(p, dtype, s);
  switch (dtype) {
    case PSB_BF16: return launch_generic<__nv_bfloat16, false>(p, s);
    case PSB_F16: return launch_generic<__half, false>(p, s);
    default: return launch_generic<float, false>(p, s);
  }
}

extern "C" int psb_paged_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache,
                                 const void* v_cache, const int32_t* block_tables, int64_t table_stride,
                                 const int32_t* context_lens, void* out, int64_t o_stride_t, int64_t o_stride_h,
                                 const int32_t* cu_seqlens, int32_t num_seqs, int32_t total_tokens,
                                 int32_t max_seqlen, int32_t max_context, int32_t q_heads, int32_t layer,
                                 int32_t num_layers, int64_t num_blocks, int32_t num_kv_heads, int32_t block_size,
                                 int32_t head_dim, int32_t dtype, float scale, int32_t* error_flag,
                                 psb_stream_t stream) {
  if (num_seqs < 0 || total_tokens < 0 || max_seqlen < 0 || max_context < max_seqlen || q_heads <= 0 ||
      num_kv_heads <= 0 || q_heads % num_kv_heads || head_dim <= 0 || head_dim > 32 * kMaxDimPerLane ||
      num_layers <= 0 || layer < 0 || layer >= num_layers || num_blocks <= 0 || block_size <= 0 ||
      table_stride < (max_context + block_size - 1) / block_size)
    return PSB_ERR_INVALID;
  if (dtype != PSB_F32 && dtype != PSB_F16 && dtype != PSB_BF16) return PSB_ERR_INVALID;
  if (static_cast<int64_t>(num_layers) * num_blocks * num_kv_heads >= (int64_t(1) << 31)) return PSB_ERR_UNSUPPORTED;
  if (num_seqs == 0 || total_tokens == 0) return PSB_OK;
  if (!q || !k_cache || !v_cache || !out || !cu_seqlens || !block_tables || !context_lens) return PSB_ERR_INVALID;
  PrefillParams p;
  p.q = q;
  p.k = k_cache;
  p.v = v_cache;
  p.out = out;
  p.qst = q_stride_t;
  p.qsh = q_stride_h;
  p.kst = p.ksh = p.vst = p.vsh = 0;
  p.ost = o_stride_t;
  p.osh = o_stride_h;
  p.cu = cu_seqlens;
  p.num_seqs = num_seqs;
  p.total = total_tokens;
  p.max_seqlen = max_seqlen;
  p.hq = q_heads;
  p.hkv = num_kv_heads;
  p.head_dim = head_dim;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = error_flag;
  p.paged = true;
  p.tables = block_tables;
  p.table_stride = table_stride;
  p.ctx = context_lens;
  p.layer = layer;
  p.num_layers_total = num_layers;
  p.block_size = block_size;
  p.max_context = max_context;
  p.num_blocks = num_blocks;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (error_flag != nullptr) {
    discard_stale_error();
    check_seqlens_kernel<<<1, 256, 0, s>>>(cu_seqlens, num_seqs, total_tokens, error_flag);
  }
  if (prefill_tc_supported(p, dtype)) return prefill_tc_launch(p, dtype, s);
  switch (dtype) {
    case PSB_BF16: return launch_generic<__nv_bfloat16, true>(p, s);
    case PSB_F16: return launch_generic<__half, true>(p, s);
    default: return launch_generic<float, true>(p, s);
  }
}
