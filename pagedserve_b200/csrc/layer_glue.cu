// Elementwise glue of a Qwen2 decoder layer around the attention hot path:
// the residual add fused with RMSNorm, and SiLU(gate) * up.
//
// The reference's model runner calls these through transformers' Qwen2
// modules once per layer (pagedserve/model/engine.py:577-596 for a decode
// step, :628-646 for a prefill): ``residual + attention_output``, then
// ``post_attention_layernorm``, ``mlp`` (act_fn(gate_proj(x)) * up_proj(x)),
// ``residual + mlp_output``, and the next layer's ``input_layernorm``.  Each
// is several small PyTorch kernels; here each is one launch, so a captured
// decode iteration is bounded by its weight and KV streams, not by launches.
//
// Roundings follow PyTorch's evaluation of the same expressions on 16-bit
// tensors: the residual sum is formed in fp32 and rounded to the storage
// type; RMSNorm squares and averages the rounded sum in fp32, scales by
// rsqrt(mean + eps), rounds, then multiplies by the weight and rounds again
// (Qwen2RMSNorm: ``weight * hidden.to(input_dtype)``); SiLU is evaluated in
// fp32 and rounded before the product with ``up``, which is rounded again.
// Only the order of the fp32 sum of squares differs from PyTorch's.
#include <algorithm>

#include "common.cuh"
#include "host_util.h"

namespace psb {
namespace {

constexpr int kGlueThreads = 256;

template <typename T, int VEC>
struct Pack {
  T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ Pack<T, VEC> load_pack(const T* p) {
  Pack<T, VEC> r;
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(r.v) = __ldg(reinterpret_cast<const uint4*>(p));
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) r.v[i] = p[i];
  }
  return r;
}

template <typename T, int VEC>
__device__ __forceinline__ void store_pack(T* p, const Pack<T, VEC>& r) {
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(r.v);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) p[i] = r.v[i];
  }
}

// One warp per row.  Pass 1 forms the (rounded) residual sum, stores it and
// accumulates its squares; pass 2 re-reads the row this lane wrote (an L1
// hit), normalises it and applies the weight.
template <typename T, int VEC>
__global__ void __launch_bounds__(kGlueThreads) add_rms_norm_kernel(
    const T* __restrict__ x, int64_t xs, T* residual, int64_t rs, const T* __restrict__ weight, T* __restrict__ out,
    int64_t os, int32_t rows, int32_t hidden, float eps) {
  const int warp = static_cast<int>((blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int nvec = hidden / VEC;
  const T* xr = x + static_cast<int64_t>(warp) * xs;
  T* rr = residual != nullptr ? residual + static_cast<int64_t>(warp) * rs : nullptr;
  float ss = 0.f;
  for (int i = lane; i < nvec; i += 32) {
    Pack<T, VEC> a = load_pack<T, VEC>(xr + i * VEC);
    if (rr != nullptr) {
      const Pack<T, VEC> b = load_pack<T, VEC>(rr + i * VEC);
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        a.v[j] = Elem<T>::from_float(Elem<T>::to_float(a.v[j]) + Elem<T>::to_float(b.v[j]));
      store_pack<T, VEC>(rr + i * VEC, a);
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float f = Elem<T>::to_float(a.v[j]);
      ss = fmaf(f, f, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  const float inv = rsqrtf(ss / static_cast<float>(hidden) + eps);
  const T* src = rr != nullptr ? rr : xr;
  T* dst = out + static_cast<int64_t>(warp) * os;
  for (int i = lane; i < nvec; i += 32) {
    Pack<T, VEC> a = rr != nullptr ? *reinterpret_cast<const Pack<T, VEC>*>(src + i * VEC)
                                   : load_pack<T, VEC>(src + i * VEC);
    const Pack<T, VEC> w = load_pack<T, VEC>(weight + i * VEC);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const T n = Elem<T>::from_float(Elem<T>::to_float(a.v[j]) * inv);
      a.v[j] = Elem<T>::from_float(Elem<T>::to_float(w.v[j]) * Elem<T>::to_float(n));
    }
    store_pack<T, VEC>(dst + i * VEC, a);
  }
}

// One CTA of kRowThreads per row, each thread holding up to MAXV vectors of
// the row in registers: every load (x, residual, weight) is issued before
// the first use, and one block-wide sum replaces the warp's serial passes.
constexpr int kRowThreads = 128;

template <typename T, int VEC, int MAXV>
__global__ void __launch_bounds__(kRowThreads) add_rms_norm_row_kernel(
    const T* __restrict__ x, int64_t xs, T* residual, int64_t rs, const T* __restrict__ weight, T* __restrict__ out,
    int64_t os, int32_t hidden, float eps) {
  __shared__ float s_part[kRowThreads / 32];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nvec = hidden / VEC;
  const T* xr = x + static_cast<int64_t>(row) * xs;
  T* rr = residual != nullptr ? residual + static_cast<int64_t>(row) * rs : nullptr;
  Pack<T, VEC> a[MAXV], w[MAXV];
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = tid + k * kRowThreads;
    if (i < nvec) {
      a[k] = load_pack<T, VEC>(xr + i * VEC);
      w[k] = load_pack<T, VEC>(weight + i * VEC);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = tid + k * kRowThreads;
    if (i < nvec) {
      if (rr != nullptr) {
        const Pack<T, VEC> b = *reinterpret_cast<const Pack<T, VEC>*>(rr + i * VEC);
#pragma unroll
        for (int j = 0; j < VEC; ++j)
          a[k].v[j] = Elem<T>::from_float(Elem<T>::to_float(a[k].v[j]) + Elem<T>::to_float(b.v[j]));
        store_pack<T, VEC>(rr + i * VEC, a[k]);
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = Elem<T>::to_float(a[k].v[j]);
        ss = fmaf(f, f, ss);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  if ((tid & 31) == 0) s_part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kRowThreads / 32; ++i) tot += s_part[i];
  const float inv = rsqrtf(tot / static_cast<float>(hidden) + eps);
  T* dst = out + static_cast<int64_t>(row) * os;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = tid + k * kRowThreads;
    if (i < nvec) {
      Pack<T, VEC> o;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const T n = Elem<T>::from_float(Elem<T>::to_float(a[k].v[j]) * inv);
        o.v[j] = Elem<T>::from_float(Elem<T>::to_float(w[k].v[j]) * Elem<T>::to_float(n));
      }
      store_pack<T, VEC>(dst + i * VEC, o);
    }
  }
}

// out[r, j] = round(round(silu(g)) * u), g = gate_up[r, j], u = gate_up[r, inter + j].
template <typename T, int VEC>
__global__ void __launch_bounds__(kGlueThreads) silu_and_mul_kernel(const T* __restrict__ gu, int64_t gs,
                                                                      T* __restrict__ out, int64_t os, int32_t rows,
                                                                      int32_t inter) {
  const int nvec = inter / VEC;
  const int64_t total = static_cast<int64_t>(rows) * nvec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nvec;
    const int c = static_cast<int>(i - r * nvec) * VEC;
    const T* row = gu + r * gs;
    const Pack<T, VEC> g = load_pack<T, VEC>(row + c);
    const Pack<T, VEC> u = load_pack<T, VEC>(row + inter + c);
    Pack<T, VEC> o;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float gf = Elem<T>::to_float(g.v[j]);
      const T s = Elem<T>::from_float(gf / (1.0f + expf(-gf)));
      o.v[j] = Elem<T>::from_float(Elem<T>::to_float(s) * Elem<T>::to_float(u.v[j]));
    }
    store_pack<T, VEC>(out + r * os + c, o);
  }
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

template <typename T>
int launch_add_rms_norm(const void* x, int64_t xs, void* residual, int64_t rs, const void* weight, void* out,
                        int64_t os, int32_t rows, int32_t hidden, float eps, cudaStream_t s) {
  constexpr int VEC = 16 / sizeof(T);
  const bool vec = hidden % VEC == 0 && xs % VEC == 0 && os % VEC == 0 && aligned16(x) && aligned16(weight) &&
                   aligned16(out) && (residual == nullptr || (rs % VEC == 0 && aligned16(residual)));
  discard_stale_error();
  if (vec) {
    // one CTA per row while the row fits the CTA's registers (hidden up to
    // 4096 bf16 / 2048 fp32 elements)
    const int per = (hidden / VEC + kRowThreads - 1) / kRowThreads;
    const T* xt = static_cast<const T*>(x);
    T* rt = static_cast<T*>(residual);
    const T* wt = static_cast<const T*>(weight);
    T* ot = static_cast<T*>(out);
    const unsigned g = static_cast<unsigned>(rows);
    switch (per) {
      case 1: add_rms_norm_row_kernel<T, VEC, 1><<<g, kRowThreads, 0, s>>>(xt, xs, rt, rs, wt, ot, os, hidden, eps);
        return check_launch();
      case 2: add_rms_norm_row_kernel<T, VEC, 2><<<g, kRowThreads, 0, s>>>(xt, xs, rt, rs, wt, ot, os, hidden, eps);
        return check_launch();
      case 3:
      case 4: add_rms_norm_row_kernel<T, VEC, 4><<<g, kRowThreads, 0, s>>>(xt, xs, rt, rs, wt, ot, os, hidden, eps);
        return check_launch();
      default: break;
    }
  }
  const unsigned grid = static_cast<unsigned>((static_cast<int64_t>(rows) * 32 + kGlueThreads - 1) / kGlueThreads);
  if (vec)
    add_rms_norm_kernel<T, VEC><<<grid, kGlueThreads, 0, s>>>(
        static_cast<const T*>(x), xs, static_cast<T*>(residual), rs, static_cast<const T*>(weight),
        static_cast<T*>(out), os, rows, hidden, eps);
  else
    add_rms_norm_kernel<T, 1><<<grid, kGlueThreads, 0, s>>>(static_cast<const T*>(x), xs, static_cast<T*>(residual),
                                                             rs, static_cast<const T*>(weight), static_cast<T*>(out),
                                                             os, rows, hidden, eps);
  return check_launch();
}

template <typename T>
int launch_silu_and_mul(const void* gu, int64_t gs, void* out, int64_t os, int32_t rows, int32_t inter,
                        cudaStream_t s) {
  constexpr int VEC = 16 / sizeof(T);
  const bool vec = inter % VEC == 0 && gs % VEC == 0 && os % VEC == 0 && aligned16(gu) && aligned16(out);
  const int64_t items = static_cast<int64_t>(rows) * (vec ? inter / VEC : inter);
  const int sms = device_sm_count();
  if (sms <= 0) return PSB_ERR_CUDA;
  const unsigned grid = static_cast<unsigned>(
      std::max<int64_t>(1, std::min<int64_t>((items + kGlueThreads - 1) / kGlueThreads, int64_t(sms) * 8)));
  discard_stale_error();
  if (vec)
    silu_and_mul_kernel<T, VEC><<<grid, kGlueThreads, 0, s>>>(static_cast<const T*>(gu), gs, static_cast<T*>(out), os,
                                                               rows, inter);
  else
    silu_and_mul_kernel<T, 1><<<grid, kGlueThreads, 0, s>>>(static_cast<const T*>(gu), gs, static_cast<T*>(out), os,
                                                             rows, inter);
  return check_launch();
}

}  // namespace
}  // namespace psb

using namespace psb;

extern "C" int psb_add_rms_norm(const void* x, int64_t x_stride, void* residual, int64_t residual_stride,
                                const void* weight, void* out, int64_t out_stride, int32_t rows, int32_t hidden,
                                float eps, int32_t dtype, psb_stream_t stream) {
  if (!x || !weight || !out || rows < 0 || hidden <= 0 || x_stride < hidden || out_stride < hidden ||
      (residual != nullptr && residual_stride < hidden) || !(eps >= 0.f))
    return PSB_ERR_INVALID;
  if (rows == 0) return PSB_OK;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PSB_BF16:
      return launch_add_rms_norm<__nv_bfloat16>(x, x_stride, residual, residual_stride, weight, out, out_stride, rows,
                                                hidden, eps, s);
    case PSB_F16:
      return launch_add_rms_norm<__half>(x, x_stride, residual, residual_stride, weight, out, out_stride, rows, hidden,
                                         eps, s);
    case PSB_F32:
      return launch_add_rms_norm<float>(x, x_stride, residual, residual_stride, weight, out, out_stride, rows, hidden,
                                        eps, s);
    default:
      return PSB_ERR_INVALID;
  }
}

extern "C" int psb_silu_and_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                                int32_t rows, int32_t intermediate, int32_t dtype, psb_stream_t stream) {
  if (!gate_up || !out || rows < 0 || intermediate <= 0 || gate_up_stride < 2 * static_cast<int64_t>(intermediate) ||
      out_stride < intermediate)
    return PSB_ERR_INVALID;
  if (rows == 0) return PSB_OK;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PSB_BF16:
      return launch_silu_and_mul<__nv_bfloat16>(gate_up, gate_up_stride, out, out_stride, rows, intermediate, s);
    case PSB_F16:
      return launch_silu_and_mul<__half>(gate_up, gate_up_stride, out, out_stride, rows, intermediate, s);
    case PSB_F32:
      return launch_silu_and_mul<float>(gate_up, gate_up_stride, out, out_stride, rows, intermediate, s);
    default:
      return PSB_ERR_INVALID;
  }
}
