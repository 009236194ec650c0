// rope_reshape_and_cache: the rotary position embedding of q and k fused with
// the slot-mapped K/V write, one launch per layer.
//
// Replaces, in the reference's decode glue, the transformers Qwen2
// ``apply_rotary_pos_emb`` (imported at
// pagedserve/attention/batched_paged_attention.py:8, applied at :105-112)
// followed by the per-row ``write_token`` loop (:115-124):
//     q' = q * cos + rotate_half(q) * sin,  k' likewise,
//     rotate_half(x) = cat(-x[D/2:], x[:D/2]),
//     cache[layer, slot / BS, h, slot % BS, :] = k'[t, h, :]  (and v[t, h, :]).
// cos/sin are the caller's per-token rows (the engine's position embeddings,
// pagedserve/model/engine.py:572-575), so the angles are the reference's own.
// Every product and the sum are evaluated in fp32 and rounded to the storage
// type, as PyTorch evaluates that expression on bf16/f16 tensors, so q', k'
// and the pool bytes are bit-identical to the reference's (for bf16/f16 the
// kernel uses paired 16-bit multiplies and adds, which round identically; see
// Pair below).  A thread rotates one VEC-element piece of each half of one
// head (the two halves meet in the rotation), or of two heads of one role,
// 16-byte accesses when rows allow.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "host_util.h"

namespace psb {
namespace {

struct RopeParams {
  const char* q;
  int64_t qst, qsh;  // bytes
  char* qo;
  int64_t qost, qosh;
  const char* k;
  int64_t kst, ksh;
  char* ko;  // may be null
  int64_t kost, kosh;
  const char* v;
  int64_t vst, vsh;
  const char* cos;
  const char* sin;
  int64_t cst;
  char* kc;
  char* vc;
  const int64_t* slots;
  int32_t tokens, hq, hkv, block_size, head_dim;
  int64_t layer_base_tiles, pool_slots;
  int32_t* err;
};

// VEC consecutive elements, moved as one 16-byte access when VEC * sizeof(T) == 16
template <typename T, int VEC>
struct Piece {
  alignas(VEC * sizeof(T) == 16 ? 16 : alignof(T)) T e[VEC];
  __device__ __forceinline__ void load(const char* src) {
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(e) = __ldg(reinterpret_cast<const uint4*>(src));
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) e[i] = reinterpret_cast<const T*>(src)[i];
    }
  }
  __device__ __forceinline__ void store(char* dst) const {
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(e);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) reinterpret_cast<T*>(dst)[i] = e[i];
    }
  }
};

// x rounded to T and back (the identity for fp32)
template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return Elem<T>::to_float(Elem<T>::from_float(x));
}

// Packed pairs for the 16-bit types.  A paired multiply or add rounds the
// exact result once, to nearest even; PyTorch computes the same operation in
// fp32 and rounds that to the 16-bit type.  The two agree: the product of two
// 16-bit values is exact in fp32, and an fp32 sum of two 16-bit values is
// inexact only when their magnitudes differ by more than 2^16 (bf16) / 2^13
// (f16), where both give the larger operand.
// The operations are written as PTX with an explicit .rn rounding modifier,
// which the compiler never contracts into a fused multiply-add.
template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  __device__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ static uint32_t add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};
template <> struct Pair<__half> {
  __device__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  __device__ static uint32_t add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};

// first half: x1 cos - x2 sin; second half: x2 cos + x1 sin; each product and
// the sum rounded to T
template <typename T, int VEC>
__device__ __forceinline__ void rotate(const Piece<T, VEC>& x1, const Piece<T, VEC>& x2, const Piece<T, VEC>& c1,
                                       const Piece<T, VEC>& c2, const Piece<T, VEC>& s1, const Piece<T, VEC>& s2,
                                       Piece<T, VEC>& o1, Piece<T, VEC>& o2) {
  if constexpr (!std::is_same<T, float>::value && VEC % 2 == 0) {
    using P = Pair<T>;
    const uint32_t* a = reinterpret_cast<const uint32_t*>(x1.e);
    const uint32_t* b = reinterpret_cast<const uint32_t*>(x2.e);
    const uint32_t* cc1 = reinterpret_cast<const uint32_t*>(c1.e);
    const uint32_t* cc2 = reinterpret_cast<const uint32_t*>(c2.e);
    const uint32_t* ss1 = reinterpret_cast<const uint32_t*>(s1.e);
    const uint32_t* ss2 = reinterpret_cast<const uint32_t*>(s2.e);
#pragma unroll
    for (int j = 0; j < VEC / 2; ++j) {
      const uint32_t nb = b[j] ^ 0x80008000u;  // -x2: both sign bits flipped, exact
      reinterpret_cast<uint32_t*>(o1.e)[j] = P::add(P::mul(a[j], cc1[j]), P::mul(nb, ss1[j]));
      reinterpret_cast<uint32_t*>(o2.e)[j] = P::add(P::mul(b[j], cc2[j]), P::mul(a[j], ss2[j]));
    }
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float a = Elem<T>::to_float(x1.e[j]), b = Elem<T>::to_float(x2.e[j]);
      o1.e[j] = Elem<T>::from_float(__fadd_rn(rnd<T>(__fmul_rn(a, Elem<T>::to_float(c1.e[j]))),
                                              rnd<T>(__fmul_rn(-b, Elem<T>::to_float(s1.e[j])))));
      o2.e[j] = Elem<T>::from_float(__fadd_rn(rnd<T>(__fmul_rn(b, Elem<T>::to_float(c2.e[j]))),
                                              rnd<T>(__fmul_rn(a, Elem<T>::to_float(s2.e[j])))));
    }
  }
}

// Idx: int32 when the unit count fits (the common case: cheap index
// arithmetic), int64 otherwise.  (Giving a thread a run of heads that share
// the token's cos/sin and slot measured slower: 23.5 against 21.1 us on a
// 16 K-token pack.)
template <typename T, int VEC, typename Idx>
__global__ void __launch_bounds__(256) rope_cache_kernel(const RopeParams p) {
  // a programmatic dependent, like reshape_and_cache: the next kernel may
  // launch now; this one waits for its predecessor before touching memory
  pdl_launch_dependents();
  pdl_wait();
  const int half = p.head_dim / 2;
  const int pieces = half / VEC;
  const int heads = p.hq + 2 * p.hkv;
  const Idx per_tok = static_cast<Idx>(heads) * pieces;
  const Idx total = per_tok * p.tokens;
  const int64_t hb = static_cast<int64_t>(half) * sizeof(T);  // byte offset of the second half
  for (Idx i = blockIdx.x * static_cast<Idx>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<Idx>(gridDim.x) * blockDim.x) {
    const Idx t = i / per_tok;
    const int r = static_cast<int>(i - t * per_tok);
    const int hs = r / pieces;
    const int64_t e0 = static_cast<int64_t>(r - hs * pieces) * VEC * sizeof(T);  // byte offset in the first half
    const bool is_q = hs < p.hq, is_k = !is_q && hs < p.hq + p.hkv;
    // the pool slot (keys and values only)
    int64_t dst = -1;
    if (!is_q) {
      const int h = is_k ? hs - p.hq : hs - p.hq - p.hkv;
      const int64_t s = __ldg(p.slots + t);
      if (s >= p.pool_slots) {
        if (h == 0 && e0 == 0 && is_k) flag_error(p.err, PSB_DEVERR_SLOT_RANGE);
      } else if (s >= 0) {
        const int64_t blk = s / p.block_size, off = s - blk * p.block_size;
        dst = (((p.layer_base_tiles + blk * p.hkv + h) * p.block_size + off) * p.head_dim) * sizeof(T) + e0;
      }
    }
    if (!is_q && !is_k) {  // value: copied unchanged
      if (dst < 0) continue;
      const char* src = p.v + t * p.vst + (hs - p.hq - p.hkv) * p.vsh + e0;
      Piece<T, VEC> a, b;
      a.load(src);
      b.load(src + hb);
      a.store(p.vc + dst);
      b.store(p.vc + dst + hb);
      continue;
    }
    const int h = is_q ? hs : hs - p.hq;
    const char* src = is_q ? p.q + t * p.qst + h * p.qsh + e0 : p.k + t * p.kst + h * p.ksh + e0;
    const char* cs = p.cos + t * p.cst + e0;
    const char* sn = p.sin + t * p.cst + e0;
    Piece<T, VEC> x1, x2, c1, c2, s1, s2;
    x1.load(src);
    x2.load(src + hb);
    c1.load(cs);
    c2.load(cs + hb);
    s1.load(sn);
    s2.load(sn + hb);
    Piece<T, VEC> o1, o2;
    rotate<T, VEC>(x1, x2, c1, c2, s1, s2, o1, o2);
    if (is_q) {
      char* out = p.qo + t * p.qost + h * p.qosh + e0;
      o1.store(out);
      o2.store(out + hb);
      continue;
    }
    if (p.ko != nullptr) {
      char* out = p.ko + t * p.kost + h * p.kosh + e0;
      o1.store(out);
      o2.store(out + hb);
    }
    if (dst >= 0) {
      o1.store(p.kc + dst);
      o2.store(p.kc + dst + hb);
    }
  }
}

// Two heads of one role (q, k or v) per unit: the same piece of heads 2m and
// 2m + 1 of one token, both heads' loads issued before any arithmetic and
// the token's cos/sin pieces loaded once for the two (64 bytes of q/k/v in
// flight per thread instead of 32 at the same occupancy: 19.3 -> 18.0-18.8 us
// on a 16 K-token pack).  Used when the q and kv head counts are both even,
// so that no pair straddles two roles.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) rope_pair_kernel(const RopeParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int half = p.head_dim / 2;
  const int pieces = half / VEC;
  const int pairs = (p.hq + 2 * p.hkv) / 2;
  const int per_tok = pairs * pieces;
  const int64_t total = static_cast<int64_t>(per_tok) * p.tokens;
  const int64_t hb = static_cast<int64_t>(half) * sizeof(T);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / per_tok;
    const int r = static_cast<int>(i - t * per_tok);
    const int pr = r / pieces;
    const int64_t e0 = static_cast<int64_t>(r - pr * pieces) * VEC * sizeof(T);
    const int hs = 2 * pr;  // first head of the pair (both of one role: the host checks even head counts)
    const bool is_q = hs < p.hq, is_k = !is_q && hs < p.hq + p.hkv;
    const int h = is_q ? hs : (is_k ? hs - p.hq : hs - p.hq - p.hkv);
    const char* src = is_q ? p.q + t * p.qst + h * p.qsh + e0
                           : (is_k ? p.k + t * p.kst + h * p.ksh + e0 : p.v + t * p.vst + h * p.vsh + e0);
    const int64_t hst = is_q ? p.qsh : (is_k ? p.ksh : p.vsh);
    Piece<T, VEC> xa1, xa2, xb1, xb2;
    xa1.load(src);
    xa2.load(src + hb);
    xb1.load(src + hst);
    xb2.load(src + hst + hb);
    int64_t dst = -1;  // pool row of head h (head h + 1's row is block_size * head_dim elements on)
    if (!is_q) {
      const int64_t sl = __ldg(p.slots + t);
      if (sl >= p.pool_slots) {
        if (is_k && h == 0 && e0 == 0) flag_error(p.err, PSB_DEVERR_SLOT_RANGE);
      } else if (sl >= 0) {
        const int64_t blk = sl / p.block_size, off = sl - blk * p.block_size;
        dst = (((p.layer_base_tiles + blk * p.hkv + h) * p.block_size + off) * p.head_dim) * sizeof(T) + e0;
      }
    }
    const int64_t pool_head = static_cast<int64_t>(p.block_size) * p.head_dim * sizeof(T);
    if (!is_q && !is_k) {
      if (dst < 0) continue;
      xa1.store(p.vc + dst);
      xa2.store(p.vc + dst + hb);
      xb1.store(p.vc + dst + pool_head);
      xb2.store(p.vc + dst + pool_head + hb);
      continue;
    }
    Piece<T, VEC> c1, c2, s1, s2;
    const char* cs = p.cos + t * p.cst + e0;
    const char* sn = p.sin + t * p.cst + e0;
    c1.load(cs);
    c2.load(cs + hb);
    s1.load(sn);
    s2.load(sn + hb);
    Piece<T, VEC> oa1, oa2, ob1, ob2;
    rotate<T, VEC>(xa1, xa2, c1, c2, s1, s2, oa1, oa2);
    rotate<T, VEC>(xb1, xb2, c1, c2, s1, s2, ob1, ob2);
    if (is_q) {
      char* out = p.qo + t * p.qost + h * p.qosh + e0;
      oa1.store(out);
      oa2.store(out + hb);
      ob1.store(out + p.qosh);
      ob2.store(out + p.qosh + hb);
      continue;
    }
    if (p.ko != nullptr) {
      char* out = p.ko + t * p.kost + h * p.kosh + e0;
      oa1.store(out);
      oa2.store(out + hb);
      ob1.store(out + p.kosh);
      ob2.store(out + p.kosh + hb);
    }
    if (dst >= 0) {
      oa1.store(p.kc + dst);
      oa2.store(p.kc + dst + hb);
      ob1.store(p.kc + dst + pool_head);
      ob2.store(p.kc + dst + pool_head + hb);
    }
  }
}

template <typename T, int VEC>
int launch_rope_pair(const RopeParams& p, cudaStream_t s, int sms) {
  const auto kern = rope_pair_kernel<T, VEC>;
  int occ = 0;
  if (!kernel_occupancy(reinterpret_cast<const void*>(kern), 256, 0, &occ)) return PSB_ERR_CUDA;
  if (!prefer_max_l1(reinterpret_cast<const void*>(kern))) return PSB_ERR_CUDA;
  const int64_t units = static_cast<int64_t>(p.tokens) * ((p.hq + 2 * p.hkv) / 2) * (p.head_dim / 2 / VEC);
  const int64_t blocks =
      std::max<int64_t>(1, std::min<int64_t>((units + 255) / 256, static_cast<int64_t>(sms) * std::min(std::max(occ, 1), 8)));
  discard_stale_error();
  const cudaError_t e = launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, p);
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}

template <typename T, int VEC>
int launch_rope(const RopeParams& p, cudaStream_t s, int sms) {
  const int64_t units = static_cast<int64_t>(p.tokens) * (p.hq + 2 * p.hkv) * (p.head_dim / 2 / VEC);
  // int32 indices while every index and the grid stride past the last one fit
  const auto kern = units + static_cast<int64_t>(sms) * 8 * 256 < (int64_t(1) << 31) ? rope_cache_kernel<T, VEC, int32_t>
                                                                                     : rope_cache_kernel<T, VEC, int64_t>;
  int occ = 0;
  if (!kernel_occupancy(reinterpret_cast<const void*>(kern), 256, 0, &occ)) return PSB_ERR_CUDA;
  // no shared memory: the L1 holds the loads in flight (measured 10 % faster
  // on the 16K-token pack than under the full shared-memory carve-out)
  if (!prefer_max_l1(reinterpret_cast<const void*>(kern))) return PSB_ERR_CUDA;
  // one wave of resident CTAs striding over the units: no partial second wave
  // (an index plus the stride stays below 2^31 with at most 8 CTAs per SM)
  const int64_t blocks =
      std::max<int64_t>(1, std::min<int64_t>((units + 255) / 256, static_cast<int64_t>(sms) * std::min(std::max(occ, 1), 8)));
  discard_stale_error();
  const cudaError_t e = launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, p);
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}

bool aligned16(const void* ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; }

}  // namespace
}  // namespace psb

using namespace psb;

extern "C" int psb_rope_reshape_and_cache(const void* query, int64_t q_stride_t, int64_t q_stride_h, void* query_out,
                                          int64_t qo_stride_t, int64_t qo_stride_h, const void* key,
                                          int64_t k_stride_t, int64_t k_stride_h, void* key_out, int64_t ko_stride_t,
                                          int64_t ko_stride_h, const void* value, int64_t v_stride_t,
                                          int64_t v_stride_h, const void* cos, const void* sin,
                                          int64_t cs_stride_t, void* k_cache, void* v_cache,
                                          const int64_t* slot_mapping, int32_t num_tokens, int32_t num_q_heads,
                                          int32_t layer, int32_t num_layers, int64_t num_blocks,
                                          int32_t num_kv_heads, int32_t block_size, int32_t head_dim, int32_t dtype,
                                          int32_t* error_flag, psb_stream_t stream) {
  if (num_tokens < 0 || num_q_heads < 0 || num_layers <= 0 || layer < 0 || layer >= num_layers ||
      num_blocks <= 0 || num_kv_heads <= 0 || block_size <= 0 || head_dim <= 0 || head_dim % 2)
    return PSB_ERR_INVALID;
  if (dtype != PSB_F32 && dtype != PSB_F16 && dtype != PSB_BF16) return PSB_ERR_INVALID;
  if (num_tokens == 0) return PSB_OK;
  if (!key || !value || !cos || !sin || !k_cache || !v_cache || !slot_mapping) return PSB_ERR_INVALID;
  if (num_q_heads > 0 && (!query || !query_out)) return PSB_ERR_INVALID;
  const int esz = elem_bytes(dtype);
  RopeParams p;
  p.q = static_cast<const char*>(query);
  p.qst = q_stride_t * esz;
  p.qsh = q_stride_h * esz;
  p.qo = static_cast<char*>(query_out);
  p.qost = qo_stride_t * esz;
  p.qosh = qo_stride_h * esz;
  p.k = static_cast<const char*>(key);
  p.kst = k_stride_t * esz;
  p.ksh = k_stride_h * esz;
  p.ko = static_cast<char*>(key_out);
  p.kost = ko_stride_t * esz;
  p.kosh = ko_stride_h * esz;
  p.v = static_cast<const char*>(value);
  p.vst = v_stride_t * esz;
  p.vsh = v_stride_h * esz;
  p.cos = static_cast<const char*>(cos);
  p.sin = static_cast<const char*>(sin);
  p.cst = cs_stride_t * esz;
  p.kc = static_cast<char*>(k_cache);
  p.vc = static_cast<char*>(v_cache);
  p.slots = slot_mapping;
  p.tokens = num_tokens;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.block_size = block_size;
  p.head_dim = head_dim;
  p.layer_base_tiles = static_cast<int64_t>(layer) * num_blocks * num_kv_heads;
  p.pool_slots = num_blocks * block_size;
  p.err = error_flag;
  const int sms = device_sm_count();
  if (sms <= 0) return PSB_ERR_CUDA;
  // 16-byte pieces when every row, stride and half-row is 16-byte aligned
  const int64_t half_bytes = static_cast<int64_t>(head_dim / 2) * esz;
  bool vec = half_bytes % 16 == 0 && aligned16(key) && aligned16(value) && aligned16(cos) && aligned16(sin) &&
             aligned16(k_cache) && aligned16(v_cache) && p.kst % 16 == 0 && p.ksh % 16 == 0 && p.vst % 16 == 0 &&
             p.vsh % 16 == 0 && p.cst % 16 == 0;
  if (num_q_heads > 0)
    vec = vec && aligned16(query) && aligned16(query_out) && p.qst % 16 == 0 && p.qsh % 16 == 0 &&
          p.qost % 16 == 0 && p.qosh % 16 == 0;
  if (key_out != nullptr) vec = vec && aligned16(key_out) && p.kost % 16 == 0 && p.kosh % 16 == 0;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (vec && num_q_heads % 2 == 0 && num_kv_heads % 2 == 0) {
    switch (dtype) {
      case PSB_BF16: return launch_rope_pair<__nv_bfloat16, 8>(p, s, sms);
      case PSB_F16: return launch_rope_pair<__half, 8>(p, s, sms);
      default: return launch_rope_pair<float, 4>(p, s, sms);
    }
  }
  switch (dtype) {
    case PSB_BF16: return vec ? launch_rope<__nv_bfloat16, 8>(p, s, sms) : launch_rope<__nv_bfloat16, 1>(p, s, sms);
    case PSB_F16: return vec ? launch_rope<__half, 8>(p, s, sms) : launch_rope<__half, 1>(p, s, sms);
    default: return vec ? launch_rope<float, 4>(p, s, sms) : launch_rope<float, 1>(p, s, sms);
  }
}
