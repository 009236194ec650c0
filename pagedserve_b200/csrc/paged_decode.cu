// Paged GQA decode attention for B200 (sm_100a).
//
// Replaces PagedServe's Triton decode kernel
// (pagedserve/attention/triton_paged_decode.py:10-95) with the numerics of its
// PyTorch reference (pagedserve/attention/vectorized_batched_attention.py:79-159).
//
// Work decomposition.  A "unit" is (sequence b, kv head h, context chunk c).
// Every CTA of a persistent grid first scans context_lens into a per-sequence
// chunk prefix in shared memory, then walks units u = blockIdx.x, +gridDim.x, ...
// Units are numbered u = (chunk_prefix[b] + c) * Hkv + h.  Sequences shorter
// than one chunk finish in their single unit; longer ones write an fp32
// partial (running max, sum, unnormalised output) to the workspace and the
// last CTA to arrive for (b, h) - found with an atomic counter, no waiting -
// merges the partials in the same launch.
//
// Fast path (bf16/f16, head_dim 64, block_size 16, up to 8 q heads per kv
// head): 4 warps per CTA, each owns up to 4 pool blocks (64 tokens) of the
// 256-token chunk.  Each warp's lane 0 pulls its K and V tiles (one
// 16 x 64 tile per (layer, block, kv head), 2 KiB, contiguous in the pool)
// into shared memory with TMA, 128-byte swizzled, completion on an mbarrier.
// All q heads of the kv head sit in one m16n8k16 A fragment (rows = q heads),
// so every K/V byte leaves HBM exactly once; QK^T and PV run on the tensor
// pipe with fp32 accumulation, the softmax max/sum are quad shuffles.
// Probabilities are rounded to the cache dtype before P.V, as the reference
// does (vectorized_batched_attention.py:152-156).
//
// Generic path (fp32, or any other geometry): CUDA-core kernel with the same
// unit decomposition and the same split-K finish, 64-token chunks.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "host_util.h"

namespace psb {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kFastChunk = 256;        // tokens per split-K unit, fast path
constexpr int kFastBlocksPerWarp = 4;  // 4 x 16 tokens
constexpr int kTileBytes = 16 * 64 * 2;
constexpr int kFastMaxGroup = 8;
constexpr int kGenericChunk = 64;

struct DecodeParams {
  const char* q;
  int64_t qsb, qsh;  // elements
  char* out;
  int64_t osb, osh;
  const char* k_cache;
  const char* v_cache;
  const int32_t* tables;
  int64_t table_stride;
  const int32_t* ctx;
  int32_t batch, hq, hkv, group, layer, num_layers_total, block_size, head_dim, max_context, chunk;
  int64_t num_blocks;
  float scale_log2;  // scale * log2(e)
  float* part_o;     // [max_units, group, head_dim]
  float* part_ml;    // [max_units, group, 2]
  int32_t* counters; // [batch * hkv]
  int64_t max_units;
  int32_t* err;
};

// ---------------------------------------------------------------------------
// unit bookkeeping shared by both kernels
// ---------------------------------------------------------------------------

__device__ __forceinline__ int clamp_ctx(const DecodeParams& p, int b) {
  int n = p.ctx[b];
  if (n < 0 || n > p.max_context) {
    flag_error(p.err, PSB_DEVERR_CONTEXT);
    n = n < 0 ? 0 : p.max_context;
  }
  return n;
}

// Exclusive prefix over sequences of max(1, ceil(ctx / chunk)); returns total
// chunk count (units = total * hkv).  Called by all threads of the CTA.
__device__ int build_chunk_prefix(const DecodeParams& p, int32_t* prefix) {
  __shared__ int32_t warp_sums[kWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (p.batch + kThreads - 1) / kThreads;
  const int begin = min(tid * per, p.batch), end = min(begin + per, p.batch);
  int local = 0;
  for (int b = begin; b < end; ++b) {
    const int n = clamp_ctx(p, b);
    local += n <= 0 ? 1 : (n + p.chunk - 1) / p.chunk;
  }
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += warp_sums[w];
  int run = base + incl - local;
  for (int b = begin; b < end; ++b) {
    prefix[b] = run;
    const int n = clamp_ctx(p, b);
    run += n <= 0 ? 1 : (n + p.chunk - 1) / p.chunk;
  }
  int total = 0;
  for (int w = 0; w < kWarps; ++w) total += warp_sums[w];
  if (tid == 0) prefix[p.batch] = total;
  __syncthreads();
  return total;
}

// Largest b with prefix[b] <= sc.
__device__ __forceinline__ int find_seq(const int32_t* prefix, int batch, int sc) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= sc) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <typename T>
__device__ __forceinline__ void store_out(const DecodeParams& p, int b, int qh, int d, float v) {
  T* o = reinterpret_cast<T*>(p.out) + b * p.osb + qh * p.osh + d;
  *o = Elem<T>::from_float(v);
}

// Finish a unit whose merged state (raw-score max m, sum l, unnormalised o)
// is in shared memory: write the output directly, or write a partial and let
// the last arriving CTA of (b, h) merge all partials.
template <typename T>
__device__ void finish_unit(const DecodeParams& p, int b, int h, int c, int nch, int64_t u, int64_t u_first,
                            const float* s_m, const float* s_l, const float* s_o, float* s_scratch) {
  const int G = p.group, D = p.head_dim, tid = threadIdx.x;
  if (nch == 1) {
    for (int i = tid; i < G * D; i += kThreads) {
      const int g = i / D, d = i - g * D;
      const float l = s_l[g];
      store_out<T>(p, b, h * G + g, d, l > 0.f ? s_o[i] / l : 0.f);
    }
    return;
  }
  __shared__ int s_last;
  if (u >= p.max_units) {  // cannot happen with a correctly sized workspace
    if (tid == 0) flag_error(p.err, PSB_DEVERR_WORKSPACE);
    return;
  }
  float* po = p.part_o + u * G * D;
  float* pml = p.part_ml + u * G * 2;
  for (int i = tid; i < G * D; i += kThreads) po[i] = s_o[i];
  for (int g = tid; g < G; g += kThreads) {
    pml[2 * g] = s_m[g];
    pml[2 * g + 1] = s_l[g];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(p.counters + b * p.hkv + h, 1);
    s_last = (old == nch - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // s_scratch: [G] max, [G] 1/sum
  float* s_M = s_scratch;
  float* s_R = s_scratch + G;
  for (int g = tid; g < G; g += kThreads) {
    float M = -INFINITY;
    for (int cc = 0; cc < nch; ++cc) {
      const int64_t uc = u_first + static_cast<int64_t>(cc) * p.hkv;
      M = fmaxf(M, __ldcg(p.part_ml + uc * G * 2 + 2 * g));
    }
    float L = 0.f;
    if (M != -INFINITY) {
      for (int cc = 0; cc < nch; ++cc) {
        const int64_t uc = u_first + static_cast<int64_t>(cc) * p.hkv;
        const float m = __ldcg(p.part_ml + uc * G * 2 + 2 * g);
        const float l = __ldcg(p.part_ml + uc * G * 2 + 2 * g + 1);
        L += l * exp2f((m - M) * p.scale_log2);
      }
    }
    s_M[g] = M;
    s_R[g] = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D;
    const float M = s_M[g];
    float acc = 0.f;
    if (M != -INFINITY) {
      for (int cc = 0; cc < nch; ++cc) {
        const int64_t uc = u_first + static_cast<int64_t>(cc) * p.hkv;
        const float m = __ldcg(p.part_ml + uc * G * 2 + 2 * g);
        if (m == -INFINITY) continue;
        acc += __ldcg(p.part_o + uc * G * D + i) * exp2f((m - M) * p.scale_log2);
      }
    }
    store_out<T>(p, b, h * G + g, i - g * D, acc * s_R[g]);
  }
  if (tid == 0) p.counters[b * p.hkv + h] = 0;
  (void)c;
}

// ---------------------------------------------------------------------------
// fast path: TMA + mma.sync, bf16/f16, D = 64, block_size = 16, group <= 8
// ---------------------------------------------------------------------------
struct FastSmem {
  // tiles: [warp][K: 4 tiles][V: 4 tiles], 1024-byte aligned base
  static constexpr int kWarpBytes = 2 * kFastBlocksPerWarp * kTileBytes;  // 16 KiB
  static constexpr int kTilesBytes = kWarps * kWarpBytes;                   // 64 KiB
  static constexpr int kMergeFloats = kWarps * kFastMaxGroup * (64 + 2);
  static constexpr int kFinFloats = kFastMaxGroup * (64 + 2) + 2 * kFastMaxGroup;
  static size_t bytes(int batch) {
    return 1024 /*align slack*/ + kTilesBytes + sizeof(float) * (kMergeFloats + kFinFloats) +
           sizeof(uint64_t) * 2 * kWarps + sizeof(int32_t) * (batch + 1);
  }
};

template <typename T>
__global__ void __launch_bounds__(kThreads) decode_fast_kernel(const __grid_constant__ CUtensorMap kmap,
                                                               const __grid_constant__ CUtensorMap vmap,
                                                               const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* s_merge = reinterpret_cast<float*>(tiles + FastSmem::kTilesBytes);
  float* s_mo = s_merge;                                         // [warp][8][64]
  float* s_mm = s_merge + kWarps * kFastMaxGroup * 64;           // [warp][8]
  float* s_ml = s_mm + kWarps * kFastMaxGroup;                   // [warp][8]
  float* s_fo = s_merge + FastSmem::kMergeFloats;                // [8][64]
  float* s_fm = s_fo + kFastMaxGroup * 64;                       // [8]
  float* s_fl = s_fm + kFastMaxGroup;                            // [8]
  float* s_scr = s_fl + kFastMaxGroup;                           // [16]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_merge + FastSmem::kMergeFloats + FastSmem::kFinFloats);
  int32_t* prefix = reinterpret_cast<int32_t*>(bars + 2 * kWarps);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.group;
  uint64_t* kbar = bars + 2 * warp;
  uint64_t* vbar = kbar + 1;
  uint8_t* ktiles = tiles + warp * FastSmem::kWarpBytes;
  uint8_t* vtiles = ktiles + kFastBlocksPerWarp * kTileBytes;

  if (lane == 0) {
    mbar_init(kbar, 1);
    mbar_init(vbar, 1);
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
  }
  fence_barrier_init();
  const int total_chunks = build_chunk_prefix(p, prefix);  // includes __syncthreads
  const int64_t total_units = static_cast<int64_t>(total_chunks) * p.hkv;
  uint32_t phase = 0;
  bool failed = false;
  const uint64_t policy = l2_policy_evict_first();

  for (int64_t u = blockIdx.x; u < total_units && !failed; u += gridDim.x) {
    const int sc = static_cast<int>(u / p.hkv);
    const int h = static_cast<int>(u - static_cast<int64_t>(sc) * p.hkv);
    const int b = find_seq(prefix, p.batch, sc);
    const int c = sc - prefix[b];
    const int nch = prefix[b + 1] - prefix[b];
    const int ctx = clamp_ctx(p, b);
    const int wtok0 = c * kFastChunk + warp * (kFastBlocksPerWarp * 16);
    const int wn = max(0, min(kFastBlocksPerWarp * 16, ctx - wtok0));
    const int nblk = (wn + 15) >> 4;

    // ---- issue this warp's TMA loads -----------------------------------
    uint32_t valid_mask = 0;
    {
      int32_t blk = -1;
      if (lane < nblk) {
        blk = p.tables[b * p.table_stride + (wtok0 >> 4) + lane];
        if (blk < 0 || blk >= p.num_blocks) {
          flag_error(p.err, PSB_DEVERR_BLOCK_RANGE);
          blk = -1;
        }
      }
      valid_mask = __ballot_sync(0xffffffffu, blk >= 0) & ((1u << nblk) - 1u);
      if (lane == 0 && valid_mask != 0) {
        const uint32_t bytes = __popc(valid_mask) * kTileBytes;
        mbar_arrive_expect_tx(kbar, bytes);
        mbar_arrive_expect_tx(vbar, bytes);
      }
      __syncwarp();
      if (lane < nblk && blk >= 0) {
        fence_proxy_async_smem();  // order this warp's earlier generic reads of the buffers before the copy
        const int32_t z = static_cast<int32_t>((static_cast<int64_t>(p.layer) * p.num_blocks + blk) * p.hkv + h);
        tma_load_3d_hint(ktiles + lane * kTileBytes, &kmap, 0, 0, z, kbar, policy);
        tma_load_3d_hint(vtiles + lane * kTileBytes, &vmap, 0, 0, z, vbar, policy);
      }
    }

    // ---- q fragments (rows = q heads of this kv head) ------------------
    uint32_t qa0[4], qa2[4];
    {
      const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.qsb + (h * G + g) * p.qsh;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        if (g < G) {
          qa0[ks] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t);
          qa2[ks] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t);
        } else {
          qa0[ks] = 0u;
          qa2[ks] = 0u;
        }
      }
    }

    float mx = -INFINITY, lsum = 0.f;
    float o[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    if (valid_mask != 0) {
      if (!mbar_wait(kbar, phase)) {
        flag_error(p.err, PSB_DEVERR_TIMEOUT);
        failed = true;
      }
    }
    // ---- S = Q K^T ------------------------------------------------------
    float s[kFastBlocksPerWarp][2][4];
#pragma unroll
    for (int j = 0; j < kFastBlocksPerWarp; ++j) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[j][nt][0] = s[j][nt][1] = s[j][nt][2] = s[j][nt][3] = 0.f;
        if ((valid_mask >> j) & 1u) {
          const uint32_t tile = smem_u32(ktiles + j * kTileBytes);
          const int tok = nt * 8 + (lane & 7);
#pragma unroll
          for (int kp = 0; kp < 2; ++kp) {
            const int chunk = kp * 4 + (lane >> 3);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(tile + tok * 128 + ((chunk ^ (tok & 7)) << 4), b0, b1, b2, b3);
            mma_16816<T>(s[j][nt], qa0[2 * kp], 0u, qa2[2 * kp], 0u, b0, b1);
            mma_16816<T>(s[j][nt], qa0[2 * kp + 1], 0u, qa2[2 * kp + 1], 0u, b2, b3);
          }
        }
      }
    }
    // mask + row max
#pragma unroll
    for (int j = 0; j < kFastBlocksPerWarp; ++j) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = j * 16 + nt * 8 + 2 * t + e;
          const bool ok = tk < wn && ((valid_mask >> j) & 1u);
          s[j][nt][e] = ok ? s[j][nt][e] : -INFINITY;
          mx = fmaxf(mx, s[j][nt][e]);
        }
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mxs = mx == -INFINITY ? 0.f : mx * p.scale_log2;

    if (valid_mask != 0 && !failed) {
      if (!mbar_wait(vbar, phase)) {
        flag_error(p.err, PSB_DEVERR_TIMEOUT);
        failed = true;
      }
    }
    // ---- O = P V ----------------------------------------------------------
#pragma unroll
    for (int j = 0; j < kFastBlocksPerWarp; ++j) {
      float pr[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float sv = s[j][nt][e];
          pr[nt][e] = sv == -INFINITY ? 0.f : exp2f(fmaf(sv, p.scale_log2, -mxs));
          lsum += pr[nt][e];
        }
      }
      if ((valid_mask >> j) & 1u) {
        const uint32_t pa0 = pack2<T>(pr[0][0], pr[0][1]);
        const uint32_t pa2 = pack2<T>(pr[1][0], pr[1][1]);
        const uint32_t tile = smem_u32(vtiles + j * kTileBytes);
        const int tok = ((lane >> 3) & 1) * 8 + (lane & 7);
        const int valid_in_block = wn - j * 16;  // >= 1 here
        // token coverage of this thread's B fragments: b0 -> 2t, 2t+1 ; b1 -> 8+2t, 8+2t+1
        uint32_t keep0 = 0xffffffffu, keep1 = 0xffffffffu;
        if (valid_in_block < 16) {
          keep0 = (2 * t < valid_in_block ? 0x0000ffffu : 0u) | (2 * t + 1 < valid_in_block ? 0xffff0000u : 0u);
          keep1 = (8 + 2 * t < valid_in_block ? 0x0000ffffu : 0u) |
                  (8 + 2 * t + 1 < valid_in_block ? 0xffff0000u : 0u);
        }
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {
          const int chunk = dp * 2 + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(tile + tok * 128 + ((chunk ^ (tok & 7)) << 4), b0, b1, b2, b3);
          mma_16816<T>(o[2 * dp], pa0, 0u, pa2, 0u, b0 & keep0, b1 & keep1);
          mma_16816<T>(o[2 * dp + 1], pa0, 0u, pa2, 0u, b2 & keep0, b3 & keep1);
        }
      }
    }
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
    if (valid_mask != 0) phase ^= 1u;

    // ---- merge the 4 warps ---------------------------------------------
    {
      float* mo = s_mo + (warp * kFastMaxGroup + g) * 64;
#pragma unroll
      for (int n = 0; n < 8; ++n) *reinterpret_cast<float2*>(mo + n * 8 + 2 * t) = make_float2(o[n][0], o[n][1]);
      if (t == 0) {
        s_mm[warp * kFastMaxGroup + g] = mx;
        s_ml[warp * kFastMaxGroup + g] = lsum;
      }
    }
    if (__syncthreads_or(failed ? 1 : 0)) {
      failed = true;
      break;
    }
    for (int i = tid; i < G * 64; i += kThreads) {
      const int gg = i >> 6, d = i & 63;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_mm[w * kFastMaxGroup + gg]);
      float L = 0.f, acc = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          const float m = s_mm[w * kFastMaxGroup + gg];
          if (m == -INFINITY) continue;
          const float wt = exp2f((m - M) * p.scale_log2);
          L += s_ml[w * kFastMaxGroup + gg] * wt;
          acc += s_mo[(w * kFastMaxGroup + gg) * 64 + d] * wt;
        }
      }
      s_fo[i] = acc;
      if (d == 0) {
        s_fm[gg] = M;
        s_fl[gg] = L;
      }
    }
    __syncthreads();
    const int64_t u_first = static_cast<int64_t>(prefix[b]) * p.hkv + h;
    finish_unit<T>(p, b, h, c, nch, u, u_first, s_fm, s_fl, s_fo, s_scr);
    __syncthreads();
  }
  // A failed wait leaves copies possibly in flight into this CTA's shared
  // memory: give them one more bounded chance to land before exiting.
  if (failed && lane == 0) {
    mbar_wait(kbar, phase);
    mbar_wait(vbar, phase);
  }
}

// ---------------------------------------------------------------------------
// generic path: CUDA cores, any dtype / head_dim / block_size / group
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) decode_generic_kernel(const DecodeParams p) {
  extern __shared__ float gsm[];
  const int G = p.group, D = p.head_dim, BS = p.block_size, tid = threadIdx.x;
  const int ldk = D + 1;
  float* q_s = gsm;                        // [G][D]
  float* kv_s = q_s + G * D;               // [64][D+1]
  float* sc_s = kv_s + kGenericChunk * ldk;  // [G][64]
  float* m_s = sc_s + G * kGenericChunk;   // [G]
  float* l_s = m_s + G;                    // [G]
  float* o_s = l_s + G;                    // [G][D]
  float* scr = o_s + G * D;                // [2G]
  int32_t* prefix = reinterpret_cast<int32_t*>(scr + 2 * G);

  const int total_chunks = build_chunk_prefix(p, prefix);
  const int64_t total_units = static_cast<int64_t>(total_chunks) * p.hkv;
  const int64_t layer_base = static_cast<int64_t>(p.layer) * p.num_blocks;

  for (int64_t u = blockIdx.x; u < total_units; u += gridDim.x) {
    const int sc = static_cast<int>(u / p.hkv);
    const int h = static_cast<int>(u - static_cast<int64_t>(sc) * p.hkv);
    const int b = find_seq(prefix, p.batch, sc);
    const int c = sc - prefix[b];
    const int nch = prefix[b + 1] - prefix[b];
    const int ctx = clamp_ctx(p, b);
    const int tok0 = c * kGenericChunk;
    const int ntok = max(0, min(kGenericChunk, ctx - tok0));

    for (int i = tid; i < G * D; i += kThreads) {
      const int g = i / D, d = i - g * D;
      q_s[i] = Elem<T>::to_float(reinterpret_cast<const T*>(p.q)[b * p.qsb + (h * G + g) * p.qsh + d]);
    }
    // K rows of this chunk -> fp32 shared; rows past the context and rows of
    // out-of-range blocks are zero (and masked below)
    auto load_rows = [&](const char* pool) {
      for (int i = tid; i < kGenericChunk * D; i += kThreads) {
        const int r = i / D, d = i - r * D;
        float v = 0.f;
        if (r < ntok) {
          const int pos = tok0 + r;
          const int blk = p.tables[b * p.table_stride + pos / BS];
          if (blk >= 0 && blk < p.num_blocks) {
            const int64_t off = (((layer_base + blk) * p.hkv + h) * BS + pos % BS) * D + d;
            v = Elem<T>::to_float(reinterpret_cast<const T*>(pool)[off]);
          } else if (d == 0) {
            flag_error(p.err, PSB_DEVERR_BLOCK_RANGE);
          }
        }
        kv_s[r * ldk + d] = v;
      }
    };
    load_rows(p.k_cache);
    __syncthreads();
    for (int i = tid; i < G * kGenericChunk; i += kThreads) {
      const int g = i / kGenericChunk, r = i - g * kGenericChunk;
      float acc = -INFINITY;
      if (r < ntok) {
        const int pos = tok0 + r;
        const int blk = p.tables[b * p.table_stride + pos / BS];
        if (blk >= 0 && blk < p.num_blocks) {
          acc = 0.f;
          for (int d = 0; d < D; ++d) acc = fmaf(q_s[g * D + d], kv_s[r * ldk + d], acc);
        }
      }
      sc_s[i] = acc;
    }
    __syncthreads();
    // per-row max / probabilities / sum, one warp per q head
    for (int g = tid >> 5; g < G; g += kWarps) {
      const int lane = tid & 31;
      float mx = -INFINITY;
      for (int r = lane; r < kGenericChunk; r += 32) mx = fmaxf(mx, sc_s[g * kGenericChunk + r]);
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mxs = mx == -INFINITY ? 0.f : mx * p.scale_log2;
      float sum = 0.f;
      for (int r = lane; r < kGenericChunk; r += 32) {
        const float sv = sc_s[g * kGenericChunk + r];
        const float pr = sv == -INFINITY ? 0.f : exp2f(fmaf(sv, p.scale_log2, -mxs));
        sum += pr;
        // probabilities are rounded to the cache dtype before P.V, as the reference does
        sc_s[g * kGenericChunk + r] = Elem<T>::to_float(Elem<T>::from_float(pr));
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        m_s[g] = mx;
        l_s[g] = sum;
      }
    }
    __syncthreads();
    load_rows(p.v_cache);
    __syncthreads();
    for (int i = tid; i < G * D; i += kThreads) {
      const int g = i / D, d = i - g * D;
      float acc = 0.f;
      for (int r = 0; r < ntok; ++r) acc = fmaf(sc_s[g * kGenericChunk + r], kv_s[r * ldk + d], acc);
      o_s[i] = acc;
    }
    __syncthreads();
    const int64_t u_first = static_cast<int64_t>(prefix[b]) * p.hkv + h;
    finish_unit<T>(p, b, h, c, nch, u, u_first, m_s, l_s, o_s, scr);
    __syncthreads();
  }
}

size_t generic_smem_bytes(int group, int head_dim, int batch) {
  return sizeof(float) * (static_cast<size_t>(group) * head_dim * 2 + kGenericChunk * (head_dim + 1) +
                          static_cast<size_t>(group) * kGenericChunk + 4 * group) +
         sizeof(int32_t) * (batch + 1);
}

bool fast_path_ok(int dtype, int head_dim, int block_size, int group) {
  return (dtype == PSB_BF16 || dtype == PSB_F16) && head_dim == 64 && block_size == 16 && group <= kFastMaxGroup;
}

int64_t max_units_for(int batch, int hkv, int max_context, int chunk) {
  const int64_t per = std::max<int64_t>(1, (static_cast<int64_t>(max_context) + chunk - 1) / chunk);
  return per * batch * hkv;
}

struct WorkspaceLayout {
  size_t counters_off, ml_off, o_off, total;
};

WorkspaceLayout workspace_layout(int batch, int hkv, int group, int head_dim, int64_t max_units) {
  WorkspaceLayout w;
  w.counters_off = 0;
  w.ml_off = align_up(sizeof(int32_t) * static_cast<size_t>(batch) * hkv, 256);
  w.o_off = align_up(w.ml_off + sizeof(float) * static_cast<size_t>(max_units) * group * 2, 256);
  w.total = w.o_off + sizeof(float) * static_cast<size_t>(max_units) * group * head_dim;
  return w;
}

template <typename T>
int launch_decode(DecodeParams prm, bool fast, cudaStream_t stream) {
  const int sms = device_sm_count();
  if (sms <= 0) return PSB_ERR_CUDA;
  const int64_t upper_units = prm.max_units;
  if constexpr (!std::is_same<T, float>::value) {
    if (fast) {
    const size_t smem = FastSmem::bytes(prm.batch);
    if (smem > 227 * 1024) return PSB_ERR_UNSUPPORTED;
    const void* kern = reinterpret_cast<const void*>(decode_fast_kernel<T>);
    int occ = 0;
    if (!kernel_occupancy(kern, kThreads, smem, &occ)) return PSB_ERR_CUDA;
    CUtensorMap kmap, vmap;
    const int64_t pool_tiles = static_cast<int64_t>(prm.num_layers_total) * prm.num_blocks * prm.hkv;
    if (!encode_pool_tile_map(&kmap, prm.k_cache, pool_tiles, prm.block_size, prm.head_dim,
                              dtype_to_tmap(Elem<T>::code)) ||
        !encode_pool_tile_map(&vmap, prm.v_cache, pool_tiles, prm.block_size, prm.head_dim,
                              dtype_to_tmap(Elem<T>::code)))
      return PSB_ERR_CUDA;
    const int64_t grid = std::min<int64_t>(upper_units, static_cast<int64_t>(sms) * std::max(occ, 1));
    decode_fast_kernel<T><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(kmap, vmap, prm);
    return check_launch();
    }
  }
  const size_t smem = generic_smem_bytes(prm.group, prm.head_dim, prm.batch);
  if (smem > 227 * 1024) return PSB_ERR_UNSUPPORTED;
  const void* kern = reinterpret_cast<const void*>(decode_generic_kernel<T>);
  int occ = 0;
  if (!kernel_occupancy(kern, kThreads, smem, &occ)) return PSB_ERR_CUDA;
  const int64_t grid = std::min<int64_t>(upper_units, static_cast<int64_t>(sms) * std::max(occ, 1));
  decode_generic_kernel<T><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(prm);
  return check_launch();
}

}  // namespace
}  // namespace psb

using namespace psb;

extern "C" size_t psb_paged_decode_workspace_size(int32_t batch, int32_t q_heads, int32_t num_kv_heads,
                                                  int32_t head_dim, int32_t block_size, int32_t max_context,
                                                  int32_t dtype) {
  if (batch <= 0 || num_kv_heads <= 0 || q_heads <= 0 || q_heads % num_kv_heads || head_dim <= 0 ||
      max_context < 0)
    return 0;
  const int group = q_heads / num_kv_heads;
  const int chunk = fast_path_ok(dtype, head_dim, block_size, group) ? kFastChunk : kGenericChunk;
  const int64_t mu = max_units_for(batch, num_kv_heads, max_context, chunk);
  return workspace_layout(batch, num_kv_heads, group, head_dim, mu).total;
}

extern "C" int psb_paged_decode_workspace_init(void* workspace, size_t workspace_bytes, int32_t batch,
                                               int32_t num_kv_heads, psb_stream_t stream) {
  const size_t need = sizeof(int32_t) * static_cast<size_t>(batch) * num_kv_heads;
  if (workspace == nullptr || batch <= 0 || num_kv_heads <= 0) return PSB_ERR_INVALID;
  if (workspace_bytes < need) return PSB_ERR_WORKSPACE;
  const cudaError_t e = cudaMemsetAsync(workspace, 0, need, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return PSB_ERR_CUDA;
  }
  return PSB_OK;
}

extern "C" int psb_paged_decode(const void* query, int64_t q_stride_b, int64_t q_stride_h, void* out,
                                int64_t o_stride_b, int64_t o_stride_h, const void* k_cache, const void* v_cache,
                                const int32_t* block_tables, int64_t table_stride, const int32_t* context_lens,
                                int32_t batch, int32_t q_heads, int32_t layer, int32_t num_layers,
                                int64_t num_blocks, int32_t num_kv_heads, int32_t block_size, int32_t head_dim,
                                int32_t dtype, int32_t max_context, float scale, void* workspace,
                                size_t workspace_bytes, int32_t* error_flag, psb_stream_t stream) {
  if (!query || !out || !k_cache || !v_cache || !block_tables || !context_lens) return PSB_ERR_INVALID;
  if (batch <= 0 || q_heads <= 0 || num_kv_heads <= 0 || q_heads % num_kv_heads || head_dim <= 0 ||
      block_size <= 0 || num_blocks <= 0 || num_layers <= 0 || layer < 0 || layer >= num_layers ||
      max_context < 0 || table_stride < (max_context + block_size - 1) / block_size)
    return PSB_ERR_INVALID;
  if (dtype != PSB_F32 && dtype != PSB_F16 && dtype != PSB_BF16) return PSB_ERR_INVALID;
  const int group = q_heads / num_kv_heads;
  const bool fast = fast_path_ok(dtype, head_dim, block_size, group) && q_stride_h % 2 == 0 &&
                    q_stride_b % 2 == 0 && reinterpret_cast<uintptr_t>(query) % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(k_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(v_cache) % 16 == 0;
  const int chunk = fast ? kFastChunk : kGenericChunk;
  const int64_t mu = max_units_for(batch, num_kv_heads, max_context, chunk);
  const WorkspaceLayout wl = workspace_layout(batch, num_kv_heads, group, head_dim, mu);
  if (workspace == nullptr || workspace_bytes < wl.total) return PSB_ERR_WORKSPACE;
  if (static_cast<int64_t>(num_layers) * num_blocks * num_kv_heads >= (int64_t(1) << 31)) return PSB_ERR_UNSUPPORTED;

  DecodeParams p;
  p.q = static_cast<const char*>(query);
  p.qsb = q_stride_b;
  p.qsh = q_stride_h;
  p.out = static_cast<char*>(out);
  p.osb = o_stride_b;
  p.osh = o_stride_h;
  p.k_cache = static_cast<const char*>(k_cache);
  p.v_cache = static_cast<const char*>(v_cache);
  p.tables = block_tables;
  p.table_stride = table_stride;
  p.ctx = context_lens;
  p.batch = batch;
  p.hq = q_heads;
  p.hkv = num_kv_heads;
  p.group = group;
  p.layer = layer;
  p.num_layers_total = num_layers;
  p.block_size = block_size;
  p.head_dim = head_dim;
  p.max_context = max_context;
  p.chunk = chunk;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * 1.4426950408889634f;
  char* ws = static_cast<char*>(workspace);
  p.counters = reinterpret_cast<int32_t*>(ws + wl.counters_off);
  p.part_ml = reinterpret_cast<float*>(ws + wl.ml_off);
  p.part_o = reinterpret_cast<float*>(ws + wl.o_off);
  p.max_units = mu;
  p.err = error_flag;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PSB_BF16: return launch_decode<__nv_bfloat16>(p, fast, s);
    case PSB_F16: return launch_decode<__half>(p, fast, s);
    default: return launch_decode<float>(p, false, s);
  }
}
