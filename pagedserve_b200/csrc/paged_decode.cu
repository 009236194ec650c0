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
  int32_t* work;     // [2]: next unit of the work queue, warps done
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

// Clamped context lengths into s_ctx[B] and the exclusive prefix of
// max(1, ceil(ctx / chunk)) into prefix[B + 1]; returns the total chunk count
// (units = total * hkv).  Called by all threads of the CTA.
__device__ int build_chunk_prefix(const DecodeParams& p, int32_t* prefix, int32_t* s_ctx) {
  __shared__ int32_t warp_sums[kWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (p.batch + kThreads - 1) / kThreads;
  const int begin = min(tid * per, p.batch), end = min(begin + per, p.batch);
  int local = 0;
  for (int b = begin; b < end; ++b) {
    const int n = clamp_ctx(p, b);
    s_ctx[b] = n;
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
  int run = incl - local;
  for (int w = 0; w < warp; ++w) run += warp_sums[w];
  for (int b = begin; b < end; ++b) {
    prefix[b] = run;
    const int n = s_ctx[b];
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

struct Unit {
  int b, h, c, nch, ctx;
};

__device__ __forceinline__ Unit decode_unit(const DecodeParams& p, const int32_t* prefix, const int32_t* s_ctx,
                                            int64_t u) {
  Unit w;
  const int sc = static_cast<int>(u / p.hkv);
  w.h = static_cast<int>(u - static_cast<int64_t>(sc) * p.hkv);
  w.b = find_seq(prefix, p.batch, sc);
  w.c = sc - prefix[w.b];
  w.nch = prefix[w.b + 1] - prefix[w.b];
  w.ctx = s_ctx[w.b];
  return w;
}

template <typename T>
__device__ __forceinline__ void store_out(const DecodeParams& p, int b, int qh, int d, float v) {
  T* o = reinterpret_cast<T*>(p.out) + b * p.osb + qh * p.osh + d;
  *o = Elem<T>::from_float(v);
}

// Finish a unit whose merged state (raw-score max s_m[G], sum s_l[G],
// unnormalised output s_o[G*D]) is in shared memory.  A sequence that fits
// one chunk writes its output directly.  Otherwise the unit's partial goes to
// the workspace and the last CTA to arrive for (b, h) - an atomic ticket, no
// waiting - merges all partials of (b, h) in batches of chunks, loading
// them with full memory-level parallelism.  ``scr`` is shared scratch of
// ``scr_cap`` floats; ``s_o`` is reused as the merge accumulator.
template <typename T>
__device__ void finish_unit(const DecodeParams& p, const Unit& w, int64_t u, const float* s_m, const float* s_l,
                            float* s_o, float* scr, int scr_cap) {
  const int G = p.group, D = p.head_dim, tid = threadIdx.x, GD = G * D;
  const bool vec4 = (D & 3) == 0;
  if (w.nch == 1) {
    for (int i = tid; i < GD; i += kThreads) {
      const int g = i / D;
      const float l = s_l[g];
      store_out<T>(p, w.b, w.h * G + g, i - g * D, l > 0.f ? s_o[i] / l : 0.f);
    }
    return;
  }
  __shared__ int s_last;
  if (u >= p.max_units) {  // cannot happen with a correctly sized workspace
    if (tid == 0) flag_error(p.err, PSB_DEVERR_WORKSPACE);
    return;
  }
  {
    float* po = p.part_o + u * GD;
    float* pml = p.part_ml + u * G * 2;
    if (vec4) {
      for (int i = tid; i < GD / 4; i += kThreads)
        reinterpret_cast<float4*>(po)[i] = reinterpret_cast<const float4*>(s_o)[i];
    } else {
      for (int i = tid; i < GD; i += kThreads) po[i] = s_o[i];
    }
    for (int g = tid; g < G; g += kThreads) {
      pml[2 * g] = s_m[g];
      pml[2 * g + 1] = s_l[g];
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(p.counters + w.b * p.hkv + w.h, 1) == w.nch - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  const int64_t u_first = (static_cast<int64_t>(u / p.hkv) - w.c) * p.hkv + w.h;
  float* s_M = scr;              // [G] running max
  float* s_L = scr + G;          // [G] running sum
  float* s_S = scr + 2 * G;      // [G] rescale of the running state
  float* s_pw = scr + 3 * G;     // [CB][G] chunk max -> chunk weight
  const int CB = max(1, (scr_cap - 3 * G) / (2 * G));
  float* s_pl = s_pw + CB * G;   // [CB][G] chunk sums
  float* s_acc = s_o;
  for (int g = tid; g < G; g += kThreads) {
    s_M[g] = -INFINITY;
    s_L[g] = 0.f;
  }
  for (int i = tid; i < GD; i += kThreads) s_acc[i] = 0.f;
  __syncthreads();
  for (int cb = 0; cb < w.nch; cb += CB) {
    const int n = min(CB, w.nch - cb);
    for (int i = tid; i < n * G; i += kThreads) {
      const int c = i / G, g = i - c * G;
      const int64_t uc = u_first + static_cast<int64_t>(cb + c) * p.hkv;
      s_pw[i] = __ldcg(p.part_ml + uc * G * 2 + 2 * g);
      s_pl[i] = __ldcg(p.part_ml + uc * G * 2 + 2 * g + 1);
    }
    __syncthreads();
    for (int g = tid; g < G; g += kThreads) {
      const float mo = s_M[g];
      float mb = mo;
      for (int c = 0; c < n; ++c) mb = fmaxf(mb, s_pw[c * G + g]);
      const float so = (mo == -INFINITY) ? 0.f : exp2f((mo - mb) * p.scale_log2);
      float l = s_L[g] * so;
      for (int c = 0; c < n; ++c) {
        const float m = s_pw[c * G + g];
        const float wt = (m == -INFINITY) ? 0.f : exp2f((m - mb) * p.scale_log2);
        l += s_pl[c * G + g] * wt;
        s_pw[c * G + g] = wt;
      }
      s_M[g] = mb;
      s_L[g] = l;
      s_S[g] = so;
    }
    __syncthreads();
    if (vec4) {
      for (int col = tid; col < GD / 4; col += kThreads) {
        const int g = (col * 4) / D;
        float4 a = reinterpret_cast<float4*>(s_acc)[col];
        const float so = s_S[g];
        a.x *= so; a.y *= so; a.z *= so; a.w *= so;
#pragma unroll 8
        for (int c = 0; c < n; ++c) {
          const int64_t uc = u_first + static_cast<int64_t>(cb + c) * p.hkv;
          const float4 v = __ldcg(reinterpret_cast<const float4*>(p.part_o + uc * GD) + col);
          const float wt = s_pw[c * G + g];
          a.x = fmaf(v.x, wt, a.x); a.y = fmaf(v.y, wt, a.y); a.z = fmaf(v.z, wt, a.z); a.w = fmaf(v.w, wt, a.w);
        }
        reinterpret_cast<float4*>(s_acc)[col] = a;
      }
    } else {
      for (int i = tid; i < GD; i += kThreads) {
        const int g = i / D;
        float a = s_acc[i] * s_S[g];
#pragma unroll 8
        for (int c = 0; c < n; ++c) {
          const int64_t uc = u_first + static_cast<int64_t>(cb + c) * p.hkv;
          a = fmaf(__ldcg(p.part_o + uc * GD + i), s_pw[c * G + g], a);
        }
        s_acc[i] = a;
      }
    }
    __syncthreads();
  }
  for (int i = tid; i < GD; i += kThreads) {
    const int g = i / D;
    const float l = s_L[g];
    store_out<T>(p, w.b, w.h * G + g, i - g * D, l > 0.f ? s_acc[i] / l : 0.f);
  }
  if (tid == 0) p.counters[w.b * p.hkv + w.h] = 0;
}

// ---------------------------------------------------------------------------
// fast path: warp-pipelined TMA + mma.sync (bf16/f16, D = 64, block 16, G <= 8)
// ---------------------------------------------------------------------------
//
// Each warp is an independent stream: it pulls units from a global work
// queue (longest sequences first), keeps kRing pool blocks (K tile + V tile,
// plus the q rows with a unit's first block) in flight in its own shared-
// memory ring, and consumes them one block at a time with an online softmax.
// There are no CTA-wide barriers after the prologue; a finished unit is
// written by the warp that finished it (directly, or as a split-K partial
// merged by the last warp to finish its (sequence, kv head)).
constexpr int kFastWarps = 8;
constexpr int kFastThreads = kFastWarps * 32;
constexpr int kRing = 5;
constexpr int kQBytes = kFastMaxGroup * 64 * 2;            // q rows of one unit
constexpr int kSlotBytes = 2 * kTileBytes + kQBytes;        // K tile, V tile, q rows
constexpr int kLptMaxBatch = 1024;                          // O(B^2) longest-first ranking up to here

struct FastLayout {
  static size_t bytes(int batch) {
    return 1024 + static_cast<size_t>(kFastWarps) * kRing * kSlotBytes + sizeof(uint64_t) * kFastWarps * kRing +
           sizeof(int32_t) * (3 * static_cast<size_t>(batch) + 1) + 64;
  }
};

__device__ __forceinline__ int chunks_of(int ctx, int chunk) { return ctx <= 0 ? 1 : (ctx + chunk - 1) / chunk; }

// s_ctx[b] = clamped context; order[i] = sequence at longest-first position i
// (context length descending, ties by index; natural order above kLptMaxBatch);
// prefix[i] = exclusive prefix of chunk counts along that order.  Every CTA
// computes the same arrays, so unit numbers mean the same thing everywhere.
__device__ int build_lpt_prefix(const DecodeParams& p, int32_t* order, int32_t* prefix, int32_t* s_ctx) {
  __shared__ int32_t warp_sums[kFastWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = p.batch;
  for (int b = tid; b < B; b += kFastThreads) s_ctx[b] = clamp_ctx(p, b);
  __syncthreads();
  if (B <= kLptMaxBatch) {
    // rank by context length, longest first, ties by index
    for (int b = tid; b < B; b += kFastThreads) {
      const int key = s_ctx[b];
      int rank = 0;
      for (int o = 0; o < B; ++o) {
        const int k2 = s_ctx[o];
        rank += (k2 > key) | ((k2 == key) & (o < b));
      }
      order[rank] = b;
    }
  } else {
    for (int b = tid; b < B; b += kFastThreads) order[b] = b;
  }
  __syncthreads();
  const int per = (B + kFastThreads - 1) / kFastThreads;
  const int begin = min(tid * per, B), end = min(begin + per, B);
  int local = 0;
  for (int i = begin; i < end; ++i) local += chunks_of(s_ctx[order[i]], p.chunk);
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
  for (int i = begin; i < end; ++i) {
    prefix[i] = run;
    run += chunks_of(s_ctx[order[i]], p.chunk);
  }
  int total = 0;
  for (int w = 0; w < kFastWarps; ++w) total += warp_sums[w];
  if (tid == 0) prefix[B] = total;
  __syncthreads();
  return total;
}

// Unit u of the longest-first numbering: u = (prefix[i] + c) * hkv + h.
struct FastUnit {
  int b, h, c, nch, ctx, nblk;
};

__device__ __forceinline__ FastUnit fast_unit(const DecodeParams& p, const int32_t* order, const int32_t* prefix,
                                              const int32_t* s_ctx, int u) {
  FastUnit w;
  const int sc = u / p.hkv;
  w.h = u - sc * p.hkv;
  const int i = find_seq(prefix, p.batch, sc);
  w.b = order[i];
  w.c = sc - prefix[i];
  w.nch = prefix[i + 1] - prefix[i];
  w.ctx = s_ctx[w.b];
  w.nblk = max(1, (min(kFastChunk, w.ctx - w.c * kFastChunk) + 15) >> 4);
  return w;
}

// Block ids of one unit: lane j < nblk holds entry j (-1 when out of range).
__device__ __forceinline__ int32_t load_unit_table(const DecodeParams& p, const FastUnit& w, int lane) {
  int32_t blk = -1;
  const int ntok = min(kFastChunk, w.ctx - w.c * kFastChunk);
  if (lane < w.nblk && lane * 16 < ntok) {
    blk = __ldg(p.tables + w.b * p.table_stride + w.c * (kFastChunk / 16) + lane);
    if (blk < 0 || blk >= p.num_blocks) {
      flag_error(p.err, PSB_DEVERR_BLOCK_RANGE);
      blk = -1;
    }
  }
  return blk;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kFastThreads, 1) decode_fast_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                      const __grid_constant__ CUtensorMap vmap,
                                                                      const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring_all = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars_all = reinterpret_cast<uint64_t*>(ring_all + kFastWarps * kRing * kSlotBytes);
  int32_t* order = reinterpret_cast<int32_t*>(bars_all + kFastWarps * kRing);
  int32_t* prefix = order + p.batch;
  int32_t* s_ctx = prefix + p.batch + 1;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.group;
  uint8_t* ring = ring_all + warp * kRing * kSlotBytes;
  uint64_t* full = bars_all + warp * kRing;
  if (lane < kRing) mbar_init(full + lane, 1);
  if (threadIdx.x == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
  }
  fence_barrier_init();
  const int total_units = build_lpt_prefix(p, order, prefix, s_ctx) * p.hkv;  // ends with __syncthreads
  const uint64_t policy = l2_policy_evict_first();
  const int total_warps = gridDim.x * kFastWarps;
  const size_t q_row_bytes = static_cast<size_t>(p.qsh) * sizeof(T);

  auto grab = [&]() -> int {
    int v = 0;
    if (lane == 0) v = atomicAdd(p.work, 1);
    v = __shfl_sync(0xffffffffu, v, 0);
    return v < total_units ? v : -1;
  };

  // ---- issue side --------------------------------------------------------
  int iu = grab();                      // unit whose blocks are being issued
  FastUnit iw{};
  int32_t itab = -1;
  int ib = 0;
  if (iu >= 0) {
    iw = fast_unit(p, order, prefix, s_ctx, iu);
    itab = load_unit_table(p, iw, lane);
  }
  int nu = iu >= 0 ? grab() : -1;       // next unit: decoded, table prefetched
  FastUnit nw{};
  int32_t ntab = -1;
  if (nu >= 0) {
    nw = fast_unit(p, order, prefix, s_ctx, nu);
    ntab = load_unit_table(p, nw, lane);
  }
  uint32_t issued = 0, consumed = 0;
  int32_t meta = 0;     // lane s: flags of ring slot s
  int32_t meta_u = -1;  // lane s: unit of ring slot s
  bool failed = false;

  auto issue_one = [&]() {
    const uint32_t slot = issued % kRing;
    uint8_t* st = ring + slot * kSlotBytes;
    const int32_t blk = __shfl_sync(0xffffffffu, itab, ib);
    const int tok0 = iw.c * kFastChunk + ib * 16;
    const int valid = max(0, min(16, iw.ctx - tok0));
    const bool ok = blk >= 0 && valid > 0;
    const bool first = ib == 0;
    if (lane == 0) {
      fence_proxy_async_smem();  // this warp's earlier reads of the slot precede the new copies
      uint32_t bytes = ok ? 2u * kTileBytes : 0u;
      if (first) bytes += static_cast<uint32_t>(G) * 128u;
      if (bytes) mbar_arrive_expect_tx(full + slot, bytes); else mbar_arrive(full + slot);
      if (ok) {
        const int32_t z = static_cast<int32_t>((static_cast<int64_t>(p.layer) * p.num_blocks + blk) * p.hkv + iw.h);
        tma_load_3d_hint(st, &kmap, 0, 0, z, full + slot, policy);
        tma_load_3d_hint(st + kTileBytes, &vmap, 0, 0, z, full + slot, policy);
      }
      if (first) {
        const char* qsrc = reinterpret_cast<const char*>(p.q) +
                           (static_cast<int64_t>(iw.b) * p.qsb + static_cast<int64_t>(iw.h) * G * p.qsh) * sizeof(T);
        for (int r = 0; r < G; ++r) bulk_g2s(st + 2 * kTileBytes + r * 128, qsrc + r * q_row_bytes, 128, full + slot);
      }
    }
    if (lane == static_cast<int>(slot)) {
      meta = (ok ? 1 : 0) | (valid << 1) | ((first ? 1 : 0) << 6) | ((ib == iw.nblk - 1 ? 1 : 0) << 7);
      meta_u = iu;
    }
    ++issued;
    if (++ib == iw.nblk) {  // advance to the next unit
      iu = nu;
      iw = nw;
      itab = ntab;
      ib = 0;
      if (iu >= 0) {
        nu = grab();
        if (nu >= 0) {
          nw = fast_unit(p, order, prefix, s_ctx, nu);
          ntab = load_unit_table(p, nw, lane);
        }
      }
    }
  };

  while (iu >= 0 && issued - consumed < static_cast<uint32_t>(kRing)) issue_one();

  // ---- consume side ------------------------------------------------------
  uint32_t qa0[4], qa2[4];
  float o[8][4];
  float m_run = -INFINITY, l_run = 0.f;
  FastUnit cw{};
  while (consumed != issued && !failed) {
    const uint32_t slot = consumed % kRing;
    const uint32_t parity = (consumed / kRing) & 1u;
    const int32_t mt = __shfl_sync(0xffffffffu, meta, slot);
    const int cu = __shfl_sync(0xffffffffu, meta_u, slot);
    const bool ok = mt & 1;
    const int valid = (mt >> 1) & 31;
    const bool first = (mt >> 6) & 1, last = (mt >> 7) & 1;
    if (!mbar_wait(full + slot, parity)) {
      flag_error(p.err, PSB_DEVERR_TIMEOUT);
      failed = true;
      break;
    }
    const uint8_t* st = ring + slot * kSlotBytes;
    if (first) {
      cw = fast_unit(p, order, prefix, s_ctx, cu);
      m_run = -INFINITY;
      l_run = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      // A fragments of the q rows (rows >= G are zero)
      const uint32_t qs = smem_u32(st + 2 * kTileBytes);
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        uint32_t r0, r1, r2, r3;
        // matrices: (rows 0-7, dims 32kp + 0..7 | 8..15 | 16..23 | 24..31)
        ldsm_x4(qs + (lane & 7) * 128 + ((kp * 4 + (lane >> 3)) << 4), r0, r1, r2, r3);
        qa0[2 * kp] = g < G ? r0 : 0u;
        qa2[2 * kp] = g < G ? r1 : 0u;
        qa0[2 * kp + 1] = g < G ? r2 : 0u;
        qa2[2 * kp + 1] = g < G ? r3 : 0u;
      }
    }
    if (ok) {
      // ---- S = Q K^T for the 16 tokens of this block -------------------
      float s[2][4];
      const uint32_t ktile = smem_u32(st);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
        const int tok = nt * 8 + (lane & 7);
#pragma unroll
        for (int kp = 0; kp < 2; ++kp) {
          const int chunk = kp * 4 + (lane >> 3);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(ktile + tok * 128 + ((chunk ^ (tok & 7)) << 4), b0, b1, b2, b3);
          mma_16816<T>(s[nt], qa0[2 * kp], 0u, qa2[2 * kp], 0u, b0, b1);
          mma_16816<T>(s[nt], qa0[2 * kp + 1], 0u, qa2[2 * kp + 1], 0u, b2, b3);
        }
      }
      float mb = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = nt * 8 + 2 * t + e;
          s[nt][e] = tk < valid ? s[nt][e] : -INFINITY;
          mb = fmaxf(mb, s[nt][e]);
        }
      }
      mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
      mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
      const float m_new = fmaxf(m_run, mb);
      const float alpha = m_run == -INFINITY ? 0.f : exp2f((m_run - m_new) * p.scale_log2);
      const float ms = m_new * p.scale_log2;
      float pr[2][2];
      float psum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          pr[nt][e] = s[nt][e] == -INFINITY ? 0.f : exp2f(fmaf(s[nt][e], p.scale_log2, -ms));
          psum += pr[nt][e];
        }
      }
      l_run = l_run * alpha + psum;
      m_run = m_new;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        o[n][0] *= alpha;
        o[n][1] *= alpha;
      }
      // ---- O += P V ------------------------------------------------------
      const uint32_t pa0 = pack2<T>(pr[0][0], pr[0][1]);
      const uint32_t pa2 = pack2<T>(pr[1][0], pr[1][1]);
      const uint32_t vtile = smem_u32(st + kTileBytes);
      const int tok = ((lane >> 3) & 1) * 8 + (lane & 7);
      // rows past the context may hold anything (even NaN): zero them
      uint32_t keep0 = 0xffffffffu, keep1 = 0xffffffffu;
      if (valid < 16) {
        keep0 = (2 * t < valid ? 0x0000ffffu : 0u) | (2 * t + 1 < valid ? 0xffff0000u : 0u);
        keep1 = (8 + 2 * t < valid ? 0x0000ffffu : 0u) | (8 + 2 * t + 1 < valid ? 0xffff0000u : 0u);
      }
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        const int chunk = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vtile + tok * 128 + ((chunk ^ (tok & 7)) << 4), b0, b1, b2, b3);
        mma_16816<T>(o[2 * dp], pa0, 0u, pa2, 0u, b0 & keep0, b1 & keep1);
        mma_16816<T>(o[2 * dp + 1], pa0, 0u, pa2, 0u, b2 & keep0, b3 & keep1);
      }
    }
    __syncwarp();
    ++consumed;
    if (iu >= 0) issue_one();  // refill the slot just freed

    if (last) {
      // ---- finish the unit ------------------------------------------------
      float l = l_run;
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      const int qh = cw.h * G + g;
      if (cw.nch == 1) {
        if (g < G) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          T* orow = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(cw.b) * p.osb + static_cast<int64_t>(qh) * p.osh;
#pragma unroll
          for (int n = 0; n < 8; ++n)
            *reinterpret_cast<uint32_t*>(orow + n * 8 + 2 * t) = pack2<T>(o[n][0] * inv, o[n][1] * inv);
        }
      } else {
        const int64_t u = cu;
        float* po = p.part_o + u * G * 64;
        float* pml = p.part_ml + u * G * 2;
        if (g < G) {
#pragma unroll
          for (int n = 0; n < 8; ++n)
            *reinterpret_cast<float2*>(po + g * 64 + n * 8 + 2 * t) = make_float2(o[n][0], o[n][1]);
          if (t == 0) *reinterpret_cast<float2*>(pml + 2 * g) = make_float2(m_run, l);
        }
        __threadfence();
        __syncwarp();
        int prev = 0;
        if (lane == 0) prev = atomicAdd(p.counters + cw.b * p.hkv + cw.h, 1);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == cw.nch - 1) {
          __threadfence();
          const int64_t u_first = (u / p.hkv - cw.c) * p.hkv + cw.h;
          if (g < G) {
            // max and sum over the chunks: each of the 4 lanes of a row takes every 4th chunk
            float M = -INFINITY;
            for (int cc = t; cc < cw.nch; cc += 4)
              M = fmaxf(M, __ldcg(p.part_ml + (u_first + static_cast<int64_t>(cc) * p.hkv) * G * 2 + 2 * g));
            const uint32_t rows = G >= 8 ? 0xffffffffu : ((1u << (4 * G)) - 1u);
            M = fmaxf(M, __shfl_xor_sync(rows, M, 1));
            M = fmaxf(M, __shfl_xor_sync(rows, M, 2));
            float acc[8][2];
#pragma unroll
            for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = 0.f;
            float L = 0.f;
#pragma unroll 4
            for (int cc = 0; cc < cw.nch; ++cc) {
              const int64_t uc = u_first + static_cast<int64_t>(cc) * p.hkv;
              const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml + uc * G * 2 + 2 * g));
              const float wgt = ml.x == -INFINITY ? 0.f : exp2f((ml.x - M) * p.scale_log2);
              L += ml.y * wgt;
              const float* pr = p.part_o + uc * G * 64 + g * 64 + 2 * t;
#pragma unroll
              for (int n = 0; n < 8; ++n) {
                const float2 v = __ldcg(reinterpret_cast<const float2*>(pr + n * 8));
                acc[n][0] = fmaf(v.x, wgt, acc[n][0]);
                acc[n][1] = fmaf(v.y, wgt, acc[n][1]);
              }
            }
            const float inv = L > 0.f ? 1.f / L : 0.f;
            T* orow = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(cw.b) * p.osb + static_cast<int64_t>(qh) * p.osh;
#pragma unroll
            for (int n = 0; n < 8; ++n)
              *reinterpret_cast<uint32_t*>(orow + n * 8 + 2 * t) = pack2<T>(acc[n][0] * inv, acc[n][1] * inv);
          }
          if (lane == 0) p.counters[cw.b * p.hkv + cw.h] = 0;
        }
      }
    }
  }
  if (failed) {
    // copies may still be in flight into this warp's ring: one more bounded
    // chance for each to land before the warp leaves
    for (uint32_t k = consumed; k != issued; ++k) mbar_wait(full + k % kRing, (k / kRing) & 1u);
  }
  // the last warp of the launch leaves the work queue at zero for the next one
  if (lane == 0) {
    if (atomicAdd(p.work + 1, 1) == total_warps - 1) {
      p.work[0] = 0;
      p.work[1] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// generic path: CUDA cores, any dtype / head_dim / block_size / group
// ---------------------------------------------------------------------------
constexpr int kGenericScratch = 1024;  // floats of combine scratch

// Shared-memory carve-up of the generic kernel; every array starts on a
// 16-byte boundary (the split-K finish moves float4s).
struct GenericLayout {
  int q, kv, sc, m, l, o, scr, ints, scr_cap;
  __host__ __device__ static int r4(int x) { return (x + 3) & ~3; }
  __host__ __device__ GenericLayout(int G, int D) {
    scr_cap = kGenericScratch + 6 * G;
    q = 0;
    kv = q + r4(G * D);
    sc = kv + r4(kGenericChunk * (D + 1));
    m = sc + r4(G * kGenericChunk);
    l = m + r4(G);
    o = l + r4(G);
    scr = o + r4(G * D);
    ints = scr + r4(scr_cap);
  }
};

template <typename T>
__global__ void __launch_bounds__(kThreads) decode_generic_kernel(const DecodeParams p) {
  extern __shared__ float4 gsm4[];
  float* gsm = reinterpret_cast<float*>(gsm4);
  const int G = p.group, D = p.head_dim, BS = p.block_size, tid = threadIdx.x;
  const int ldk = D + 1;
  const GenericLayout lay(G, D);
  float* q_s = gsm + lay.q;    // [G][D]
  float* kv_s = gsm + lay.kv;  // [64][D+1]
  float* sc_s = gsm + lay.sc;  // [G][64]
  float* m_s = gsm + lay.m;    // [G]
  float* l_s = gsm + lay.l;    // [G]
  float* o_s = gsm + lay.o;    // [G][D]
  float* scr = gsm + lay.scr;  // combine scratch
  const int scr_cap = lay.scr_cap;
  int32_t* prefix = reinterpret_cast<int32_t*>(gsm + lay.ints);
  int32_t* s_ctx = prefix + p.batch + 1;

  const int total_chunks = build_chunk_prefix(p, prefix, s_ctx);
  const int64_t total_units = static_cast<int64_t>(total_chunks) * p.hkv;
  const int64_t layer_base = static_cast<int64_t>(p.layer) * p.num_blocks;

  for (int64_t u = blockIdx.x; u < total_units; u += gridDim.x) {
    const Unit w = decode_unit(p, prefix, s_ctx, u);
    const int b = w.b, h = w.h;
    const int tok0 = w.c * kGenericChunk;
    const int ntok = max(0, min(kGenericChunk, w.ctx - tok0));

    for (int i = tid; i < G * D; i += kThreads) {
      const int g = i / D, d = i - g * D;
      q_s[i] = Elem<T>::to_float(reinterpret_cast<const T*>(p.q)[b * p.qsb + (h * G + g) * p.qsh + d]);
    }
    // rows of this chunk -> fp32 shared; rows past the context and rows of
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
    finish_unit<T>(p, w, u, m_s, l_s, o_s, scr, scr_cap);
    __syncthreads();
  }
}

size_t generic_smem_bytes(int group, int head_dim, int batch) {
  return sizeof(float) * static_cast<size_t>(GenericLayout(group, head_dim).ints) +
         sizeof(int32_t) * (2 * static_cast<size_t>(batch) + 1);
}

bool fast_path_ok(int dtype, int head_dim, int block_size, int group) {
  return (dtype == PSB_BF16 || dtype == PSB_F16) && head_dim == 64 && block_size == 16 && group <= kFastMaxGroup;
}

int64_t max_units_for(int batch, int hkv, int max_context, int chunk) {
  const int64_t per = std::max<int64_t>(1, (static_cast<int64_t>(max_context) + chunk - 1) / chunk);
  return per * batch * hkv;
}

struct WorkspaceLayout {
  size_t work_off, counters_off, ml_off, o_off, total;
};

// [work queue: 2 x int32 | pad to 256][arrival counters: batch * hkv int32]
// [partial max/sum: max_units * group * 2 f32][partial outputs: max_units * group * head_dim f32]
// Everything before ml_off must be zero before the first launch.
WorkspaceLayout workspace_layout(int batch, int hkv, int group, int head_dim, int64_t max_units) {
  WorkspaceLayout w;
  w.work_off = 0;
  w.counters_off = 256;
  w.ml_off = align_up(w.counters_off + sizeof(int32_t) * static_cast<size_t>(batch) * hkv, 256);
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
      const size_t smem = FastLayout::bytes(prm.batch);
      if (smem > 227 * 1024) return PSB_ERR_UNSUPPORTED;
      const void* kern = reinterpret_cast<const void*>(decode_fast_kernel<T>);
      int occ = 0;
      if (!kernel_occupancy(kern, kFastThreads, smem, &occ) || occ < 1) return PSB_ERR_CUDA;
      CUtensorMap kmap, vmap;
      const int64_t pool_tiles = static_cast<int64_t>(prm.num_layers_total) * prm.num_blocks * prm.hkv;
      if (!encode_pool_tile_map(&kmap, prm.k_cache, pool_tiles, prm.block_size, prm.head_dim,
                                dtype_to_tmap(Elem<T>::code)) ||
          !encode_pool_tile_map(&vmap, prm.v_cache, pool_tiles, prm.block_size, prm.head_dim,
                                dtype_to_tmap(Elem<T>::code)))
        return PSB_ERR_CUDA;
      const int64_t grid = std::min<int64_t>(static_cast<int64_t>(sms) * occ,
                                             (upper_units + kFastWarps - 1) / kFastWarps);
      discard_stale_error();
      decode_fast_kernel<T><<<static_cast<unsigned>(grid), kFastThreads, smem, stream>>>(kmap, vmap, prm);
    return check_launch();
    }
  }
  const size_t smem = generic_smem_bytes(prm.group, prm.head_dim, prm.batch);
  if (smem > 227 * 1024) return PSB_ERR_UNSUPPORTED;
  const void* kern = reinterpret_cast<const void*>(decode_generic_kernel<T>);
  int occ = 0;
  if (!kernel_occupancy(kern, kThreads, smem, &occ)) return PSB_ERR_CUDA;
  const int64_t grid = std::min<int64_t>(upper_units, static_cast<int64_t>(sms) * std::max(occ, 1));
  discard_stale_error();
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
  const size_t need = workspace_layout(batch, num_kv_heads, 1, 1, 0).ml_off;
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
  // the fast path bulk-copies q rows (16-byte aligned rows) and writes out in 4-byte pairs
  const bool fast = fast_path_ok(dtype, head_dim, block_size, group) && q_stride_h % 8 == 0 &&
                    q_stride_b % 8 == 0 && reinterpret_cast<uintptr_t>(query) % 16 == 0 &&
                    o_stride_h % 2 == 0 && o_stride_b % 2 == 0 && reinterpret_cast<uintptr_t>(out) % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(k_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(v_cache) % 16 == 0 &&
                    FastLayout::bytes(batch) <= 227 * 1024;
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
  p.work = reinterpret_cast<int32_t*>(ws + wl.work_off);
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
