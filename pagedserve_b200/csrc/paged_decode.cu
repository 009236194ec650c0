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
constexpr int kFastChunk = 128;        // tokens per split-K unit, fast path
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
  int32_t* plan;     // [2 * batch + 1]: longest-first order, chunk prefix (fast path)
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
// fast path: warp-pipelined TMA + mma.sync (bf16/f16, D = 64, block 16)
// ---------------------------------------------------------------------------
//
// Each warp is an independent stream: it pulls units from a global work
// queue (longest sequences first), keeps up to kRing pool blocks in flight
// in its own shared-memory ring and consumes them one block at a time with
// an online softmax.  No CTA-wide barrier follows the prologue; a finished
// unit is written by the warp that finished it (directly, or as a split-K
// partial merged by the last warp to finish its (sequence, head group)).
//
// Row packing.  The 16 rows of the m16n8k16 tile hold the q heads of HP kv
// heads: with HP = 2 rows 0-7 are the (<= 8) q heads of kv head 2p and rows
// 8-15 those of kv head 2p+1, so one TMA box brings both heads' 16 x 64 tiles
// (adjacent in the pool) and every accumulator register carries a real
// output; with HP = 1 the 16 rows are up to 16 q heads of one kv head.  Each
// K/V byte still leaves HBM exactly once.
constexpr int kFastWarps = 6;
constexpr int kFastThreads = kFastWarps * 32;
constexpr int kRing = 3;                           // slots per warp
constexpr int kKeys = 64;                          // sort buckets: chunk counts >= 64 share the last

template <int HP>
struct FastGeom {
  static constexpr int kKV = HP * kTileBytes;      // K tiles of one block (HP heads)
  static constexpr int kQ = 16 * 128;              // 16 q rows of 64 bf16/f16
  static constexpr int kSlot = 2 * kKV + kQ;       // K box, V box, q rows
  static constexpr int kRowsPerHead = 16 / HP;     // q heads per kv head the tile can hold
  static size_t bytes(int batch) {
    const size_t segs = (static_cast<size_t>(batch) + 31) / 32;
    return 1024 + static_cast<size_t>(kFastWarps) * kRing * kSlot +
           sizeof(int32_t) * (3 * static_cast<size_t>(batch) + 1 + segs * kKeys) + 64;
  }
};

__device__ __forceinline__ int chunks_of(int ctx, int chunk) { return ctx <= 0 ? 1 : (ctx + chunk - 1) / chunk; }

// s_ctx[b] = clamped context; order[i] = sequence at longest-first position i
// (chunk count descending, ties by index); prefix[i] = exclusive prefix of
// chunk counts along that order.  The order is a stable counting sort done by
// the whole CTA: each warp ranks its 32 sequences among equal keys with
// __match_any_sync, per-warp key histograms give each key's offset per warp.
// Every CTA computes the same arrays, so unit numbers mean the same thing
// everywhere; CTA 0 also leaves them in the workspace for the combine kernel.

__device__ int build_lpt_prefix(const DecodeParams& p, int32_t* order, int32_t* prefix, int32_t* s_ctx,
                                int32_t* whist) {
  __shared__ int32_t warp_sums[kFastWarps];
  __shared__ int32_t key_base[kKeys];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = p.batch;
  const int nseg = (B + 31) / 32;  // 32-sequence segments, whist[seg][key]
  for (int i = tid; i < nseg * kKeys; i += kFastThreads) whist[i] = 0;
  for (int b = tid; b < B; b += kFastThreads) s_ctx[b] = clamp_ctx(p, b);
  __syncthreads();
  auto key_of = [&](int b) { return kKeys - min(chunks_of(s_ctx[b], kFastChunk), kKeys); };  // 0 = longest
  // per-segment histograms
  for (int seg = warp; seg < nseg; seg += kFastWarps) {
    const int b = seg * 32 + lane;
    const int key = b < B ? key_of(b) : kKeys;  // kKeys: padding, no bucket
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    if (key < kKeys && lane == __ffs(peers) - 1) whist[seg * kKeys + key] = __popc(peers);
  }
  __syncthreads();
  // per key: exclusive prefix over segments (in place), total into key_base
  for (int k = tid; k < kKeys; k += kFastThreads) {
    int run = 0;
    for (int seg = 0; seg < nseg; ++seg) {
      const int c = whist[seg * kKeys + k];
      whist[seg * kKeys + k] = run;
      run += c;
    }
    key_base[k] = run;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive prefix over keys (ascending key = descending length)
    int v0 = key_base[lane], v1 = key_base[lane + 32];
    int incl0 = v0, incl1 = v1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a0 = __shfl_up_sync(0xffffffffu, incl0, o), a1 = __shfl_up_sync(0xffffffffu, incl1, o);
      if (lane >= o) incl0 += a0, incl1 += a1;
    }
    const int tot0 = __shfl_sync(0xffffffffu, incl0, 31);
    key_base[lane] = incl0 - v0;
    key_base[lane + 32] = tot0 + incl1 - v1;
  }
  __syncthreads();
  for (int seg = warp; seg < nseg; seg += kFastWarps) {
    const int b = seg * 32 + lane;
    const int key = b < B ? key_of(b) : kKeys;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    if (key < kKeys)
      order[key_base[key] + whist[seg * kKeys + key] + __popc(peers & ((1u << lane) - 1u))] = b;
  }
  __syncthreads();
  const int per = (B + kFastThreads - 1) / kFastThreads;
  const int begin = min(tid * per, B), end = min(begin + per, B);
  int local = 0;
  for (int i = begin; i < end; ++i) local += chunks_of(s_ctx[order[i]], kFastChunk);
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
    run += chunks_of(s_ctx[order[i]], kFastChunk);
  }
  int total = 0;
  for (int w = 0; w < kFastWarps; ++w) total += warp_sums[w];
  if (tid == 0) prefix[B] = total;
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int i = tid; i < B; i += kFastThreads) p.plan[i] = order[i];
    for (int i = tid; i <= B; i += kFastThreads) p.plan[B + i] = prefix[i];
  }
  return total;
}

// Unit u of the longest-first numbering: u = (prefix[i] + c) * groups + hg,
// groups = hkv / HP head groups.
struct FastUnit {
  int b, hg, c, nch, ctx, nblk;
};

__device__ __forceinline__ FastUnit fast_unit(const DecodeParams& p, const int32_t* order, const int32_t* prefix,
                                              const int32_t* s_ctx, int u, int groups) {
  FastUnit w;
  const int sc = u / groups;
  w.hg = u - sc * groups;
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

// 16-byte asynchronous global -> shared copy (L2 only), grouped per block.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <typename T, int HP>
__global__ void __launch_bounds__(kFastThreads, 1) decode_fast_kernel(const DecodeParams p) {
  using Geo = FastGeom<HP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring_all = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int32_t* order = reinterpret_cast<int32_t*>(ring_all + kFastWarps * kRing * Geo::kSlot);
  int32_t* prefix = order + p.batch;
  int32_t* s_ctx = prefix + p.batch + 1;
  int32_t* whist = s_ctx + p.batch;  // [ceil(B / 32)][kKeys]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.group;
  const int groups = p.hkv / HP;
  // tile rows this thread's accumulators cover: row g and row g + 8
  const bool row_lo = g < G;
  const bool row_hi = HP == 2 ? g < G : g + 8 < G;
  uint8_t* ring = ring_all + warp * kRing * Geo::kSlot;
  const int total_units = build_lpt_prefix(p, order, prefix, s_ctx, whist) * groups;  // ends with __syncthreads
  const int total_warps = gridDim.x * kFastWarps;
  const T* kpool = reinterpret_cast<const T*>(p.k_cache);
  const T* vpool = reinterpret_cast<const T*>(p.v_cache);
  const int64_t zlayer = static_cast<int64_t>(p.layer) * p.num_blocks * p.hkv;
  // per-lane ldmatrix row offsets inside a 16 x 64 swizzled tile
  const int kr = lane & 7;                                        // K: token row within an n-tile
  const int vr = ((lane >> 3) & 1) * 8 + (lane & 7);             // V: token row
  const uint32_t koff0 = kr * 128 + (((lane >> 3) ^ kr) << 4);          // dims 0..31
  const uint32_t koff1 = kr * 128 + (((4 + (lane >> 3)) ^ kr) << 4);    // dims 32..63
  uint32_t voff[4];
#pragma unroll
  for (int dp = 0; dp < 4; ++dp) voff[dp] = vr * 128 + (((dp * 2 + (lane >> 4)) ^ (vr & 7)) << 4);
  // per-lane copy pattern of one K (or V) box: 16-byte chunk lane + 32 i of the
  // HP contiguous 2 KB tiles lands at row r = chunk / 8, swizzled column
  // (chunk % 8) ^ (r % 8) - the 128-byte swizzle the ldmatrix offsets expect
  const uint32_t cp_col = lane & 7, cp_row0 = lane >> 3;
  const uint32_t cp_dst_even = cp_row0 * 128 + ((cp_col ^ cp_row0) << 4);
  const uint32_t cp_dst_odd = cp_row0 * 128 + ((cp_col ^ (cp_row0 + 4)) << 4);

  // Every warp's first unit is its global warp index; later units come from
  // the queue (numbered after those).  Grabs are issued one unit ahead and
  // their results read one unit later, so the atomic's round trip never
  // stalls the warp.
  auto grab_issue = [&]() -> int { return lane == 0 ? atomicAdd(p.work, 1) + total_warps : 0; };
  auto grab_read = [&](int raw) -> int {
    const int v = __shfl_sync(0xffffffffu, raw, 0);
    return v < total_units ? v : -1;
  };

  // ---- issue side --------------------------------------------------------
  const int wid = blockIdx.x * kFastWarps + warp;
  int iu = wid < total_units ? wid : -1;  // unit whose blocks are being issued
  FastUnit iw{};
  int32_t itab = -1;
  int ib = 0;
  if (iu >= 0) {
    iw = fast_unit(p, order, prefix, s_ctx, iu, groups);
    itab = load_unit_table(p, iw, lane);
  }
  int nu = iu >= 0 ? grab_read(grab_issue()) : -1;  // next unit: decoded, table prefetched
  FastUnit nw{};
  int32_t ntab = -1;
  if (nu >= 0) {
    nw = fast_unit(p, order, prefix, s_ctx, nu, groups);
    ntab = load_unit_table(p, nw, lane);
  }
  int graw = nu >= 0 ? grab_issue() : 0;  // pending grab for the unit after nu
  bool gpending = nu >= 0;
  uint32_t issued = 0, consumed = 0;
  int32_t meta = 0;     // lane s: flags of ring slot s (bit 0 data, 1-5 valid tokens, 6 first, 7 last)
  int32_t meta_u = -1;  // lane s: unit of ring slot s

  // Copy one block (K and V of the HP packed heads, and the unit's q rows
  // with its first block) into the next ring slot as one cp.async group.
  auto issue_one = [&]() {
    const uint32_t slot = issued % kRing;
    const uint32_t sdst = smem_u32(ring + slot * Geo::kSlot);
    const int32_t blk = __shfl_sync(0xffffffffu, itab, ib);
    const int valid = max(0, min(16, iw.ctx - (iw.c * kFastChunk + ib * 16)));
    const bool ok = blk >= 0 && valid > 0;
    const bool first = ib == 0;
    // The slot's previous contents were read (ldmatrix) before the __syncwarp
    // that precedes every refill.
    if (ok) {
      const int64_t tile = zlayer + static_cast<int64_t>(blk) * p.hkv + iw.hg * HP;
      const char* ksrc = reinterpret_cast<const char*>(kpool + tile * (16 * 64)) + lane * 16;
      const char* vsrc = reinterpret_cast<const char*>(vpool + tile * (16 * 64)) + lane * 16;
      // a 16 x 64 tile is 2 KB = 128 chunks: 4 per lane, HP tiles per box;
      // chunk lane + 32 i sits at row 4 i + lane / 8, so the swizzled column
      // alternates between two per-lane values
#pragma unroll
      for (int i = 0; i < HP * 4; ++i) {
        const uint32_t d = sdst + i * 512 + ((i & 1) ? cp_dst_odd : cp_dst_even);
        cp_async16(d, ksrc + i * 512);
        cp_async16(d + Geo::kKV, vsrc + i * 512);
      }
    }
    if (first) {
      // q rows of kv head hg*HP + s go to tile rows s*8 (HP = 2) or 0 (HP = 1)
      const T* qb = reinterpret_cast<const T*>(p.q) + static_cast<int64_t>(iw.b) * p.qsb;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = cp_row0 + 4 * i;  // tile row 0..15
        const int s = HP == 2 ? r >> 3 : 0;
        const int rr = HP == 2 ? r & 7 : r;
        if (rr < G) {
          const T* src = qb + static_cast<int64_t>((iw.hg * HP + s) * G + rr) * p.qsh + cp_col * 8;
          cp_async16(sdst + 2 * Geo::kKV + r * 128 + cp_col * 16, src);
        }
      }
    }
    cp_async_commit();
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
      nu = -1;
      if (gpending) {
        nu = grab_read(graw);
        gpending = false;
        if (nu >= 0) {
          nw = fast_unit(p, order, prefix, s_ctx, nu, groups);
          ntab = load_unit_table(p, nw, lane);
          graw = grab_issue();
          gpending = true;
        }
      }
    }
  };

  // Everything above reads only lengths, tables and the workspace.  The pool
  // and q may still be being written by the stream predecessor (a
  // reshape_and_cache launched just before lets this kernel start early), so
  // wait for it here; the combine kernel may launch as soon as every CTA is
  // past this point.
  pdl_wait();
  pdl_launch_dependents();
  while (iu >= 0 && issued - consumed < static_cast<uint32_t>(kRing)) issue_one();

  // ---- consume side ------------------------------------------------------
  uint32_t qa[4][4];   // A fragments per k-step (a0..a3)
  float o[8][4];       // rows g (c0, c1) and g + 8 (c2, c3), dims 8n + 2t + {0, 1}
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  FastUnit cw{};
  int cu = -1;
  static_assert(kRing == 3, "the wait below assumes a three-slot ring");
  while (consumed != issued) {
    const uint32_t slot = consumed % kRing;
    const int32_t mt = __shfl_sync(0xffffffffu, meta, slot);
    const bool first = (mt >> 6) & 1, last = (mt >> 7) & 1;
    const int valid = (mt & 1) ? (mt >> 1) & 31 : 0;
    if (first) cu = __shfl_sync(0xffffffffu, meta_u, slot);
    // the oldest copy group is complete once at most the newer ones are pending
    const uint32_t inflight = issued - consumed;
    if (inflight >= 3) cp_async_wait<2>(); else if (inflight == 2) cp_async_wait<1>(); else cp_async_wait<0>();
    __syncwarp();  // every lane's copies are visible to every lane
    const uint32_t sbase = smem_u32(ring + slot * Geo::kSlot);
    if (first) {
      cw = fast_unit(p, order, prefix, s_ctx, cu, groups);
      m_lo = m_hi = -INFINITY;
      l_lo = l_hi = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      const uint32_t qs = sbase + 2 * Geo::kKV;
      // A fragments: matrices (rows 0-7 | 8-15) x (k 0-7 | 8-15) of each k-step
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4(qs + ((lane & 7) + ((lane >> 3) & 1) * 8) * 128 + ((ks * 2 + (lane >> 4)) << 4), r0, r1, r2, r3);
        qa[ks][0] = row_lo ? r0 : 0u;
        qa[ks][1] = row_hi ? r1 : 0u;
        qa[ks][2] = row_lo ? r2 : 0u;
        qa[ks][3] = row_hi ? r3 : 0u;
      }
    }
    if (valid) {
      // ---- S = Q K^T (both packed heads), one accumulator per (n-tile, head slot)
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        float acc[HP][4];
#pragma unroll
        for (int hs = 0; hs < HP; ++hs) {
          acc[hs][0] = acc[hs][1] = acc[hs][2] = acc[hs][3] = 0.f;
          const uint32_t kt = sbase + hs * kTileBytes + nt * 8 * 128;
          uint32_t b[8];
          ldsm_x4(kt + koff0, b[0], b[1], b[2], b[3]);
          ldsm_x4(kt + koff1, b[4], b[5], b[6], b[7]);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            // HP = 2: head slot 0 feeds rows 0-7, head slot 1 rows 8-15
            const bool use_lo = HP == 1 || hs == 0, use_hi = HP == 1 || hs == 1;
            mma_16816<T>(acc[hs], use_lo ? qa[ks][0] : 0u, use_hi ? qa[ks][1] : 0u, use_lo ? qa[ks][2] : 0u,
                         use_hi ? qa[ks][3] : 0u, b[2 * ks], b[2 * ks + 1]);
          }
        }
        s[nt][0] = acc[0][0];
        s[nt][1] = acc[0][1];
        s[nt][2] = acc[HP - 1][2];
        s[nt][3] = acc[HP - 1][3];
      }
      if (valid < 16) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if (nt * 8 + 2 * t + e >= valid) {
              s[nt][e] = -INFINITY;
              s[nt][2 + e] = -INFINITY;
            }
          }
        }
      }
      float mb_lo = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
      float mb_hi = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
      mb_lo = fmaxf(mb_lo, __shfl_xor_sync(0xffffffffu, mb_lo, 1));
      mb_hi = fmaxf(mb_hi, __shfl_xor_sync(0xffffffffu, mb_hi, 1));
      mb_lo = fmaxf(mb_lo, __shfl_xor_sync(0xffffffffu, mb_lo, 2));
      mb_hi = fmaxf(mb_hi, __shfl_xor_sync(0xffffffffu, mb_hi, 2));
      // every block holds >= 1 valid token, so the new maxima are finite
      const float mn_lo = fmaxf(m_lo, mb_lo), mn_hi = fmaxf(m_hi, mb_hi);
      const float al_lo = exp2f((m_lo - mn_lo) * p.scale_log2);  // exp2(-inf) = 0 on the first block
      const float al_hi = exp2f((m_hi - mn_hi) * p.scale_log2);
      m_lo = mn_lo;
      m_hi = mn_hi;
      const float ms_lo = mn_lo * p.scale_log2, ms_hi = mn_hi * p.scale_log2;
      float pr[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        pr[nt][0] = exp2f(fmaf(s[nt][0], p.scale_log2, -ms_lo));
        pr[nt][1] = exp2f(fmaf(s[nt][1], p.scale_log2, -ms_lo));
        pr[nt][2] = exp2f(fmaf(s[nt][2], p.scale_log2, -ms_hi));
        pr[nt][3] = exp2f(fmaf(s[nt][3], p.scale_log2, -ms_hi));
      }
      l_lo = l_lo * al_lo + ((pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]));
      l_hi = l_hi * al_hi + ((pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]));
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        o[n][0] *= al_lo;
        o[n][1] *= al_lo;
        o[n][2] *= al_hi;
        o[n][3] *= al_hi;
      }
      // ---- O += P V --------------------------------------------------------
      const uint32_t pa0 = pack2<T>(pr[0][0], pr[0][1]);  // rows g, tokens 2t, 2t+1
      const uint32_t pa1 = pack2<T>(pr[0][2], pr[0][3]);  // rows g+8
      const uint32_t pa2 = pack2<T>(pr[1][0], pr[1][1]);  // rows g, tokens 8+2t, 9+2t
      const uint32_t pa3 = pack2<T>(pr[1][2], pr[1][3]);  // rows g+8
      // rows past the context may hold anything (even NaN): zero them
      uint32_t keep0 = 0xffffffffu, keep1 = 0xffffffffu;
      if (valid < 16) {
        keep0 = (2 * t < valid ? 0x0000ffffu : 0u) | (2 * t + 1 < valid ? 0xffff0000u : 0u);
        keep1 = (8 + 2 * t < valid ? 0x0000ffffu : 0u) | (8 + 2 * t + 1 < valid ? 0xffff0000u : 0u);
      }
#pragma unroll
      for (int hs = 0; hs < HP; ++hs) {
        const uint32_t vt = sbase + Geo::kKV + hs * kTileBytes;
        const bool use_lo = HP == 1 || hs == 0, use_hi = HP == 1 || hs == 1;
        const uint32_t x0 = use_lo ? pa0 : 0u, x2 = use_lo ? pa2 : 0u;
        const uint32_t x1 = use_hi ? pa1 : 0u, x3 = use_hi ? pa3 : 0u;
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vt + voff[dp], b0, b1, b2, b3);
          mma_16816<T>(o[2 * dp], x0, x1, x2, x3, b0 & keep0, b1 & keep1);
          mma_16816<T>(o[2 * dp + 1], x0, x1, x2, x3, b2 & keep0, b3 & keep1);
        }
      }
    }
    __syncwarp();
    ++consumed;
    if (iu >= 0) issue_one();  // refill the slot just freed

    if (last) {
      // ---- finish the unit --------------------------------------------------
      float ll = l_lo, lh = l_hi;
      ll += __shfl_xor_sync(0xffffffffu, ll, 1);
      lh += __shfl_xor_sync(0xffffffffu, lh, 1);
      ll += __shfl_xor_sync(0xffffffffu, ll, 2);
      lh += __shfl_xor_sync(0xffffffffu, lh, 2);
      if (cw.nch == 1) {
        const int qh_lo = HP == 2 ? (cw.hg * 2) * G + g : cw.hg * G + g;
        const int qh_hi = HP == 2 ? (cw.hg * 2 + 1) * G + g : cw.hg * G + g + 8;
        const float il = ll > 0.f ? 1.f / ll : 0.f, ih = lh > 0.f ? 1.f / lh : 0.f;
        T* olo = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(cw.b) * p.osb + static_cast<int64_t>(qh_lo) * p.osh;
        T* ohi = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(cw.b) * p.osb + static_cast<int64_t>(qh_hi) * p.osh;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          if (row_lo) *reinterpret_cast<uint32_t*>(olo + n * 8 + 2 * t) = pack2<T>(o[n][0] * il, o[n][1] * il);
          if (row_hi) *reinterpret_cast<uint32_t*>(ohi + n * 8 + 2 * t) = pack2<T>(o[n][2] * ih, o[n][3] * ih);
        }
      } else {
        // partial rows: 16 per unit, row g (lo) and g + 8 (hi)
        float* po = p.part_o + static_cast<int64_t>(cu) * 16 * 64;
        float* pml = p.part_ml + static_cast<int64_t>(cu) * 16 * 2;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          *reinterpret_cast<float2*>(po + g * 64 + n * 8 + 2 * t) = make_float2(o[n][0], o[n][1]);
          *reinterpret_cast<float2*>(po + (g + 8) * 64 + n * 8 + 2 * t) = make_float2(o[n][2], o[n][3]);
        }
        if (t == 0) {
          *reinterpret_cast<float2*>(pml + 2 * g) = make_float2(m_lo, ll);
          *reinterpret_cast<float2*>(pml + 2 * (g + 8)) = make_float2(m_hi, lh);
        }
        // merged after this launch by decode_combine_kernel
      }
    }
  }
  // The last warp of the launch leaves the work queue at zero for the next
  // one.  The release-acquire "done" ticket orders every warp's grabs (a
  // pending one included) before the reset.
  if (lane == 0) {
    if (atom_add_acq_rel_gpu(p.work + 1, 1) == total_warps - 1) {
      p.work[0] = 0;
      p.work[1] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// split-K merge for the fast path: one CTA per (sequence, head group) with
// more than one chunk, launched right after decode_fast_kernel on the same
// stream (stream order makes every partial visible; no fences or atomics).
// 16 warps: warp r first reduces row r's maximum over the chunks; then 4
// groups of 128 threads take every 4th chunk, thread (row, 8-dim slice)
// accumulating with full memory-level parallelism, and the groups are summed
// through shared memory.
// ---------------------------------------------------------------------------
constexpr int kCombThreads = 512;

template <typename T, int HP>
__global__ void __launch_bounds__(kCombThreads) decode_combine_kernel(const DecodeParams p) {
  pdl_wait();  // every partial of the decode launch before is complete and visible
  const int groups = p.hkv / HP;
  const int i = blockIdx.x / groups, hg = blockIdx.x - (blockIdx.x / groups) * groups;
  const int32_t* order = p.plan;
  const int32_t* prefix = p.plan + p.batch;
  const int nch = prefix[i + 1] - prefix[i];
  if (nch <= 1) return;
  const int b = order[i];
  const int64_t u0 = static_cast<int64_t>(prefix[i]) * groups + hg;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float s_M[16];
  __shared__ float s_acc[4][128][9];
  __shared__ float s_l[4][16];
  {
    const int r = warp;  // 16 warps, one per tile row
    float M = -INFINITY;
    for (int c = lane; c < nch; c += 32) M = fmaxf(M, __ldcg(p.part_ml + (u0 + static_cast<int64_t>(c) * groups) * 32 + 2 * r));
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (lane == 0) s_M[r] = M;
  }
  __syncthreads();
  const int cg = tid >> 7, rq = tid & 127, r = rq >> 3, q8 = rq & 7;
  const float M = s_M[r];
  float acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
  float l = 0.f;
  if (M != -INFINITY) {
#pragma unroll 4
    for (int c = cg; c < nch; c += 4) {
      const int64_t uc = u0 + static_cast<int64_t>(c) * groups;
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml + uc * 32 + 2 * r));
      const float w = ml.x == -INFINITY ? 0.f : exp2f((ml.x - M) * p.scale_log2);
      const float4* src = reinterpret_cast<const float4*>(p.part_o + uc * 16 * 64 + r * 64 + q8 * 8);
      const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
      l = fmaf(ml.y, w, l);
      acc[0] = fmaf(v0.x, w, acc[0]); acc[1] = fmaf(v0.y, w, acc[1]);
      acc[2] = fmaf(v0.z, w, acc[2]); acc[3] = fmaf(v0.w, w, acc[3]);
      acc[4] = fmaf(v1.x, w, acc[4]); acc[5] = fmaf(v1.y, w, acc[5]);
      acc[6] = fmaf(v1.z, w, acc[6]); acc[7] = fmaf(v1.w, w, acc[7]);
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) s_acc[cg][rq][k] = acc[k];
  if (q8 == 0) s_l[cg][r] = l;
  __syncthreads();
  if (cg != 0) return;
  const float L = s_l[0][r] + s_l[1][r] + s_l[2][r] + s_l[3][r];
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int G = p.group;
  const int s = HP == 2 ? r >> 3 : 0, rr = HP == 2 ? r & 7 : r;
  if (rr >= G) return;
  const int qh = (hg * HP + s) * G + rr;
  T* orow = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(b) * p.osb + static_cast<int64_t>(qh) * p.osh + q8 * 8;
#pragma unroll
  for (int k = 0; k < 8; k += 2) {
    const float x = (s_acc[0][rq][k] + s_acc[1][rq][k] + s_acc[2][rq][k] + s_acc[3][rq][k]) * inv;
    const float y = (s_acc[0][rq][k + 1] + s_acc[1][rq][k + 1] + s_acc[2][rq][k + 1] + s_acc[3][rq][k + 1]) * inv;
    *reinterpret_cast<uint32_t*>(orow + k) = pack2<T>(x, y);
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

// Packed kv heads per fast-path unit: 2 when heads pair up and each has <= 8
// q heads, 1 when one kv head has <= 16 q heads, 0 = no fast path.
int fast_heads_per_unit(int dtype, int head_dim, int block_size, int group, int hkv) {
  if (!((dtype == PSB_BF16 || dtype == PSB_F16) && head_dim == 64 && block_size == 16)) return 0;
  if (hkv % 2 == 0 && group <= 8) return 2;
  if (group <= 16) return 1;
  return 0;
}

// Split-K geometry: units, rows per unit (the fast path always stores the
// 16 packed tile rows) and the arrival-counter count.
struct SplitGeom {
  int chunk, rows, counters, batch;
  int64_t max_units;
};

SplitGeom split_geometry(int hp, int batch, int hkv, int group, int max_context) {
  SplitGeom sg;
  sg.chunk = hp ? kFastChunk : kGenericChunk;
  const int groups = hp ? hkv / hp : hkv;
  const int64_t per = std::max<int64_t>(1, (static_cast<int64_t>(max_context) + sg.chunk - 1) / sg.chunk);
  sg.max_units = per * batch * groups;
  sg.rows = hp ? 16 : group;
  sg.counters = batch * groups;
  sg.batch = batch;
  return sg;
}

struct WorkspaceLayout {
  size_t work_off, counters_off, plan_off, ml_off, o_off, total;
};

// [work queue: 2 x int32 | pad to 256][arrival counters: int32 per (sequence, head group)]
// [plan: longest-first order and chunk prefix, 2 * batch + 1 int32]
// [partial max/sum: max_units * rows * 2 f32][partial outputs: max_units * rows * head_dim f32]
// Everything before ml_off must be zero before the first launch.
WorkspaceLayout workspace_layout(const SplitGeom& sg, int head_dim) {
  WorkspaceLayout w;
  w.work_off = 0;
  w.counters_off = 256;
  w.plan_off = align_up(w.counters_off + sizeof(int32_t) * static_cast<size_t>(sg.counters), 256);
  w.ml_off = align_up(w.plan_off + sizeof(int32_t) * (2 * static_cast<size_t>(sg.batch) + 1), 256);
  w.o_off = align_up(w.ml_off + sizeof(float) * static_cast<size_t>(sg.max_units) * sg.rows * 2, 256);
  w.total = w.o_off + sizeof(float) * static_cast<size_t>(sg.max_units) * sg.rows * head_dim;
  return w;
}

template <typename T, int HP>
int launch_fast(const DecodeParams& prm, cudaStream_t stream, int sms) {
  const size_t smem = FastGeom<HP>::bytes(prm.batch);
  if (smem > 227 * 1024) return PSB_ERR_UNSUPPORTED;
  const void* kern = reinterpret_cast<const void*>(decode_fast_kernel<T, HP>);
  int occ = 0;
  if (!kernel_occupancy(kern, kFastThreads, smem, &occ) || occ < 1) return PSB_ERR_CUDA;
  const int64_t grid =
      std::min<int64_t>(static_cast<int64_t>(sms) * occ, (prm.max_units + kFastWarps - 1) / kFastWarps);
  discard_stale_error();
  cudaError_t e = launch_pdl(decode_fast_kernel<T, HP>, dim3(static_cast<unsigned>(grid)), dim3(kFastThreads), smem,
                             stream, prm);
  if (e != cudaSuccess) return record_cuda_error(e);
  const int64_t merges = static_cast<int64_t>(prm.batch) * (prm.hkv / HP);
  e = launch_pdl(decode_combine_kernel<T, HP>, dim3(static_cast<unsigned>(merges)), dim3(kCombThreads), 0, stream,
                 prm);
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}

template <typename T>
int launch_decode(DecodeParams prm, int hp, cudaStream_t stream) {
  const int sms = device_sm_count();
  if (sms <= 0) return PSB_ERR_CUDA;
  if constexpr (!std::is_same<T, float>::value) {
    if (hp == 2) return launch_fast<T, 2>(prm, stream, sms);
    if (hp == 1) return launch_fast<T, 1>(prm, stream, sms);
  }
  const size_t smem = generic_smem_bytes(prm.group, prm.head_dim, prm.batch);
  if (smem > 227 * 1024) return PSB_ERR_UNSUPPORTED;
  const void* kern = reinterpret_cast<const void*>(decode_generic_kernel<T>);
  int occ = 0;
  if (!kernel_occupancy(kern, kThreads, smem, &occ)) return PSB_ERR_CUDA;
  const int64_t grid = std::min<int64_t>(prm.max_units, static_cast<int64_t>(sms) * std::max(occ, 1));
  discard_stale_error();
  decode_generic_kernel<T><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(prm);
  return check_launch();
}

// Which path a call takes (the fast path bulk-copies 16-byte q rows and
// writes the output in 4-byte pairs).
int choose_path(int dtype, int head_dim, int block_size, int group, int hkv, int batch, const void* query,
                int64_t qsb, int64_t qsh, const void* out, int64_t osb, int64_t osh, const void* kc, const void* vc) {
  const int hp = fast_heads_per_unit(dtype, head_dim, block_size, group, hkv);
  if (!hp) return 0;
  const bool aligned = qsh % 8 == 0 && qsb % 8 == 0 && reinterpret_cast<uintptr_t>(query) % 16 == 0 &&
                       osh % 2 == 0 && osb % 2 == 0 && reinterpret_cast<uintptr_t>(out) % 4 == 0 &&
                       reinterpret_cast<uintptr_t>(kc) % 16 == 0 && reinterpret_cast<uintptr_t>(vc) % 16 == 0;
  const size_t smem = hp == 2 ? FastGeom<2>::bytes(batch) : FastGeom<1>::bytes(batch);
  return aligned && smem <= 227 * 1024 ? hp : 0;
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
  // sized for whichever path the geometry allows; large enough for the other
  const int hp = fast_heads_per_unit(dtype, head_dim, block_size, group, num_kv_heads);
  const size_t fast = hp ? workspace_layout(split_geometry(hp, batch, num_kv_heads, group, max_context), head_dim).total : 0;
  const size_t gen = workspace_layout(split_geometry(0, batch, num_kv_heads, group, max_context), head_dim).total;
  return std::max(fast, gen);
}

extern "C" int psb_paged_decode_workspace_init(void* workspace, size_t workspace_bytes, int32_t batch,
                                               int32_t num_kv_heads, psb_stream_t stream) {
  SplitGeom sg{kGenericChunk, 1, batch * num_kv_heads, batch, 0};
  const size_t need = workspace_layout(sg, 1).ml_off;
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
  const int hp = choose_path(dtype, head_dim, block_size, group, num_kv_heads, batch, query, q_stride_b, q_stride_h,
                             out, o_stride_b, o_stride_h, k_cache, v_cache);
  const SplitGeom sg = split_geometry(hp, batch, num_kv_heads, group, max_context);
  const WorkspaceLayout wl = workspace_layout(sg, head_dim);
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
  p.chunk = sg.chunk;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * 1.4426950408889634f;
  char* ws = static_cast<char*>(workspace);
  p.counters = reinterpret_cast<int32_t*>(ws + wl.counters_off);
  p.work = reinterpret_cast<int32_t*>(ws + wl.work_off);
  p.plan = reinterpret_cast<int32_t*>(ws + wl.plan_off);
  p.part_ml = reinterpret_cast<float*>(ws + wl.ml_off);
  p.part_o = reinterpret_cast<float*>(ws + wl.o_off);
  p.max_units = sg.max_units;
  p.err = error_flag;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PSB_BF16: return launch_decode<__nv_bfloat16>(p, hp, s);
    case PSB_F16: return launch_decode<__half>(p, hp, s);
    default: return launch_decode<float>(p, 0, s);
  }
}
