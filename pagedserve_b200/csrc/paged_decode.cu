// Paged GQA decode attention for B200 (sm_100a).
//
// Replaces PagedServe's Triton decode kernel
// (pagedserve/attention/triton_paged_decode.py:10-95) with the numerics of its
// PyTorch reference (pagedserve/attention/vectorized_batched_attention.py:79-159).
//
// Fast path (bf16/f16, head_dim 64, block_size 16, up to 8 q heads per kv
// head, or 16 with an odd kv-head count): the pool blocks of all sequences
// are split evenly over the warps of a persistent grid (one CTA of 8 warps
// per SM).  Each warp streams its blocks through a private shared-memory ring
// with 16-byte cp.async copies, runs QK^T and PV on mma.sync m16n8k16 with
// fp32 accumulation (all q heads of two kv heads packed into the 16 tile
// rows, so every K/V byte leaves HBM once) and an online softmax reduced
// with quad shuffles.  Probabilities are rounded to the cache dtype before
// P.V, as the reference does (vectorized_batched_attention.py:152-156).  A
// sequence that spans several warps leaves fp32 partials that
// decode_combine_kernel, launched next on the same stream, merges.
//
// Generic path (fp32, or any other geometry): CUDA-core kernel; a unit is
// (sequence, kv head, 64-token chunk), and the last CTA to finish a split
// sequence - an atomic ticket, no waiting - merges its partials in the same
// launch.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "host_util.h"

namespace psb {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kFastChunk = 128;        // tokens per split-K unit, fast path
constexpr int kTileBytes = 16 * 64 * 2;
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
  int32_t total_warps;  // warps of the fast-path decode grid
  int64_t max_units;
  int32_t* err;
  // append (psb_paged_decode_append): row b's new K/V [Hkv, D] (element
  // strides), stored at position ctx[b] - 1 before attending; null otherwise
  const char* new_k;
  const char* new_v;
  int64_t nks, nkh, nvs, nvh;
  char* k_pool_w;
  char* v_pool_w;
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
// fast path: warp-streamed cp.async ring + mma.sync (bf16/f16, D = 64, block 16)
// ---------------------------------------------------------------------------
//
// Work split.  The pool blocks every sequence's context occupies, taken in
// (head group, sequence, block) order, form one list of N = Nb * groups
// "items" (Nb = sum over sequences of max(1, ceil(ctx / 16))).  Warp w of
// the grid's W warps streams items [w N / W, (w + 1) N / W): every warp gets
// the same number of blocks whatever the length distribution.  A warp's
// range is a run of "segments" (its share of one sequence); a segment that
// is a whole sequence writes its output, any other (only a range's first and
// last can be) writes an fp32 partial (row max, row sum, unnormalised
// output) to slot 2 w + {0: first segment, 1: last}, and
// decode_combine_kernel merges the partials of every sequence that spans
// several warps.  (Measured on the 256-sequence serving batch: per-warp
// streaming rates differ by about 15 %, but handing out work dynamically -
// atomic claims and steals - cost more per warp than the imbalance.)
//
// Each warp is an independent stream with its own shared-memory ring of
// kRing slots (K and V of one block of HP packed kv heads, plus the q rows
// with a segment's first block), filled by 16-byte cp.async copies, one
// commit group per block.  No CTA-wide barrier follows the prologue.  Eight
// warps of two slots each (two warps per SM sub-partition, 16 blocks in
// flight per SM) measured faster than six of three (where warps 2 and 3 have a
// sub-partition to themselves and outrun the rest by ~7 %) and than four of
// four or five.
//
// Row packing.  The 16 rows of the m16n8k16 tile hold the q heads of HP kv
// heads: with HP = 2 rows 0-7 are the (<= 8) q heads of kv head 2p and rows
// 8-15 those of kv head 2p+1, so one block's copy brings both heads' 16 x 64
// tiles (adjacent in the pool) and every accumulator register carries a real
// output; with HP = 1 the 16 rows are up to 16 q heads of one kv head.  Each
// K/V byte leaves HBM exactly once.
constexpr int kFastWarps = 8;
constexpr int kFastThreads = kFastWarps * 32;
constexpr int kRing = 2;              // slots per warp
constexpr int kFastMinBlocks = 8;     // blocks per warp below which the grid shrinks
constexpr int kMaxFastCtas = 160;     // grid limit (one CTA per SM; B200 has 148)

constexpr int kPartFloats = 16 * 64;  // one partial: 16 tile rows x 64 dims
constexpr int kMaxFastBatch = 1 << 20;

template <int HP>
struct FastGeom {
  static constexpr int kKV = HP * kTileBytes;  // K tiles of one block (HP heads)
  static constexpr int kQ = 16 * 128;          // 16 q rows of 64 bf16/f16
  static constexpr int kSlot = 2 * kKV + kQ;   // K box, V box, q rows
  static size_t bytes(int batch) {
    return 1024 + static_cast<size_t>(kFastWarps) * kRing * kSlot +
           sizeof(int32_t) * (2 * static_cast<size_t>(batch) + 1) + 64;
  }
};

__device__ __forceinline__ int blocks_of(int ctx) { return ctx <= 0 ? 1 : (ctx + 15) >> 4; }

// s_ctx[b] = clamped context; bpre[b] = exclusive prefix of blocks_of over
// sequences, bpre[B] = Nb.  Every CTA computes the same arrays.
__device__ int build_block_prefix(const DecodeParams& p, int32_t* bpre, int32_t* s_ctx) {
  __shared__ int32_t warp_sums[kFastWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = p.batch;
  const int per = (B + kFastThreads - 1) / kFastThreads;
  const int begin = min(tid * per, B), end = min(begin + per, B);
  int local = 0;
  for (int b = begin; b < end; ++b) {
    const int n = clamp_ctx(p, b);
    s_ctx[b] = n;
    local += blocks_of(n);
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
    bpre[b] = run;
    run += blocks_of(s_ctx[b]);
  }
  int total = 0;
  for (int w = 0; w < kFastWarps; ++w) total += warp_sums[w];
  if (tid == 0) bpre[B] = total;
  __syncthreads();
  return total;
}

// min(cap, left) for a 64-bit item count.
__device__ __forceinline__ int clamp_items(int cap, int64_t left) {
  return left < cap ? static_cast<int>(left) : cap;
}

// floor(x / d) for 0 <= x < 2^53 and d >= 1 given rd ~ 1 / d: a double
// estimate corrected to the exact quotient with integer multiplies (no
// division on the dependent path).
__device__ __forceinline__ int64_t div_floor(int64_t x, int64_t d, double rd) {
  int64_t q = static_cast<int64_t>(static_cast<double>(x) * rd);
  if (q * d > x) --q;
  if ((q + 1) * d <= x) ++q;
  if (q * d > x) --q;
  return q;
}

// The item list dealt evenly over the grid's W warps, each a contiguous
// range: warp w streams [floor(N w / W), floor(N (w + 1) / W)).  (Weighting
// the ranges towards the warps that have an SM sub-partition to themselves
// - warps 2 and 3 of each CTA stream ~7 % faster than the four that share
// two - measured slower on the 256-sequence serving batch.)
struct Split {
  int64_t n;
  int warps;
  double rw, rn;
  __device__ __forceinline__ Split(int64_t n_items, int n_warps) : n(n_items), warps(n_warps) {
    rw = 1.0 / static_cast<double>(n_warps);
    rn = 1.0 / static_cast<double>(n_items > 0 ? n_items : 1);
  }
  __device__ __forceinline__ int64_t start(int w) const { return div_floor(n * w, warps, rw); }
  // the warp whose range holds ``item`` (0 <= item < n): the largest w with
  // floor(N w / W) <= item, i.e. N w < (item + 1) W
  __device__ __forceinline__ int warp_of(int64_t item) const {
    const int64_t w = div_floor((item + 1) * warps - 1, n, rn);
    return w < warps - 1 ? static_cast<int>(w) : warps - 1;
  }
};

// A chunk: up to 32 consecutive items of a warp's range, lane j holding item
// beg + j - its raw block-table entry (-1 when the block holds no valid
// token), flags (bits 1-5 valid tokens, 6 first of its segment, 7 last of its
// segment, 8 first block of its sequence, 9 last block of its sequence),
// sequence | head group << 20 and partial slot.
struct Chunk {
  int64_t beg;
  int n;
  int32_t blk, meta, seg, slot;
};

// 16-byte asynchronous global -> shared copy (L2 only), grouped per block.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// The same with an L2 cache policy (``createpolicy``): the K/V stream is
// read once per launch, so it goes in as evict-first and leaves the rest of
// L2 - the split-K partials the combine kernel reads back - in place.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void cp_async16_hint(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Wait until the oldest of ``inflight`` (1 .. N) committed groups is complete.
template <int N>
__device__ __forceinline__ void cp_async_wait_oldest(uint32_t inflight) {
  if constexpr (N > 1) {
    if (inflight >= N) {
      cp_async_wait<N - 1>();
      return;
    }
    cp_async_wait_oldest<N - 1>(inflight);
  } else {
    cp_async_wait<0>();
  }
}

// APPEND: psb_paged_decode_append (the new-token store below); a separate
// instantiation so plain decode carries none of it.
template <typename T, int HP, bool APPEND>
__global__ void __launch_bounds__(kFastThreads, 1) decode_fast_kernel(const DecodeParams p) {
  using Geo = FastGeom<HP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring_all = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int32_t* bpre = reinterpret_cast<int32_t*>(ring_all + kFastWarps * kRing * Geo::kSlot);
  int32_t* s_ctx = bpre + p.batch + 1;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int G = p.group;
  const int B = p.batch;
  const int groups = p.hkv / HP;
  // tile rows this thread's accumulators cover: row g and row g + 8
  const bool row_lo = g < G;
  const bool row_hi = HP == 2 ? g < G : g + 8 < G;
  uint8_t* ring = ring_all + warp * kRing * Geo::kSlot;
  const int nb_total = build_block_prefix(p, bpre, s_ctx);  // ends with __syncthreads
  const int64_t n_items = static_cast<int64_t>(nb_total) * groups;
  const int n_warps = gridDim.x * kFastWarps;
  const int gw = blockIdx.x * kFastWarps + warp;
  const T* kpool = reinterpret_cast<const T*>(p.k_cache);
  const T* vpool = reinterpret_cast<const T*>(p.v_cache);
  const int64_t zlayer = static_cast<int64_t>(p.layer) * p.num_blocks * p.hkv;
  const uint64_t stream_pol = l2_evict_first_policy();
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

  // ---- chunks of this warp's range ----------------------------------------
  const Split split(n_items, n_warps);
  const int64_t my_a = split.start(gw), my_e = split.start(gw + 1);
  auto build_chunk = [&](int64_t cbeg) -> Chunk {
    Chunk c;
    c.beg = cbeg;
    c.n = clamp_items(32, my_e - cbeg);
    c.blk = -1;
    c.meta = 0;
    c.seg = 0;
    c.slot = 2 * gw;
    if (lane < c.n) {
      const int64_t i = cbeg + lane;
      int hg = 0;
      int64_t r = i;
      while (r >= nb_total) {
        r -= nb_total;
        ++hg;
      }
      const int b = find_seq(bpre, B, static_cast<int>(r));
      const int j = static_cast<int>(r) - bpre[b];
      const int ctx = s_ctx[b], nblk = blocks_of(ctx);
      const int valid = max(0, min(16, ctx - 16 * j));
      c.slot = 2 * gw + (i - j > my_a ? 1 : 0);  // 0 for the range's first segment
      c.meta = (valid << 1) | (j == 0 || i == my_a ? 1 << 6 : 0) | (j == nblk - 1 || i == my_e - 1 ? 1 << 7 : 0) |
               (j == 0 ? 1 << 8 : 0) | (j == nblk - 1 ? 1 << 9 : 0);
      c.seg = b | (hg << 20);
      if (valid > 0) c.blk = __ldg(p.tables + static_cast<int64_t>(b) * p.table_stride + j);
    }
    return c;
  };
  Chunk cur{}, nxt{};
  bool c_ok = false, n_ok = false;
  if (my_e > my_a) {  // the range's first two chunks
    cur = build_chunk(my_a);
    c_ok = true;
    if (my_a + cur.n < my_e) {
      nxt = build_chunk(my_a + cur.n);
      n_ok = true;
    }
  }
  int ib = 0;  // next item of cur to issue
  uint32_t issued = 0, consumed = 0;
  int32_t meta = 0;       // lane s: ring slot s flags (bit 0 data, then as in Chunk::meta)
  int32_t meta_seg = 0;   // lane s: sequence | head group << 20 of ring slot s
  int32_t meta_slot = 0;  // lane s: partial slot of ring slot s
  int32_t meta_blk = 0;   // lane s: pool block of ring slot s

  // Copy one block (K and V of the HP packed heads, and the segment's q rows
  // with its first block) into the next ring slot as one cp.async group.
  auto issue_one = [&]() {
    const uint32_t slot = issued % kRing;
    const uint32_t sdst = smem_u32(ring + slot * Geo::kSlot);
    const int32_t blk = __shfl_sync(0xffffffffu, cur.blk, ib);
    const int32_t mt = __shfl_sync(0xffffffffu, cur.meta, ib);
    const int32_t sg = __shfl_sync(0xffffffffu, cur.seg, ib);
    const int32_t sl = __shfl_sync(0xffffffffu, cur.slot, ib);
    const int valid = (mt >> 1) & 31;
    const bool first = (mt >> 6) & 1;
    const int sb = sg & 0xfffff, shg = sg >> 20;
    bool ok = valid > 0;
    if (ok && (blk < 0 || blk >= p.num_blocks)) {
      if (lane == 0) flag_error(p.err, PSB_DEVERR_BLOCK_RANGE);
      ok = false;
    }
    // The slot's previous contents were read (ldmatrix) before the __syncwarp
    // that precedes every refill.
    if (ok) {
      const int64_t tile = zlayer + static_cast<int64_t>(blk) * p.hkv + shg * HP;
      const char* ksrc = reinterpret_cast<const char*>(kpool + tile * (16 * 64)) + lane * 16;
      const char* vsrc = reinterpret_cast<const char*>(vpool + tile * (16 * 64)) + lane * 16;
      // Append: the sequence's new token is row valid - 1 of its last block.
      // That row is copied straight from the caller's new K/V - the pool row
      // is stale until the consume side stores it there from the ring - and
      // only this warp reads this block in this launch.
      const bool app = APPEND && ((mt >> 9) & 1);
      const int r_new = valid - 1;
      const char* nk = nullptr;
      const char* nv = nullptr;
      if (app) {
        nk = p.new_k + (static_cast<int64_t>(sb) * p.nks + static_cast<int64_t>(shg * HP) * p.nkh) * sizeof(T);
        nv = p.new_v + (static_cast<int64_t>(sb) * p.nvs + static_cast<int64_t>(shg * HP) * p.nvh) * sizeof(T);
      }
      // a 16 x 64 tile is 2 KB = 128 chunks: 4 per lane, HP tiles per box;
      // chunk lane + 32 i sits at row 4 (i % 4) + lane / 8 of tile i / 4, so
      // the swizzled column alternates between two per-lane values
      if (!app) {  // warp-uniform: only a sequence's last block takes the other loop
#pragma unroll
        for (int i = 0; i < HP * 4; ++i) {
          const uint32_t d = sdst + i * 512 + ((i & 1) ? cp_dst_odd : cp_dst_even);
          cp_async16_hint(d, ksrc + i * 512, stream_pol);
          cp_async16_hint(d + Geo::kKV, vsrc + i * 512, stream_pol);
        }
      } else {
#pragma unroll
        for (int i = 0; i < HP * 4; ++i) {
          const uint32_t d = sdst + i * 512 + ((i & 1) ? cp_dst_odd : cp_dst_even);
          const char* ks = ksrc + i * 512;
          const char* vs = vsrc + i * 512;
          if (4 * (i & 3) + (lane >> 3) == r_new) {
            ks = nk + (i >> 2) * p.nkh * sizeof(T) + cp_col * 16;
            vs = nv + (i >> 2) * p.nvh * sizeof(T) + cp_col * 16;
          }
          cp_async16_hint(d, ks, stream_pol);
          cp_async16_hint(d + Geo::kKV, vs, stream_pol);
        }
      }
    }
    if (first) {
      // q rows of kv head hg*HP + s go to tile rows s*8 (HP = 2) or 0 (HP = 1)
      const T* qb = reinterpret_cast<const T*>(p.q) + static_cast<int64_t>(sb) * p.qsb;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = cp_row0 + 4 * i;  // tile row 0..15
        const int s = HP == 2 ? r >> 3 : 0;
        const int rr = HP == 2 ? r & 7 : r;
        if (rr < G) {
          const T* src = qb + static_cast<int64_t>((shg * HP + s) * G + rr) * p.qsh + cp_col * 8;
          cp_async16(sdst + 2 * Geo::kKV + r * 128 + cp_col * 16, src);
        }
      }
    }
    cp_async_commit();
    if (lane == static_cast<int>(slot)) {
      meta = (ok ? 1 : 0) | (mt & ~1);
      meta_seg = sg;
      meta_slot = sl;
      meta_blk = blk;
    }
    ++issued;
    if (++ib == cur.n) {  // advance to the next chunk; build the one after it
      c_ok = n_ok;
      cur = nxt;
      ib = 0;
      n_ok = false;
      if (c_ok && cur.beg + cur.n < my_e) {
        nxt = build_chunk(cur.beg + cur.n);
        n_ok = true;
      }
    }
  };

  // Everything above reads only lengths and tables.  The pool and q may still
  // be being written by the stream predecessor (a reshape_and_cache launched
  // just before lets this kernel start early), so wait for it here; the
  // combine kernel may launch as soon as every CTA is past this point.
  pdl_wait();
  pdl_launch_dependents();
  while (c_ok && issued - consumed < static_cast<uint32_t>(kRing)) issue_one();

  // ---- consume side ------------------------------------------------------
  uint32_t qa[4][4];   // A fragments per k-step (a0..a3)
  float o[8][4];       // rows g (c0, c1) and g + 8 (c2, c3), dims 8n + 2t + {0, 1}
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  int32_t cseg = 0, cslot = 0;
  bool cfull = false;  // the current segment began at its sequence's first block
  while (consumed != issued) {
    const uint32_t slot = consumed % kRing;
    const int32_t mt = __shfl_sync(0xffffffffu, meta, slot);
    const bool first = (mt >> 6) & 1, last = (mt >> 7) & 1;
    const int valid = (mt & 1) ? (mt >> 1) & 31 : 0;
    if (first) {
      cseg = __shfl_sync(0xffffffffu, meta_seg, slot);
      cslot = __shfl_sync(0xffffffffu, meta_slot, slot);
      cfull = (mt >> 8) & 1;
    }
    // the oldest copy group is complete once at most the newer ones are pending
    const uint32_t inflight = issued - consumed;
    cp_async_wait_oldest<kRing>(inflight);
    __syncwarp();  // every lane's copies are visible to every lane
    const uint32_t sbase = smem_u32(ring + slot * Geo::kSlot);
    if (APPEND && valid && ((mt >> 9) & 1)) {  // uniform over the warp
      // append: store the new token's K/V rows, now in the ring (row r at
      // r * 128, 16-byte column c at (c ^ r % 8) * 16 of its tile), into the
      // pool; lane = (K | V) x head slot x column
      const int32_t blk = __shfl_sync(0xffffffffu, meta_blk, slot);
      const int kv = lane >> 4, hs = (lane >> 3) & 1, col = lane & 7, r_new = valid - 1;
      if (hs < HP) {
        const int64_t tile = zlayer + static_cast<int64_t>(blk) * p.hkv + ((cseg >> 20) & 0xff) * HP + hs;
        const uint4 row = ld_shared_v4(sbase + kv * Geo::kKV + hs * kTileBytes + r_new * 128 +
                                       ((col ^ (r_new & 7)) << 4));
        *reinterpret_cast<uint4*>((kv ? p.v_pool_w : p.k_pool_w) + (tile * 16 + r_new) * 128 + col * 16) = row;
      }
    }
    if (first) {
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
    if (c_ok) issue_one();  // refill the slot just freed

    if (last) {
      // ---- finish the segment ----------------------------------------------
      float ll = l_lo, lh = l_hi;
      ll += __shfl_xor_sync(0xffffffffu, ll, 1);
      lh += __shfl_xor_sync(0xffffffffu, lh, 1);
      ll += __shfl_xor_sync(0xffffffffu, ll, 2);
      lh += __shfl_xor_sync(0xffffffffu, lh, 2);
      const int sb = cseg & 0xfffff, shg = (cseg >> 20) & 0xff;
      if (cfull && ((mt >> 9) & 1)) {  // the segment is the whole sequence
        const int qh_lo = HP == 2 ? (shg * 2) * G + g : shg * G + g;
        const int qh_hi = HP == 2 ? (shg * 2 + 1) * G + g : shg * G + g + 8;
        const float il = ll > 0.f ? 1.f / ll : 0.f, ih = lh > 0.f ? 1.f / lh : 0.f;
        T* olo = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(sb) * p.osb + static_cast<int64_t>(qh_lo) * p.osh;
        T* ohi = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(sb) * p.osb + static_cast<int64_t>(qh_hi) * p.osh;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          if (row_lo) *reinterpret_cast<uint32_t*>(olo + n * 8 + 2 * t) = pack2<T>(o[n][0] * il, o[n][1] * il);
          if (row_hi) *reinterpret_cast<uint32_t*>(ohi + n * 8 + 2 * t) = pack2<T>(o[n][2] * ih, o[n][3] * ih);
        }
      } else {
        // partial: 16 tile rows, row g (lo) and g + 8 (hi), merged after this
        // launch by decode_combine_kernel
        float* po = p.part_o + static_cast<int64_t>(cslot) * kPartFloats;
        float* pml = p.part_ml + static_cast<int64_t>(cslot) * 32;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          *reinterpret_cast<float2*>(po + g * 64 + n * 8 + 2 * t) = make_float2(o[n][0], o[n][1]);
          *reinterpret_cast<float2*>(po + (g + 8) * 64 + n * 8 + 2 * t) = make_float2(o[n][2], o[n][3]);
        }
        if (t == 0) {
          *reinterpret_cast<float2*>(pml + 2 * g) = make_float2(m_lo, ll);
          *reinterpret_cast<float2*>(pml + 2 * (g + 8)) = make_float2(m_hi, lh);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// split-K merge for the fast path: one CTA per (sequence, head group).
// Launched right after decode_fast_kernel on the same stream, it starts while
// the decode still runs: from the context lengths alone (stable for the whole
// decode) it works out which warps hold pieces of its sequence, exactly as
// the decode split them, and lists their partial slots in shared memory.  A
// sequence inside one warp's range was finished by the decode and the CTA
// exits.  Then griddepcontrol.wait - every partial visible - and thread (row,
// 4-dim slice) loads the partials of up to kCombBatch warps at once (one
// memory round trip for most sequences), rescales them to their common
// maximum and writes the normalised output.
// ---------------------------------------------------------------------------
constexpr int kCombThreads = 256;  // 16 tile rows x 16 slices of 4 dims
constexpr int kCombBatch = 12;

template <typename T, int HP>
__global__ void __launch_bounds__(kCombThreads, 2) decode_combine_kernel(const DecodeParams p) {
  __shared__ int32_t s_slot[kFastWarps * kMaxFastCtas];  // a piece per warp at most
  __shared__ int32_t s_red[2][kCombThreads / 32];
  __shared__ int32_t s_nblk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int groups = p.hkv / HP;
  const int b = blockIdx.x / groups, hg = blockIdx.x - b * groups;
  // blocks before sequence b and in total (item counts are below 2^31), with
  // the decode's clamp of each length (the decode flags bad lengths)
  int before = 0, total = 0;
  for (int i = tid; i < p.batch; i += kCombThreads) {
    int n = p.ctx[i];
    n = n < 0 ? 0 : (n > p.max_context ? p.max_context : n);
    const int nb = blocks_of(n);
    total += nb;
    before += i < b ? nb : 0;
    if (i == b) s_nblk = nb;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    before += __shfl_xor_sync(0xffffffffu, before, o);
    total += __shfl_xor_sync(0xffffffffu, total, o);
  }
  if (lane == 0) {
    s_red[0][warp] = before;
    s_red[1][warp] = total;
  }
  __syncthreads();
  before = total = 0;
#pragma unroll
  for (int w = 0; w < kCombThreads / 32; ++w) {
    before += s_red[0][w];
    total += s_red[1][w];
  }
  const int64_t nb_total = total;
  const Split split(nb_total * groups, p.total_warps);
  const int64_t first = hg * nb_total + before, last = first + s_nblk - 1;
  const int wa = split.warp_of(first), wb = split.warp_of(last);
  if (wa == wb) return;  // inside one warp's range: written by the decode
  const int np = wb - wa + 1;
  for (int k = tid; k < np; k += kCombThreads) {
    const int64_t s0 = split.start(wa + k), s1 = split.start(wa + k + 1);
    s_slot[k] = s0 == s1 ? -1 : 2 * (wa + k) + (s0 < first ? 1 : 0);  // an empty range wrote nothing
  }
  __syncthreads();

  pdl_wait();
  // the next kernel on the stream may launch now; if it is a programmatic
  // dependent it waits for this grid before touching memory
  pdl_launch_dependents();
  const int r = tid >> 4, q4 = tid & 15;
  float M = -INFINITY, L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < np; k0 += kCombBatch) {
    float2 ml[kCombBatch];
    float4 v[kCombBatch];
#pragma unroll
    for (int k = 0; k < kCombBatch; ++k) {
      ml[k] = make_float2(-INFINITY, 0.f);
      v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int slot_id = k0 + k < np ? s_slot[k0 + k] : -1;
      if (slot_id >= 0) {
        ml[k] = __ldcg(reinterpret_cast<const float2*>(p.part_ml) + slot_id * 16 + r);
        v[k] = __ldcg(reinterpret_cast<const float4*>(p.part_o) + slot_id * (kPartFloats / 4) + r * 16 + q4);
      }
    }
    float mb = M;
#pragma unroll
    for (int k = 0; k < kCombBatch; ++k) mb = fmaxf(mb, ml[k].x);
    if (mb == -INFINITY) continue;
    const float sc = exp2f((M - mb) * p.scale_log2);  // 0 while M is -inf
    M = mb;
    L *= sc;
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] *= sc;
#pragma unroll
    for (int k = 0; k < kCombBatch; ++k) {
      if (ml[k].x == -INFINITY) continue;
      const float wt = exp2f((ml[k].x - M) * p.scale_log2);
      L = fmaf(ml[k].y, wt, L);
      acc[0] = fmaf(v[k].x, wt, acc[0]);
      acc[1] = fmaf(v[k].y, wt, acc[1]);
      acc[2] = fmaf(v[k].z, wt, acc[2]);
      acc[3] = fmaf(v[k].w, wt, acc[3]);
    }
  }
  const int G = p.group;
  const int s = HP == 2 ? r >> 3 : 0, rr = HP == 2 ? r & 7 : r;
  if (rr >= G) return;
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int qh = (hg * HP + s) * G + rr;
  T* orow = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(b) * p.osb + static_cast<int64_t>(qh) * p.osh + q4 * 4;
  *reinterpret_cast<uint32_t*>(orow) = pack2<T>(acc[0] * inv, acc[1] * inv);
  *reinterpret_cast<uint32_t*>(orow + 2) = pack2<T>(acc[2] * inv, acc[3] * inv);
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

// Append on the CUDA-core path: row b's new K/V at position ctx[b] - 1,
// located through its block table as PagedKVCache.write_token does
// (pagedserve/engine/paged_kv_cache.py:187-200), one element per thread;
// launched before decode_generic_kernel on the same stream.
template <typename T>
__global__ void __launch_bounds__(256) append_rows_kernel(const DecodeParams p) {
  const int D = p.head_dim, BS = p.block_size;
  const int64_t per = static_cast<int64_t>(p.hkv) * D;
  const int64_t total = per * p.batch;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / per);
    const int r = static_cast<int>(i - b * per);
    const int h = r / D, d = r - h * D;
    const int ctx = p.ctx[b];
    if (ctx <= 0 || ctx > p.max_context) continue;  // no position to write (the decode flags bad lengths)
    const int pos = ctx - 1;
    const int blk = p.tables[static_cast<int64_t>(b) * p.table_stride + pos / BS];
    if (blk < 0 || blk >= p.num_blocks) {
      if (h == 0 && d == 0) flag_error(p.err, PSB_DEVERR_BLOCK_RANGE);
      continue;
    }
    const int64_t off = (((static_cast<int64_t>(p.layer) * p.num_blocks + blk) * p.hkv + h) * BS + pos % BS) * D + d;
    reinterpret_cast<T*>(p.k_pool_w)[off] = reinterpret_cast<const T*>(p.new_k)[b * p.nks + h * p.nkh + d];
    reinterpret_cast<T*>(p.v_pool_w)[off] = reinterpret_cast<const T*>(p.new_v)[b * p.nvs + h * p.nvh + d];
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

// Generic-path split-K geometry: units of (sequence, kv head, 64-token
// chunk), ``group`` partial rows per unit, one arrival counter per
// (sequence, kv head).
struct SplitGeom {
  int chunk, rows, counters, batch;
  int64_t max_units;
};

SplitGeom split_geometry(int batch, int hkv, int group, int max_context) {
  SplitGeom sg;
  sg.chunk = kGenericChunk;
  const int64_t per = std::max<int64_t>(1, (static_cast<int64_t>(max_context) + sg.chunk - 1) / sg.chunk);
  sg.max_units = per * batch * hkv;
  sg.rows = group;
  sg.counters = batch * hkv;
  sg.batch = batch;
  return sg;
}

struct WorkspaceLayout {
  size_t counters_off, ml_off, o_off, total;
};

// Generic path: [arrival counters: int32 per (sequence, kv head) | pad to 256]
// [partial max/sum: max_units * rows * 2 f32][partial outputs: max_units * rows * head_dim f32].
// Every call clears the counters first (the fast path keeps scratch in the
// same bytes) and leaves them zero.
WorkspaceLayout workspace_layout(const SplitGeom& sg, int head_dim) {
  WorkspaceLayout w;
  w.counters_off = 0;
  w.ml_off = align_up(sizeof(int32_t) * static_cast<size_t>(sg.counters), 256);
  w.o_off = align_up(w.ml_off + sizeof(float) * static_cast<size_t>(sg.max_units) * sg.rows * 2, 256);
  w.total = w.o_off + sizeof(float) * static_cast<size_t>(sg.max_units) * sg.rows * head_dim;
  return w;
}

// Fast path: [partial max/sum: slots * 16 * 2 f32][partial outputs: slots *
// 16 * 64 f32], two partial slots per warp of a grid of at most kMaxFastCtas
// CTAs.  The size does not depend on the batch; nothing needs initialising.
struct FastLayout {
  size_t ml_off, o_off, total;
};

FastLayout fast_layout() {
  FastLayout f;
  const size_t slots = 2 * static_cast<size_t>(kFastWarps) * kMaxFastCtas;
  f.ml_off = 0;
  f.o_off = align_up(f.ml_off + sizeof(float) * slots * 32, 256);
  f.total = f.o_off + sizeof(float) * slots * kPartFloats;
  return f;
}

template <typename T, int HP>
int launch_fast(DecodeParams prm, cudaStream_t stream, int max_ctas) {
  const size_t smem = FastGeom<HP>::bytes(prm.batch);
  if (smem > 227 * 1024) return PSB_ERR_UNSUPPORTED;
  const bool append = prm.new_k != nullptr;
  const auto kernel = append ? decode_fast_kernel<T, HP, true> : decode_fast_kernel<T, HP, false>;
  int occ = 0;
  if (!kernel_occupancy(reinterpret_cast<const void*>(kernel), kFastThreads, smem, &occ) || occ < 1)
    return PSB_ERR_CUDA;
  // an upper bound of the items from the host-known maximum context; small
  // batches get fewer CTAs so each warp streams at least kFastMinBlocks blocks
  const int64_t max_items = static_cast<int64_t>(prm.batch) * (prm.hkv / HP) *
                            std::max<int64_t>(1, (static_cast<int64_t>(prm.max_context) + 15) / 16);
  const int64_t want = (max_items + kFastWarps * kFastMinBlocks - 1) / (kFastWarps * kFastMinBlocks);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, max_ctas)));
  prm.total_warps = grid * kFastWarps;
  discard_stale_error();
  cudaError_t e = launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), dim3(kFastThreads), smem, stream, prm);
  if (e != cudaSuccess) return record_cuda_error(e);
  const int64_t merges = static_cast<int64_t>(prm.batch) * (prm.hkv / HP);
  if (!prefer_max_shared(reinterpret_cast<const void*>(decode_combine_kernel<T, HP>))) return PSB_ERR_CUDA;
  e = launch_pdl(decode_combine_kernel<T, HP>, dim3(static_cast<unsigned>(merges)), dim3(kCombThreads), 0, stream,
                 prm);
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}

template <typename T>
int launch_generic(const DecodeParams& prm, cudaStream_t stream, int sms) {
  const size_t smem = generic_smem_bytes(prm.group, prm.head_dim, prm.batch);
  if (smem > 227 * 1024) return PSB_ERR_UNSUPPORTED;
  const void* kern = reinterpret_cast<const void*>(decode_generic_kernel<T>);
  int occ = 0;
  if (!kernel_occupancy(kern, kThreads, smem, &occ)) return PSB_ERR_CUDA;
  const int64_t grid = std::min<int64_t>(prm.max_units, static_cast<int64_t>(sms) * std::max(occ, 1));
  discard_stale_error();
  if (prm.new_k != nullptr) {
    const int64_t elems = static_cast<int64_t>(prm.batch) * prm.hkv * prm.head_dim;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((elems + 255) / 256, static_cast<int64_t>(sms) * 8));
    append_rows_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(prm);
  }
  decode_generic_kernel<T><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(prm);
  return check_launch();
}

// Which path a call takes (the fast path bulk-copies 16-byte q rows and
// writes the output in 4-byte pairs).
int choose_path(int dtype, int head_dim, int block_size, int group, int hkv, int batch, int max_context,
                const void* query, int64_t qsb, int64_t qsh, const void* out, int64_t osb, int64_t osh, const void* kc,
                const void* vc) {
  const int hp = fast_heads_per_unit(dtype, head_dim, block_size, group, hkv);
  if (!hp || batch > kMaxFastBatch) return 0;
  const bool aligned = qsh % 8 == 0 && qsb % 8 == 0 && reinterpret_cast<uintptr_t>(query) % 16 == 0 &&
                       osh % 2 == 0 && osb % 2 == 0 && reinterpret_cast<uintptr_t>(out) % 4 == 0 &&
                       reinterpret_cast<uintptr_t>(kc) % 16 == 0 && reinterpret_cast<uintptr_t>(vc) % 16 == 0;
  const size_t smem = hp == 2 ? FastGeom<2>::bytes(batch) : FastGeom<1>::bytes(batch);
  // item indices are int32 inside the kernel
  const int64_t max_items = static_cast<int64_t>(batch) * (hkv / hp) *
                            std::max<int64_t>(1, (static_cast<int64_t>(max_context) + 15) / 16);
  const bool fits = max_items < (int64_t(1) << 31);
  return aligned && fits && smem <= 227 * 1024 ? hp : 0;
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
  // (the fast path also depends on pointer alignment, known only at the call)
  const int hp = fast_heads_per_unit(dtype, head_dim, block_size, group, num_kv_heads);
  const size_t fast = hp ? fast_layout().total : 0;
  const size_t gen = workspace_layout(split_geometry(batch, num_kv_heads, group, max_context), head_dim).total;
  return std::max(fast, gen);
}

size_t psb::decode_scratch_for_call(const void* query, int64_t q_stride_b, int64_t q_stride_h, const void* out,
                                    int64_t o_stride_b, int64_t o_stride_h, const void* k_cache,
                                    const void* v_cache, int32_t batch, int32_t q_heads, int32_t num_kv_heads,
                                    int32_t block_size, int32_t head_dim, int32_t dtype, int32_t max_context) {
  if (batch <= 0 || num_kv_heads <= 0 || q_heads <= 0 || q_heads % num_kv_heads || head_dim <= 0 ||
      block_size <= 0 || max_context < 0)
    return 0;
  const int group = q_heads / num_kv_heads;
  const int hp = choose_path(dtype, head_dim, block_size, group, num_kv_heads, batch, max_context, query, q_stride_b,
                             q_stride_h, out, o_stride_b, o_stride_h, k_cache, v_cache);
  if (hp) return fast_layout().total;
  return workspace_layout(split_geometry(batch, num_kv_heads, group, max_context), head_dim).total;
}

extern "C" int psb_paged_decode_workspace_init(void* workspace, size_t workspace_bytes, int32_t batch,
                                               int32_t num_kv_heads, psb_stream_t stream) {
  if (workspace == nullptr || batch <= 0 || num_kv_heads <= 0) return PSB_ERR_INVALID;
  SplitGeom sg{kGenericChunk, 1, batch * num_kv_heads, batch, 0};
  const size_t need = workspace_layout(sg, 1).ml_off;
  if (workspace_bytes < need) return PSB_ERR_WORKSPACE;
  const cudaError_t e = cudaMemsetAsync(workspace, 0, need, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return PSB_ERR_CUDA;
  }
  return PSB_OK;
}

namespace psb {
namespace {

// psb_paged_decode, and with new_key != nullptr psb_paged_decode_append.
int paged_decode_impl(const void* query, int64_t q_stride_b, int64_t q_stride_h, void* out, int64_t o_stride_b,
                      int64_t o_stride_h, const void* k_cache, const void* v_cache, const void* new_key,
                      int64_t key_stride_b, int64_t key_stride_h, const void* new_value, int64_t value_stride_b,
                      int64_t value_stride_h, const int32_t* block_tables, int64_t table_stride,
                      const int32_t* context_lens, int32_t batch, int32_t q_heads, int32_t layer, int32_t num_layers,
                      int64_t num_blocks, int32_t num_kv_heads, int32_t block_size, int32_t head_dim, int32_t dtype,
                      int32_t max_context, float scale, void* workspace, size_t workspace_bytes, int32_t* error_flag,
                      psb_stream_t stream) {
  if (!query || !out || !k_cache || !v_cache || !block_tables || !context_lens) return PSB_ERR_INVALID;
  if (batch <= 0 || q_heads <= 0 || num_kv_heads <= 0 || q_heads % num_kv_heads || head_dim <= 0 ||
      block_size <= 0 || num_blocks <= 0 || num_layers <= 0 || layer < 0 || layer >= num_layers ||
      max_context < 0 || table_stride < (max_context + block_size - 1) / block_size)
    return PSB_ERR_INVALID;
  if (dtype != PSB_F32 && dtype != PSB_F16 && dtype != PSB_BF16) return PSB_ERR_INVALID;
  if (static_cast<int64_t>(num_layers) * num_blocks * num_kv_heads >= (int64_t(1) << 31)) return PSB_ERR_UNSUPPORTED;
  const int group = q_heads / num_kv_heads;
  int hp = choose_path(dtype, head_dim, block_size, group, num_kv_heads, batch, max_context, query, q_stride_b,
                       q_stride_h, out, o_stride_b, o_stride_h, k_cache, v_cache);
  if (new_key != nullptr) {
    // the fast path copies new rows in 16-byte pieces
    const bool rows16 = key_stride_b % 8 == 0 && key_stride_h % 8 == 0 && value_stride_b % 8 == 0 &&
                        value_stride_h % 8 == 0 && reinterpret_cast<uintptr_t>(new_key) % 16 == 0 &&
                        reinterpret_cast<uintptr_t>(new_value) % 16 == 0;
    if (!rows16) hp = 0;
  }
  const int sms = device_sm_count();
  if (sms <= 0) return PSB_ERR_CUDA;
  if (workspace == nullptr) return PSB_ERR_WORKSPACE;

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
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = error_flag;
  p.total_warps = 0;
  p.new_k = static_cast<const char*>(new_key);
  p.new_v = static_cast<const char*>(new_value);
  p.nks = key_stride_b;
  p.nkh = key_stride_h;
  p.nvs = value_stride_b;
  p.nvh = value_stride_h;
  p.k_pool_w = const_cast<char*>(static_cast<const char*>(k_cache));
  p.v_pool_w = const_cast<char*>(static_cast<const char*>(v_cache));
  char* ws = static_cast<char*>(workspace);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (hp) {
    const FastLayout fl = fast_layout();
    const int max_ctas = std::min(sms, kMaxFastCtas);
    if (workspace_bytes < fl.total) return PSB_ERR_WORKSPACE;
    p.chunk = 0;
    p.counters = nullptr;
    p.part_ml = reinterpret_cast<float*>(ws + fl.ml_off);
    p.part_o = reinterpret_cast<float*>(ws + fl.o_off);
    p.max_units = 0;
    if (dtype == PSB_BF16)
      return hp == 2 ? launch_fast<__nv_bfloat16, 2>(p, s, max_ctas) : launch_fast<__nv_bfloat16, 1>(p, s, max_ctas);
    return hp == 2 ? launch_fast<__half, 2>(p, s, max_ctas) : launch_fast<__half, 1>(p, s, max_ctas);
  }
  const SplitGeom sg = split_geometry(batch, num_kv_heads, group, max_context);
  const WorkspaceLayout wl = workspace_layout(sg, head_dim);
  if (workspace_bytes < wl.total) return PSB_ERR_WORKSPACE;
  p.chunk = sg.chunk;
  p.counters = reinterpret_cast<int32_t*>(ws + wl.counters_off);
  p.part_ml = reinterpret_cast<float*>(ws + wl.ml_off);
  p.part_o = reinterpret_cast<float*>(ws + wl.o_off);
  p.max_units = sg.max_units;
  const cudaError_t ze = cudaMemsetAsync(p.counters, 0, sizeof(int32_t) * static_cast<size_t>(sg.counters), s);
  if (ze != cudaSuccess) return record_cuda_error(ze);
  switch (dtype) {
    case PSB_BF16: return launch_generic<__nv_bfloat16>(p, s, sms);
    case PSB_F16: return launch_generic<__half>(p, s, sms);
    default: return launch_generic<float>(p, s, sms);
  }
}

}  // namespace
}  // namespace psb

extern "C" int psb_paged_decode(const void* query, int64_t q_stride_b, int64_t q_stride_h, void* out,
                                int64_t o_stride_b, int64_t o_stride_h, const void* k_cache, const void* v_cache,
                                const int32_t* block_tables, int64_t table_stride, const int32_t* context_lens,
                                int32_t batch, int32_t q_heads, int32_t layer, int32_t num_layers,
                                int64_t num_blocks, int32_t num_kv_heads, int32_t block_size, int32_t head_dim,
                                int32_t dtype, int32_t max_context, float scale, void* workspace,
                                size_t workspace_bytes, int32_t* error_flag, psb_stream_t stream) {
  return paged_decode_impl(query, q_stride_b, q_stride_h, out, o_stride_b, o_stride_h, k_cache, v_cache, nullptr, 0, 0,
                           nullptr, 0, 0, block_tables, table_stride, context_lens, batch, q_heads, layer, num_layers,
                           num_blocks, num_kv_heads, block_size, head_dim, dtype, max_context, scale, workspace,
                           workspace_bytes, error_flag, stream);
}

extern "C" size_t psb_decode_args_size(void) { return sizeof(psb_decode_args); }

// The fixed arguments from the caller's struct, the per-call ones as given.
extern "C" int psb_paged_decode_args(const psb_decode_args* a, const void* query, int64_t q_stride_b,
                                     int64_t q_stride_h, void* out, int64_t o_stride_b, int64_t o_stride_h,
                                     const void* new_key, int64_t key_stride_b, int64_t key_stride_h,
                                     const void* new_value, int64_t value_stride_b, int64_t value_stride_h,
                                     int32_t layer, psb_stream_t stream) {
  if (a == nullptr || (new_key == nullptr) != (new_value == nullptr)) return PSB_ERR_INVALID;
  return paged_decode_impl(query, q_stride_b, q_stride_h, out, o_stride_b, o_stride_h, a->k_cache, a->v_cache,
                           new_key, key_stride_b, key_stride_h, new_value, value_stride_b, value_stride_h,
                           a->block_tables, a->table_stride, a->context_lens, a->batch, a->q_heads, layer,
                           a->num_layers, a->num_blocks, a->num_kv_heads, a->block_size, a->head_dim, a->dtype,
                           a->max_context, a->scale, a->workspace, a->workspace_bytes, a->error_flag, stream);
}

extern "C" int psb_paged_decode_append(const void* query, int64_t q_stride_b, int64_t q_stride_h, void* out,
                                       int64_t o_stride_b, int64_t o_stride_h, void* k_cache, void* v_cache,
                                       const void* new_key, int64_t key_stride_b, int64_t key_stride_h,
                                       const void* new_value, int64_t value_stride_b, int64_t value_stride_h,
                                       const int32_t* block_tables, int64_t table_stride, const int32_t* context_lens,
                                       int32_t batch, int32_t q_heads, int32_t layer, int32_t num_layers,
                                       int64_t num_blocks, int32_t num_kv_heads, int32_t block_size, int32_t head_dim,
                                       int32_t dtype, int32_t max_context, float scale, void* workspace,
                                       size_t workspace_bytes, int32_t* error_flag, psb_stream_t stream) {
  if (!new_key || !new_value) return PSB_ERR_INVALID;
  return paged_decode_impl(query, q_stride_b, q_stride_h, out, o_stride_b, o_stride_h, k_cache, v_cache, new_key,
                           key_stride_b, key_stride_h, new_value, value_stride_b, value_stride_h, block_tables,
                           table_stride, context_lens, batch, q_heads, layer, num_layers, num_blocks, num_kv_heads,
                           block_size, head_dim, dtype, max_context, scale, workspace, workspace_bytes, error_flag,
                           stream);
}
