// select_tokens: greedy token selection and the stop check of one decode
// step, on the device, for every row of the batch in one launch.
//
// The reference picks each next token with
//     tokens = logits[:, -1, :].argmax(dim=-1, keepdim=True)
// and then, per row on the host, reads the token with .item(), appends it to
// the request (Request.add_generated_token raises when no tokens remain) and
// finishes the request when the token is an EOS id or no tokens remain
// (pagedserve/engine/continuous_batcher.py:333-360,
//  pagedserve/engine/request.py:84-106).  Here the argmax, the append's
// limit check, the countdown and the stop test all run on the GPU; the host
// reads B tokens and B status bytes with one copy instead of B syncs.
//
// argmax semantics are torch's: the first index of the maximum, NaN counted
// as larger than every number (the first NaN wins), -0.0 equal to +0.0.
//
// Layout: one row of V logits per request (any row stride, unit element
// stride).  Each row is split over the C CTAs of a thread-block cluster, and
// the C partial results meet in CTA 0's shared memory (distributed shared
// memory) - no global atomics, no workspace, nothing to reset between steps.
// The kernels are bound by HBM: they read B * V * sizeof(T) bytes once.
//
// Streaming kernel (16-byte aligned rows): a single wave of persistent
// clusters (as many as are co-resident), each owning an equal count of rows.
// CTA r of a cluster owns slice r of each of its rows, and each warp an equal
// contiguous part of that slice, which it streams through three 4 KB
// shared-memory slots with bulk async copies it issues itself (no cross-warp
// synchronisation).  Per piece: a branch-free packed maximum (max.NaN on
// bf16x2 / f16x2 / f32) of each lane's vectors; the lane keeps its record
// value and the piece where it first reached it.  At the end of a row the
// warp takes the maximum over its lanes and the earliest piece where a lane
// reached it, and only those lanes read their vectors of that piece again
// (from global memory: 128 bytes each) to find the first index.  The warps'
// results meet in their CTA, each CTA stores its per-row result into CTA 0's
// shared memory, and CTA 0 finishes the rows after the cluster barrier.
//
// Register kernel (rows off a 16-byte boundary): grid (C, B), one cluster
// per row; each thread keeps a running (value, first index) over its
// strided elements.
#include <cooperative_groups.h>

#include <algorithm>
#include <climits>
#include <map>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "host_util.h"

namespace cg = cooperative_groups;

namespace psb {
namespace {

constexpr int kSelThreads = 256;
constexpr int kSelUnroll = 4;
constexpr int kMaxCluster = 8;
// CTAs per row when the caller leaves it to the library.  On the
// 151936-entry bf16 vocabulary, 2 measured within 0.5 % of the fastest at 128
// and 256 rows (128: 12.43 us, 1: 12.40, 6: 12.65, 4: 14.0, 8: 14.8; 256:
// 18.98 us, 1: 18.91, 6: 19.76, 4: 19.93, 8: 24.7): fewer, longer row
// slices per warp amortise the per-row merge.  Small batches spread each row
// wider so the grid still covers the GPU.
constexpr int kAutoCluster = 2;
constexpr int kAutoClusterSmall = 6;
constexpr int kSmallBatch = 64;
constexpr int kMaxEos = 64;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSlotBytes = 4096;                  // one piece of a warp's stream
constexpr int kSlots = 3;                         // pieces in flight per warp (2: 12.3 / 19.0 us at 128 / 256 rows; 3: 11.2 / 18.6)
constexpr int kSlotVecs = kSlotBytes / 16;
constexpr int kVecPerLane = kSlotVecs / 32;
constexpr int kRingBytes = kSelWarps * kSlots * kSlotBytes;
constexpr int kMaxRowsPerCluster = 64;            // CTA 0's per-row key slots

// Monotone map of a float onto uint32 order: a > b  <=>  key(a) > key(b)
// for numbers; every NaN maps to the top key; -0.0 maps like +0.0.
__device__ __forceinline__ uint32_t order_key(float x) {
  if (x != x) return 0xFFFFFFFFu;
  uint32_t u = __float_as_uint(x);
  if (x == 0.0f) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Larger key = larger value, then smaller index.  Index < 2^31.
__device__ __forceinline__ uint64_t pack_key(uint32_t vkey, int32_t idx) {
  return (static_cast<uint64_t>(vkey) << 32) | static_cast<uint32_t>(~idx);
}

__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Float value of one 16-bit lane of a packed pair (lane 0 = low half).
template <typename T>
__device__ __forceinline__ float lane_f(uint32_t w, int lane);
template <>
__device__ __forceinline__ float lane_f<__nv_bfloat16>(uint32_t w, int lane) {
  return __uint_as_float(lane ? (w & 0xFFFF0000u) : (w << 16));
}
template <>
__device__ __forceinline__ float lane_f<__half>(uint32_t w, int lane) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(lane ? (w >> 16) : (w & 0xFFFFu))));
}

// NaN-propagating max of two packed 16-bit pairs.
template <typename T>
__device__ __forceinline__ uint32_t pair_max(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t pair_max<__nv_bfloat16>(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <>
__device__ __forceinline__ uint32_t pair_max<__half>(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ uint32_t word(const uint4& r, int i) {
  return i == 0 ? r.x : i == 1 ? r.y : i == 2 ? r.z : r.w;
}

// One 16-byte vector of T: its element count, its maximum, element i, and a
// packed running maximum (four independent accumulators, no branches).
template <typename T>
struct Vec {
  static constexpr int N = 8;
  static constexpr uint32_t kNegInfPair = std::is_same<T, __half>::value ? 0xFC00FC00u : 0xFF80FF80u;
  __device__ static float vmax(const uint4& r) {
    const uint32_t m = pair_max<T>(pair_max<T>(r.x, r.y), pair_max<T>(r.z, r.w));
    return max_nan(lane_f<T>(m, 0), lane_f<T>(m, 1));
  }
  __device__ static float at(const uint4& r, int i) { return lane_f<T>(word(r, i >> 1), i & 1); }
  struct Acc {
    uint32_t a0 = kNegInfPair, a1 = kNegInfPair, a2 = kNegInfPair, a3 = kNegInfPair;
    __device__ void add(const uint4& r) {
      a0 = pair_max<T>(a0, r.x);
      a1 = pair_max<T>(a1, r.y);
      a2 = pair_max<T>(a2, r.z);
      a3 = pair_max<T>(a3, r.w);
    }
    __device__ float result() const {
      const uint32_t m = pair_max<T>(pair_max<T>(a0, a1), pair_max<T>(a2, a3));
      return max_nan(lane_f<T>(m, 0), lane_f<T>(m, 1));
    }
  };
};

template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static float vmax(const uint4& r) {
    return max_nan(max_nan(__uint_as_float(r.x), __uint_as_float(r.y)),
                   max_nan(__uint_as_float(r.z), __uint_as_float(r.w)));
  }
  __device__ static float at(const uint4& r, int i) { return __uint_as_float(word(r, i)); }
  struct Acc {
    float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
    __device__ void add(const uint4& r) {
      a0 = max_nan(a0, __uint_as_float(r.x));
      a1 = max_nan(a1, __uint_as_float(r.y));
      a2 = max_nan(a2, __uint_as_float(r.z));
      a3 = max_nan(a3, __uint_as_float(r.w));
    }
    __device__ float result() const { return max_nan(max_nan(a0, a1), max_nan(a2, a3)); }
  };
};

__device__ __forceinline__ float load_scalar(const float* p) { return __ldcs(p); }
__device__ __forceinline__ float load_scalar(const __half* p) {
  return lane_f<__half>(__ldcs(reinterpret_cast<const unsigned short*>(p)), 0);
}
__device__ __forceinline__ float load_scalar(const __nv_bfloat16* p) {
  return lane_f<__nv_bfloat16>(__ldcs(reinterpret_cast<const unsigned short*>(p)), 0);
}

// a equals the maximum m in the order of the keys: NaN matches NaN, and
// -0.0 matches +0.0 (float equality already treats them alike)
__device__ __forceinline__ bool same_value(float a, float m) { return m == m ? a == m : a != a; }

// Lane of vector r holding the maximum m first (r is known to hold it).
template <typename T>
__device__ __forceinline__ int first_lane(const uint4& r, float m) {
  int j = 0;
#pragma unroll
  for (int e = Vec<T>::N - 1; e >= 0; --e)
    if (same_value(Vec<T>::at(r, e), m)) j = e;
  return j;
}

// The reference's per-row bookkeeping for a row whose argmax is packed in `key`.
__device__ __forceinline__ void finish_row(int row, uint64_t key, const int64_t* __restrict__ eos_ids,
                                           int32_t num_eos, int32_t* __restrict__ remaining,
                                           int64_t* __restrict__ tokens, uint8_t* __restrict__ status,
                                           int32_t* err) {
  const int32_t tok = static_cast<int32_t>(~static_cast<uint32_t>(key));
  tokens[row] = tok;
  // Request.add_generated_token: a row with no tokens left is an error
  // (the token is still reported; nothing is counted).
  const int32_t rem = remaining[row];
  uint8_t st;
  if (rem <= 0) {
    flag_error(err, PSB_DEVERR_LIMIT);
    st = PSB_SELECT_DONE | PSB_SELECT_LIMIT;
  } else {
    bool eos = false;
    for (int e = 0; e < num_eos; ++e) eos |= __ldg(eos_ids + e) == tok;
    remaining[row] = rem - 1;
    st = static_cast<uint8_t>(((eos || rem - 1 == 0) ? PSB_SELECT_DONE : 0) | (eos ? PSB_SELECT_EOS : 0));
  }
  status[row] = st;
}

// CTA 0 of the row's cluster merges the CTAs' keys (each in its own
// `s_cta`) and finishes the row.
__device__ __forceinline__ void merge_and_finish(cg::cluster_group& cluster, uint64_t* s_cta, int row,
                                                 const int64_t* __restrict__ eos_ids, int32_t num_eos,
                                                 int32_t* __restrict__ remaining, int64_t* __restrict__ tokens,
                                                 uint8_t* __restrict__ status, int32_t* err) {
  // Every CTA's key is in its shared memory before CTA 0 reads them, and no
  // CTA exits before CTA 0 has read.
  cluster.sync();
  if (cluster.block_rank() == 0 && threadIdx.x == 0) {
    uint64_t k = *s_cta;
    const int csize = static_cast<int>(cluster.num_blocks());
    for (int r = 1; r < csize; ++r) {
      const uint64_t o = *cluster.map_shared_rank(s_cta, r);
      k = o > k ? o : k;
    }
    finish_row(row, k, eos_ids, num_eos, remaining, tokens, status, err);
  }
  cluster.sync();
}

// ---------------------------------------------------------------------------
// streaming kernel
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kSelThreads) select_stream_kernel(
    const T* __restrict__ logits, int64_t row_stride, int32_t batch, int32_t vocab, int32_t chunk,
    const int64_t* __restrict__ eos_ids, int32_t num_eos, int32_t* __restrict__ remaining,
    int64_t* __restrict__ tokens, uint8_t* __restrict__ status, int32_t* err) {
  constexpr int N = Vec<T>::N;
  extern __shared__ __align__(128) uint8_t ring[];  // [warp][slot][kSlotBytes]
  __shared__ __align__(8) uint64_t full[kSelWarps][kSlots];
  __shared__ __align__(8) uint64_t wkeys[kMaxRowsPerCluster][kSelWarps];   // this CTA's warps, per row
  __shared__ __align__(8) uint64_t ckeys[kMaxRowsPerCluster][kMaxCluster];  // CTA 0: every CTA, per row

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = static_cast<int>(cluster.block_rank());
  const int csize = static_cast<int>(cluster.num_blocks());
  const int ncl = static_cast<int>(gridDim.x) / csize;
  const int cl = static_cast<int>(blockIdx.x) / csize;
  // this cluster's rows: cl, cl + ncl, ...
  const int nrows = cl < batch ? (batch - 1 - cl) / ncl + 1 : 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int32_t lo = crank * chunk;
  const int32_t n = max(0, min(vocab, lo + chunk) - lo);
  const int32_t nvec = n / N;
  // this warp's part of the slice, in 16-byte vectors
  const int32_t per = (nvec + kSelWarps - 1) / kSelWarps;
  const int32_t w0 = min(nvec, warp * per), w1 = min(nvec, w0 + per);
  const int npc = (w1 - w0 + kSlotVecs - 1) / kSlotVecs;  // pieces per row
  const int total = npc * nrows;
  uint8_t* my_ring = ring + warp * (kSlots * kSlotBytes);

  // a warp with no part of a row leaves key 0 there
  for (int i = tid; i < nrows * kSelWarps; i += kSelThreads) wkeys[i / kSelWarps][i % kSelWarps] = 0ull;
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < kSlots; ++k) mbar_init(&full[warp][k], 1);
    fence_barrier_init();
  }
  __syncwarp();
  __syncthreads();
  // Announce this CTA to the cluster; the matching wait comes before the
  // first access to another CTA's shared memory, so nothing stalls here.
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  // The logits come from the stream predecessor.
  pdl_wait();

  const uint8_t* base = reinterpret_cast<const uint8_t*>(logits + lo);
  uint64_t policy = 0;
  if (lane == 0) policy = l2_policy_evict_first();
  // lane 0's cursor: the next piece to copy (sequence number, row, piece of the row)
  int pj = 0, pri = 0, pt = 0;
  auto issue_next = [&]() {
    const int64_t row = cl + static_cast<int64_t>(pri) * ncl;
    const int32_t v0 = w0 + pt * kSlotVecs;
    const uint32_t bytes = static_cast<uint32_t>(min(kSlotVecs, w1 - v0)) * 16u;
    const int slot = pj % kSlots;
    uint64_t* bar = &full[warp][slot];
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load(my_ring + slot * kSlotBytes, base + row * row_stride * static_cast<int64_t>(sizeof(T)) +
                  static_cast<int64_t>(v0) * 16, bytes, bar, policy);
    ++pj;
    if (++pt == npc) {
      pt = 0;
      ++pri;
    }
  };
  if (lane == 0)
    for (int k = 0; k < min(kSlots, total); ++k) issue_next();

  // Lane state for the current row: its best value so far and the piece
  // where it first reached it (-1: the lane owns no vector of the row).  A
  // lane's pieces arrive in increasing index order, so only a strictly larger
  // value (or a first NaN) replaces the record.
  float bv = -INFINITY;
  int bpiece = -1;
  int ri = 0, t = 0;  // row and piece of piece j
  for (int j = 0; j < total; ++j) {
    const int slot = j % kSlots;
    const bool got = __all_sync(0xFFFFFFFFu, mbar_wait(&full[warp][slot], static_cast<uint32_t>((j / kSlots) & 1)));
    if (!got) {
      if (lane == 0) flag_error(err, PSB_DEVERR_TIMEOUT);
      // Wait (bounded) for the other slots' copies, where issued.  Slot j's
      // own copy is the one that timed out and may still be in flight when
      // the CTA exits; the error flag tells the host that this launch's
      // results, and the shared memory it leaves, are not to be trusted.
      for (int q = j + 1; q < j + kSlots && q < total; ++q)
        (void)mbar_wait(&full[warp][q % kSlots], static_cast<uint32_t>((q / kSlots) & 1));
      break;
    }
    const int32_t v0 = w0 + t * kSlotVecs;
    const int nv = min(kSlotVecs, w1 - v0);
    const uint32_t sb = smem_u32(my_ring + slot * kSlotBytes);
    uint4 r[kVecPerLane];
    typename Vec<T>::Acc acc;
#pragma unroll
    for (int i = 0; i < kVecPerLane; ++i) {
      const int v = lane + 32 * i;
      if (v < nv) {
        r[i] = ld_shared_v4(sb + v * 16u);
        acc.add(r[i]);
      }
    }
    // every lane has its vectors in registers: the slot may be refilled
    __syncwarp();
    if (lane == 0 && pj < total) {  // pj == j + kSlots
      fence_proxy_async_smem();
      issue_next();
    }
    if (lane < nv) {  // the lane owns at least one vector of this piece
      const float pm = acc.result();
      if (bpiece < 0 || pm > bv || (pm != pm && bv == bv)) {
        bv = pm;
        bpiece = t;
      }
    }
    if (++t == npc) {  // this warp's last piece of the row: merge the lanes
      const uint32_t lk = bpiece >= 0 ? order_key(bv) : 0u;
      const uint32_t mk = __reduce_max_sync(0xFFFFFFFFu, lk);
      // the earliest piece in which a lane reached the row's maximum; a lane
      // that reached it only later holds smaller values in every earlier piece
      const uint32_t pmin =
          __reduce_min_sync(0xFFFFFFFFu, (bpiece >= 0 && lk == mk) ? static_cast<uint32_t>(bpiece) : 0x7FFFFFFFu);
      uint32_t f = 0x7FFFFFFFu;
      if (bpiece >= 0 && lk == mk && static_cast<uint32_t>(bpiece) == pmin) {
        // this lane's vectors of that piece, read again (a few lanes per row)
        const int32_t pv0 = w0 + static_cast<int32_t>(pmin) * kSlotVecs;
        const int pnv = min(kSlotVecs, w1 - pv0);
        const uint4* src = reinterpret_cast<const uint4*>(logits + (cl + static_cast<int64_t>(ri) * ncl) * row_stride +
                                                          lo) + pv0;
#pragma unroll
        for (int i = 0; i < kVecPerLane; ++i) {
          const int v = lane + 32 * i;
          if (f == 0x7FFFFFFFu && v < pnv) {
            const uint4 x = __ldg(src + v);
            if (same_value(Vec<T>::vmax(x), bv)) f = static_cast<uint32_t>(lo + (pv0 + v) * N + first_lane<T>(x, bv));
          }
        }
      }
      f = __reduce_min_sync(0xFFFFFFFFu, f);
      if (lane == 0) wkeys[ri][warp] = pack_key(mk, static_cast<int32_t>(f));
      bv = -INFINITY;
      bpiece = -1;
      t = 0;
      ++ri;
    }
  }
  // row results were written by whichever lane owned them
  __syncwarp();
  // the ragged end of each row (fewer than N elements, last slice only)
  if (tid == 0 && n > nvec * N) {
    for (int ri = 0; ri < nrows; ++ri) {
      const T* p = logits + (cl + static_cast<int64_t>(ri) * ncl) * row_stride;
      uint32_t bk = 0;
      int32_t bi = 0;
      for (int32_t i = lo + nvec * N; i < lo + n; ++i) {
        const uint32_t k = order_key(load_scalar(p + i));
        if (k > bk) {
          bk = k;
          bi = i;
        }
      }
      const uint64_t k = pack_key(bk, bi);
      if (k > wkeys[ri][0]) wkeys[ri][0] = k;  // warp 0's slot; warp 0's lanes are done with it
    }
  }
  pdl_launch_dependents();
  __syncthreads();
  // every CTA of the cluster is running: CTA 0's shared memory may be written
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  // this CTA's result for each row, stored into CTA 0's slot [row][rank]
  for (int ri = tid; ri < nrows; ri += kSelThreads) {
    uint64_t k = wkeys[ri][0];
#pragma unroll
    for (int w = 1; w < kSelWarps; ++w) k = wkeys[ri][w] > k ? wkeys[ri][w] : k;
    *cluster.map_shared_rank(&ckeys[ri][crank], 0) = k;
  }
  // every CTA's results have reached CTA 0
  cluster.sync();
  if (crank == 0)
    for (int ri = tid; ri < nrows; ri += kSelThreads) {
      uint64_t k = ckeys[ri][0];
      for (int r = 1; r < csize; ++r) k = ckeys[ri][r] > k ? ckeys[ri][r] : k;
      finish_row(cl + ri * ncl, k, eos_ids, num_eos, remaining, tokens, status, err);
    }
}

// ---------------------------------------------------------------------------
// register kernel
// ---------------------------------------------------------------------------

// Running best of one thread.  Elements arrive in increasing index order, so
// replacing only on a strictly larger value (or a first NaN) keeps the first
// occurrence.  `i` starts at the thread's first index: if nothing ever
// replaces it, every element it saw was -inf and the first one is the answer.
struct Best {
  float v;
  int32_t i;
  __device__ __forceinline__ bool beaten_by(float m) const { return m > v || (m != m && v == v); }
};

template <typename T, bool VEC>
__global__ void __launch_bounds__(kSelThreads) select_tokens_kernel(
    const T* __restrict__ logits, int64_t row_stride, int32_t vocab, int32_t chunk,
    const int64_t* __restrict__ eos_ids, int32_t num_eos, int32_t* __restrict__ remaining,
    int64_t* __restrict__ tokens, uint8_t* __restrict__ status, int32_t* err) {
  __shared__ uint64_t s_warp[kSelThreads / 32];
  __shared__ uint64_t s_cta;
  // The logits come from the stream predecessor.
  pdl_wait();

  cg::cluster_group cluster = cg::this_cluster();
  const int crank = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.y;
  const T* __restrict__ p = logits + static_cast<int64_t>(row) * row_stride;
  const int32_t lo = crank * chunk;
  const int32_t hi = min(vocab, lo + chunk);
  const int tid = threadIdx.x;

  Best best{-INFINITY, -1};
  if (lo < hi) {
    if constexpr (VEC) {
      constexpr int N = Vec<T>::N;
      const int32_t vec_hi = lo + ((hi - lo) / N) * N;
      best.i = lo + tid * N < vec_hi ? lo + tid * N : vec_hi + tid;
      constexpr int32_t kStride = kSelThreads * N;
      for (int32_t base = lo + tid * N; base < vec_hi; base += kSelUnroll * kStride) {
        uint4 r[kSelUnroll];
#pragma unroll
        for (int u = 0; u < kSelUnroll; ++u) {
          const int32_t i = base + u * kStride;
          if (i < vec_hi) r[u] = __ldcs(reinterpret_cast<const uint4*>(p + i));
        }
#pragma unroll
        for (int u = 0; u < kSelUnroll; ++u) {
          const int32_t i = base + u * kStride;
          if (i >= vec_hi) break;
          const float m = Vec<T>::vmax(r[u]);
          if (best.beaten_by(m)) {
            best.v = m;
            best.i = i + first_lane<T>(r[u], m);
          }
        }
      }
      for (int32_t i = vec_hi + tid; i < hi; i += kSelThreads) {
        const float x = load_scalar(p + i);
        if (best.beaten_by(x)) {
          best.v = x;
          best.i = i;
        }
      }
    } else {
      best.i = lo + tid;
      for (int32_t i = lo + tid; i < hi; i += kSelThreads) {
        const float x = load_scalar(p + i);
        if (best.beaten_by(x)) {
          best.v = x;
          best.i = i;
        }
      }
    }
  }
  pdl_launch_dependents();
  // Threads that own no element contribute key 0, below every real key.
  uint64_t key = (best.i >= 0 && best.i < hi) ? pack_key(order_key(best.v), best.i) : 0ull;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, key, off);
    key = o > key ? o : key;
  }
  if ((tid & 31) == 0) s_warp[tid >> 5] = key;
  __syncthreads();
  if (tid == 0) {
    uint64_t k = s_warp[0];
#pragma unroll
    for (int w = 1; w < kSelThreads / 32; ++w) k = s_warp[w] > k ? s_warp[w] : k;
    s_cta = k;
  }
  merge_and_finish(cluster, &s_cta, row, eos_ids, num_eos, remaining, tokens, status, err);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <typename... KArgs, typename... Args>
cudaError_t launch_cluster(void (*kernel)(KArgs...), int cluster, dim3 grid, size_t smem, cudaStream_t s,
                           Args&&... args) {
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  attrs[1].id = cudaLaunchAttributeClusterDimension;
  attrs[1].val.clusterDim.x = static_cast<unsigned>(cluster);
  attrs[1].val.clusterDim.y = 1;
  attrs[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kSelThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Slice of one CTA: ceil(vocab / cluster) rounded up to whole 16-byte vectors.
int32_t slice_elems(int32_t vocab, int cluster, int esz) {
  const int n = 16 / esz;
  const int32_t c = static_cast<int32_t>((static_cast<int64_t>(vocab) + cluster - 1) / cluster);
  return (c + n - 1) / n * n;
}

// Clusters of `cluster` CTAs of the streaming kernel that fit on the device at once.
template <typename T>
int resident_clusters(int cluster) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(dev, cluster);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  const void* kernel = reinterpret_cast<const void*>(select_stream_kernel<T>);
  int occ = 0;
  if (!kernel_occupancy(kernel, kSelThreads, kRingBytes, &occ) || occ < 1) return 0;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = static_cast<unsigned>(cluster);
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster));
  cfg.blockDim = dim3(kSelThreads);
  cfg.dynamicSmemBytes = kRingBytes;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n < 1) {
    discard_stale_error();
    const int sms = device_sm_count();
    n = std::max(1, sms * occ / cluster);
  }
  cache[key] = n;
  return n;
}

template <typename T>
int launch_select(const void* logits, int64_t row_stride, int32_t batch, int32_t vocab, int ctas_per_row,
                  bool aligned, const int64_t* eos, int32_t num_eos, int32_t* remaining, int64_t* tokens,
                  uint8_t* status, int32_t* err, cudaStream_t s) {
  const int esz = static_cast<int>(sizeof(T));
  int cluster = ctas_per_row > 0 ? ctas_per_row : (batch < kSmallBatch ? kAutoClusterSmall : kAutoCluster);
  if (ctas_per_row == 0)
    while (cluster > 1 && vocab / cluster < 2048) --cluster;
  const int32_t chunk = slice_elems(vocab, cluster, esz);
  const auto T_ = static_cast<const T*>(logits);
  cudaError_t e;
  if (aligned) {
    // one wave: every resident cluster takes an equal count of rows
    const int cap = resident_clusters<T>(cluster);
    if (cap < 1) return PSB_ERR_CUDA;
    int per = (batch + cap - 1) / cap;
    per = std::min(per, kMaxRowsPerCluster);
    const int ncl = (batch + per - 1) / per;
    if (static_cast<int64_t>(ncl) * cluster > INT_MAX) return PSB_ERR_UNSUPPORTED;
    discard_stale_error();
    e = launch_cluster(select_stream_kernel<T>, cluster, dim3(static_cast<unsigned>(ncl * cluster)), kRingBytes, s,
                       T_, row_stride, batch, vocab, chunk, eos, num_eos, remaining, tokens, status, err);
  } else {
    auto kernel = select_tokens_kernel<T, false>;
    discard_stale_error();
    if (!prefer_max_shared(reinterpret_cast<const void*>(kernel))) return PSB_ERR_CUDA;
    e = launch_cluster(kernel, cluster, dim3(static_cast<unsigned>(cluster), static_cast<unsigned>(batch)), 0, s, T_,
                       row_stride, vocab, chunk, eos, num_eos, remaining, tokens, status, err);
  }
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}

}  // namespace
}  // namespace psb

using namespace psb;

extern "C" int psb_select_tokens(const void* logits, int64_t row_stride, int32_t batch, int32_t vocab,
                                 int32_t dtype, const int64_t* eos_ids, int32_t num_eos, int32_t* remaining,
                                 int64_t* tokens, uint8_t* status, int32_t ctas_per_row, int32_t* error_flag,
                                 psb_stream_t stream) {
  if (batch < 0 || vocab <= 0 || num_eos < 0 || num_eos > kMaxEos || ctas_per_row < 0 ||
      ctas_per_row > kMaxCluster)
    return PSB_ERR_INVALID;
  if (dtype != PSB_F32 && dtype != PSB_F16 && dtype != PSB_BF16) return PSB_ERR_INVALID;
  if (batch == 0) return PSB_OK;
  if (batch > 65535 || vocab > (1 << 30)) return PSB_ERR_UNSUPPORTED;
  if (!logits || !remaining || !tokens || !status || (num_eos > 0 && !eos_ids)) return PSB_ERR_INVALID;
  if (batch > 1 && row_stride < vocab) return PSB_ERR_INVALID;
  const int esz = elem_bytes(dtype);
  const bool aligned = reinterpret_cast<uintptr_t>(logits) % 16 == 0 && (row_stride * esz) % 16 == 0;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PSB_F32)
    return launch_select<float>(logits, row_stride, batch, vocab, ctas_per_row, aligned, eos_ids, num_eos,
                                remaining, tokens, status, error_flag, s);
  if (dtype == PSB_F16)
    return launch_select<__half>(logits, row_stride, batch, vocab, ctas_per_row, aligned, eos_ids, num_eos,
                                 remaining, tokens, status, error_flag, s);
  return launch_select<__nv_bfloat16>(logits, row_stride, batch, vocab, ctas_per_row, aligned, eos_ids, num_eos,
                                      remaining, tokens, status, error_flag, s);
}
