// Packed ragged causal prefill on the 5th-generation tensor cores (sm_100a).
//
// Replaces the reference's one-request-at-a-time prefill attention
// (pagedserve/attention/qwen_paged_attention.py:121-128 calling
// pagedserve/attention/paged_attention.py:94-145) for bf16/f16, head_dim 64:
// q [T, Hq, 64], k/v [T, Hkv, 64], sequence i = rows cu[i] .. cu[i+1], causal
// within each sequence, q head h reads kv head h / (Hq / Hkv).
//
// Work: a tile is 128 query rows of one q head; a tile of query block i
// streams 2 (i + 1) key tiles of 64 keys.  Tiles are numbered heaviest first
// (a stable counting sort of the sequences by query blocks, built by every
// CTA in shared memory), the q heads of a tile adjacent so they share K/V
// through L2.  A persistent grid of two CTAs per SM takes them in snake order.
//
// A CTA is six warps, 96 KB of shared memory and 256 TMEM columns.  Warps 0-3
// (thread r = TMEM lane r = query row r of the tile) do the softmax; one lane
// of warp 4 issues the Q loads and S = Q K^T, one lane of warp 5 the K/V
// loads and O += P V.  They meet only on mbarriers, so the tensor core works
// while the softmax runs.  A global step counter across the CTA's tiles
// drives the 4-stage K/V ring (128-byte swizzle, each stage requested again
// as soon as P.V of its step is done), the two TMEM S buffers and the
// barrier phases; Q is double-buffered per tile.  Per key tile (step):
//   producer: S = Q K^T (four tcgen05.mma, M 128, N 64, K 16; fp32 into one of
//   two TMEM S buffers) one step ahead of the softmax, once P.V of the step
//   that last used the buffer is done;
//   softmax: thread r loads its row of S, masks keys past its own position or
//   past the sequence and stores P = exp2(S - m) rounded to the input type
//   (as the reference rounds the probabilities before P.V,
//   paged_attention.py:133-137) over the first half of the same S buffer in
//   its TMEM lane, two keys per column.  m is a lazily updated row max: only
//   when a row's max grows by more than 2^8 is the O accumulated so far in
//   TMEM rescaled (so P stays below 256 and most steps touch no O at all);
//   producer: O += P V (four tcgen05.mma with P read from TMEM, N 64, V as an
//   MN-major operand) into the tile's O buffer; the first step of a tile
//   overwrites it.
// Consecutive tiles alternate between two TMEM O buffers, and a tile's output
// is read and written by the softmax warps after the next tile's first step,
// so no warp waits for a tile's last P.V at the tile boundary.  The K/V request
// cursor walks the CTA's whole tile list, kKvAhead steps ahead of P.V.
// Every mbarrier wait is bounded and each phase is waited for before the
// barrier can move two phases on; on a timeout a CTA records
// PSB_DEVERR_TIMEOUT, lets its copies and MMAs in flight land (bounded), frees
// TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "host_util.h"
#include "varlen_prefill.h"

namespace psb {
namespace {

constexpr int kSoftmaxThreads = 128;  // warps 0-3: warp w <-> TMEM lanes and tile rows 32 w .. 32 w + 31
constexpr int kTcThreads = kSoftmaxThreads + 64;  // warp 4: Q loads and Q K^T; warp 5: K/V loads and P V
constexpr int kBM = 128;         // query rows per tile
constexpr int kBN = 64;          // keys per step
constexpr int kDim = 64;
constexpr uint32_t kTile = kBM * kDim * 2;    // bytes of one Q tile (16 KB)
constexpr uint32_t kKvTile = kBN * kDim * 2;  // bytes of one K or V tile (8 KB)
constexpr int kKvStages = 4;                  // K/V ring depth
constexpr int kKvAhead = kKvStages;           // K/V of step g + kKvAhead is requested once P.V of step g is done
// TMEM columns: S buffers [0, 64) and [64, 128) (P of a step overwrites the
// first 32 columns of its S buffer, two 16-bit values per column); O buffers
// [128, 192) and [192, 256), one per tile in turn
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kSCol = 0, kOCol = 128;
constexpr float kRescaleLog2 = 8.f;  // rescale O when a row max grows by more than 2^8
// dynamic shared memory (1024-byte aligned): Q0 | Q1 | K ring | V ring | barriers | tile tables
constexpr uint32_t kOffQ = 0, kOffK = 2 * kTile, kOffV = 2 * kTile + kKvStages * kKvTile;
constexpr uint32_t kSmemTiles = 2 * kTile + 2 * kKvStages * kKvTile;
constexpr uint32_t kSmemBars = 128;
// output staging: per softmax warp, 32 rows x 64 bytes (half a row of the tile
// at a time), so each global store instruction writes whole row segments
constexpr uint32_t kOutStageWarp = 32 * 64;
constexpr uint32_t kOffOut = kSmemTiles + kSmemBars;
constexpr uint32_t kSmemOut = 4 * kOutStageWarp;
constexpr int kMaxLevels = 1024;    // query blocks per sequence (128 K tokens)
constexpr int kMaxTcSeqs = 2048;    // sequences whose order fits the shared tile table

// Length of sequence s; 0 unless 0 <= cu[s] <= cu[s+1] <= total (a malformed
// batch is reported by the caller's check and must not be read out of bounds).
__device__ __forceinline__ int seq_len(const PrefillParams& p, int s) {
  const int a = p.cu[s], b = p.cu[s + 1];
  if (a < 0 || b < a || b > p.total) return 0;
  return min(b - a, p.max_seqlen);
}

struct TileInfo {
  int q0, len, qblk, head, kvh, n_kv;
  int seq, start, ctx;  // query row i sits at position start + i of ctx keys
};

constexpr int kPoolBlock = 16;                      // paged: rows per pool block
constexpr uint32_t kPoolTile = kPoolBlock * kDim * 2;  // bytes of one (block, kv head) tile

// PAGED (psb_paged_prefill): K/V come from the pools through the block table,
// four pool tiles per 64-key step, and a sequence's query rows are the last
// positions of its context; otherwise from the packed k/v rows of the batch.

// Packed fp32 pairs (sm_100 f32x2 instructions): the exponent arguments and
// the row sum take one instruction per two scores, and the row max one
// three-input max per two scores (2 % off the 16K-token pack).
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 up2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <typename T, bool PAGED>
__global__ void __launch_bounds__(kTcThreads, 2)
    prefill_tc_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar_q = reinterpret_cast<uint64_t*>(smem + kSmemTiles);  // [2]
  uint64_t* bar_kv = bar_q + 2;                                      // [kKvStages]
  uint64_t* bar_s = bar_q + 2 + kKvStages;                           // [2]
  uint64_t* bar_pv = bar_s + 2;      // [2] P.V of step g (which read P from S buffer g & 1) done
  uint64_t* bar_p = bar_pv + 2;      // [2] softmax step done: P buffer g & 1 written
  uint64_t* bar_qfree = bar_p + 2;   // a tile's Q K^T done
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar_qfree + 1);
  static_assert(13 * sizeof(uint64_t) + sizeof(uint32_t) <= kSmemBars, "barriers fit their area");
  const int max_level = (p.max_seqlen + kBM - 1) / kBM;
  int32_t* s_lstart = reinterpret_cast<int32_t*>(smem + kOffOut + kSmemOut);  // [max_level + 1]
  int32_t* s_cnt = s_lstart + (max_level + 1);   // [max_level + 1] sequences with more than i blocks
  int32_t* s_fill = s_cnt + (max_level + 1);     // [max_level + 1] placement cursors
  int32_t* s_sorted = s_fill + (max_level + 1);  // [num_seqs] sequences by query blocks, descending, stable
  // [max_cta_tiles][2] this CTA's tiles: {seq, qblk, head, q0}, {len, ctx, n_kv, 0}
  int4* s_tiles = reinterpret_cast<int4*>(
      (reinterpret_cast<uintptr_t>(s_sorted + p.num_seqs) + 15) & ~uintptr_t(15));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hq = p.hq, group = p.hq / p.hkv;
  // cu_seqlens, q, k and v may come from the stream predecessor
  pdl_wait();

  // ---- tile table: sequences sorted by query blocks (stable), level starts
  for (int i = tid; i <= max_level; i += kTcThreads) s_cnt[i] = 0;
  __syncthreads();
  for (int s = tid; s < p.num_seqs; s += kTcThreads) {
    const int nb = (seq_len(p, s) + kBM - 1) / kBM;
    if (nb > 0) atomicAdd(&s_cnt[nb - 1], 1);  // histogram of top levels
  }
  __syncthreads();
  if (tid == 0) {
    // c_i = sequences with more than i blocks (suffix sums); level i holds
    // tiles [lstart_i, lstart_i + c_i), levels numbered from the top
    int run = 0, start = 0;
    for (int i = max_level - 1; i >= 0; --i) {
      run += s_cnt[i];
      s_cnt[i] = run;
      s_lstart[i] = start;
      start += run;
    }
    s_cnt[max_level] = 0;
    s_lstart[max_level] = start;  // tiles in all
    for (int i = 0; i <= max_level; ++i) s_fill[i] = i < max_level ? s_cnt[i + 1] : 0;  // first slot of key i + 1
  }
  __syncthreads();
  if (warp == 0) {  // stable placement: sequences with nb blocks go after those with more
    for (int s0 = 0; s0 < p.num_seqs; s0 += 32) {
      const int s = s0 + lane;
      const int nb = s < p.num_seqs ? (seq_len(p, s) + kBM - 1) / kBM : 0;
      const uint32_t peers = __match_any_sync(0xffffffffu, nb);
      if (nb > 0) {
        const int pos = s_fill[nb - 1] + __popc(peers & ((1u << lane) - 1u));
        s_sorted[pos] = s;
      }
      __syncwarp();
      if (nb > 0 && lane == __ffs(peers) - 1) s_fill[nb - 1] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  // tiles are dealt to the CTAs in snake order (round r left to right when
  // even, right to left when odd), which evens out the heaviest-first list
  const int total_tiles = s_lstart[max_level] * hq;
  const int G = gridDim.x, c = blockIdx.x;
  const int rounds = total_tiles / G, rem = total_tiles - rounds * G;
  const int my_tiles = rounds + (((rounds & 1) ? G - 1 - c : c) < rem ? 1 : 0);
  if (my_tiles == 0) return;
  if (my_tiles > p.max_cta_tiles) {  // the launch sized the tile list too small: nothing is computed
    if (tid == 0) flag_error(p.err, PSB_DEVERR_WORKSPACE);
    return;
  }
  // k-th tile of this CTA, from the sorted sequences and cu_seqlens
  auto compute_tile = [&](int k) -> TileInfo {
    const int t = k * G + ((k & 1) ? G - 1 - c : c);
    const int tt = t / hq;
    int lo = 0, hi = max_level - 1;  // the smallest level i with lstart_i <= T
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (s_lstart[mid] <= tt) hi = mid; else lo = mid + 1;
    }
    TileInfo ti;
    const int seq = s_sorted[tt - s_lstart[lo]];
    ti.qblk = lo;
    ti.head = t - tt * hq;
    ti.kvh = ti.head / group;
    ti.q0 = p.cu[seq];
    ti.len = seq_len(p, seq);
    ti.seq = seq;
    ti.ctx = ti.len;
    if constexpr (PAGED) {
      int c = p.ctx[seq];  // at least the query rows, at most max_context (else flagged, clamped)
      if (c < ti.len || c > p.max_context) {
        flag_error(p.err, PSB_DEVERR_CONTEXT);
        c = c < ti.len ? ti.len : p.max_context;
      }
      ti.ctx = c;
    }
    ti.start = ti.ctx - ti.len;
    ti.n_kv = (ti.start + min(ti.len, (lo + 1) * kBM) + kBN - 1) / kBN;  // keys [0, start + last row + 1)
    return ti;
  };
  // Every tile of this CTA is worked out once, here, by all threads at once:
  // a tile's cu_seqlens (and context) loads would otherwise sit on each
  // role's critical path at every tile change.
  for (int k = tid; k < my_tiles; k += kTcThreads) {
    const TileInfo ti = compute_tile(k);
    s_tiles[2 * k] = make_int4(ti.seq, ti.qblk, ti.head, ti.q0);
    s_tiles[2 * k + 1] = make_int4(ti.len, ti.ctx, ti.n_kv, 0);
  }
  __syncthreads();
  auto tile_of = [&](int k) -> TileInfo {
    const int4 a = s_tiles[2 * k], b = s_tiles[2 * k + 1];
    TileInfo ti;
    ti.seq = a.x;
    ti.qblk = a.y;
    ti.head = a.z;
    ti.q0 = a.w;
    ti.kvh = ti.head / group;
    ti.len = b.x;
    ti.ctx = b.y;
    ti.n_kv = b.z;
    ti.start = ti.ctx - ti.len;
    return ti;
  };
  const uint32_t s_base = smem_u32(smem);

  // ---- set-up: barriers, TMEM ------------------------------------------------
  if (tid == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_q + 1, 1);
    for (int i = 0; i < kKvStages; ++i) mbar_init(bar_kv + i, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_s + 1, 1);
    mbar_init(bar_pv, 1);
    mbar_init(bar_pv + 1, 1);
    mbar_init(bar_p, kSoftmaxThreads);
    mbar_init(bar_p + 1, kSoftmaxThreads);
    mbar_init(bar_qfree, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  bool fail = false;

  if (warp >= 4) {
    if (lane == 0) {
      const uint32_t fmt = Elem<T>::code == PSB_BF16 ? 1u : 0u;
      if (warp == 4) {
        // ---- Q loads and S = Q K^T, one step ahead of the softmax -----------
        const uint32_t idesc_s = umma_idesc_f16(fmt, kBM, kBN, 0, 0);
        // descriptors of Q buffer 0 and stage 0; a k-step of 16 elements
        // advances the address field (bytes >> 4) by 2, a Q buffer by
        // kTile >> 4, a K/V stage by kKvTile >> 4
        const uint64_t dq = umma_desc_sw128(s_base + kOffQ, 1024, 16);
        const uint64_t dk = umma_desc_sw128(s_base + kOffK, 1024, 16);
        auto load_q = [&](int k) {
          const TileInfo ti = tile_of(k);
          mbar_arrive_expect_tx(bar_q + (k & 1), kTile);
          tma_load_3d(smem + kOffQ + (k & 1) * kTile, &tm_q, 0, ti.head, ti.q0 + ti.qblk * kBM, bar_q + (k & 1));
        };
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        load_q(0);
        if (my_tiles > 1) load_q(1);
        int q_req = min(my_tiles, 2), q_seen = 0, qf_seen = 0, g = 0;
        for (int k = 0; k < my_tiles && !fail; ++k) {
          if (k > 0 && k + 1 < my_tiles) {
            // Q of tile k + 1 goes into the buffer of tile k - 1, whose Q K^T is done
            if (!mbar_wait(bar_qfree, (k - 1) & 1)) {
              fail = true;
              break;
            }
            ++qf_seen;
            load_q(k + 1);
            ++q_req;
          }
          if (!mbar_wait(bar_q + (k & 1), (k >> 1) & 1)) {
            fail = true;
            break;
          }
          ++q_seen;
          const int n_kv = tile_of(k).n_kv;
          const uint64_t dqs = dq + static_cast<uint64_t>((k & 1) * (kTile >> 4));
          for (int j = 0; j < n_kv; ++j, ++g) {
            // S buffer g & 1 held S and then P of step g - 2: free once that
            // step's P.V is done (the barrier's next phase needs this step's S,
            // so the parity cannot alias)
            if (g >= 2 && !mbar_wait(bar_pv + (g & 1), ((g - 2) >> 1) & 1)) {
              fail = true;
              break;
            }
            if (!mbar_wait(bar_kv + g % kKvStages, (g / kKvStages) & 1)) {
              fail = true;
              break;
            }
            tc_fence_after();
            const uint64_t dks = dk + static_cast<uint64_t>((g % kKvStages) * (kKvTile >> 4));
#pragma unroll
            for (int kk = 0; kk < kDim / 16; ++kk)
              umma_f16_ss(tmem + kSCol + (g & 1) * kBN, dqs + 2 * kk, dks + 2 * kk, idesc_s, kk > 0);
            umma_commit(bar_s + (g & 1));
          }
          if (fail) break;
          umma_commit(bar_qfree);  // lands once every Q K^T of tile k is done
        }
        if (fail) {
          flag_error(p.err, PSB_DEVERR_TIMEOUT);
          for (int t = q_seen; t < q_req; ++t) (void)mbar_wait(bar_q + (t & 1), (t >> 1) & 1);
          (void)qf_seen;
        }
      } else {
        // ---- K/V loads and O += P V ------------------------------------------
        const uint32_t idesc_o = umma_idesc_f16(fmt, kBM, kDim, 0, 1);
        // V descriptor of stage 0; a stage advances the address field by
        // kKvTile >> 4, a k-step of 16 keys by 2048 >> 4
        const uint64_t dv = umma_desc_sw128(s_base + kOffV, 1024, 8192);
        // The request cursor walks this CTA's whole tile list (in shared
        // memory), so requests stay kKvAhead steps ahead across tile ends.
        int ck = 0, cj = 0, rg = 0;  // tile, step and global step of the next request
        TileInfo cti = tile_of(0);
        // paged: block ids of the request the cursor points at, loaded while
        // the step before it runs (pf_g: its global step, -1 for none)
        static_assert(kBN / kPoolBlock == 4, "four pool blocks per key step");
        int4 pf_ids = make_int4(-1, -1, -1, -1);  // in registers: no local memory on the issue path
        int pf_g = -1;
        auto load_ids = [&](int seq, int ctx, int j) -> int4 {
          const int nblk = (ctx + kPoolBlock - 1) / kPoolBlock;
          const int32_t* row = p.tables + static_cast<int64_t>(seq) * p.table_stride + 4 * j;
          const int n = nblk - 4 * j;
          return make_int4(__ldg(row), n > 1 ? __ldg(row + 1) : -1, n > 2 ? __ldg(row + 2) : -1,
                           n > 3 ? __ldg(row + 3) : -1);
        };
        auto prefetch_ids = [&]() {
          if constexpr (PAGED) {
            if (ck >= my_tiles || pf_g == rg) return;
            pf_ids = load_ids(cti.seq, cti.ctx, cj);
            pf_g = rg;
          }
        };
        auto request_kv = [&](int limit_g) {
          while (rg <= limit_g && ck < my_tiles) {
            const int st = rg % kKvStages;
            if constexpr (PAGED) {
              // the step's four pool blocks; blocks past the context are not
              // loaded (the softmax zeroes their V rows), bad ids are flagged
              const int nblk = (cti.ctx + kPoolBlock - 1) / kPoolBlock;
              const int4 id4 = pf_g == rg ? pf_ids : load_ids(cti.seq, cti.ctx, cj);
              int32_t ids[kBN / kPoolBlock] = {id4.x, id4.y, id4.z, id4.w};
#pragma unroll
              for (int b = 0; b < kBN / kPoolBlock; ++b) {
                const int idx = cj * (kBN / kPoolBlock) + b;
                if (idx < nblk && (ids[b] < 0 || ids[b] >= p.num_blocks)) {
                  flag_error(p.err, PSB_DEVERR_BLOCK_RANGE);
                  ids[b] = -1;
                }
              }
              uint32_t bytes = 0;
#pragma unroll
              for (int b = 0; b < kBN / kPoolBlock; ++b) bytes += ids[b] >= 0 ? 2 * kPoolTile : 0;
              mbar_arrive_expect_tx(bar_kv + st, bytes);
#pragma unroll
              for (int b = 0; b < kBN / kPoolBlock; ++b) {
                if (ids[b] < 0) continue;
                const int32_t tile = static_cast<int32_t>((static_cast<int64_t>(p.layer) * p.num_blocks + ids[b]) *
                                                          p.hkv + cti.kvh);
                tma_load_3d(smem + kOffK + st * kKvTile + b * kPoolTile, &tm_k, 0, 0, tile, bar_kv + st);
                tma_load_3d(smem + kOffV + st * kKvTile + b * kPoolTile, &tm_v, 0, 0, tile, bar_kv + st);
              }
            } else {
              mbar_arrive_expect_tx(bar_kv + st, 2 * kKvTile);
              tma_load_3d(smem + kOffK + st * kKvTile, &tm_k, 0, cti.kvh, cti.q0 + cj * kBN, bar_kv + st);
              tma_load_3d(smem + kOffV + st * kKvTile, &tm_v, 0, cti.kvh, cti.q0 + cj * kBN, bar_kv + st);
            }
            ++rg;
            if (++cj >= cti.n_kv) {
              cj = 0;
              if (++ck < my_tiles) cti = tile_of(ck);
            }
          }
        };
        request_kv(kKvAhead - 1);
        int pv_issued = 0, pv_seen = 0, g = 0;
        for (int k = 0; k < my_tiles && !fail; ++k) {
          const int n_kv = tile_of(k).n_kv;
          const uint32_t obuf = tmem + kOCol + (k & 1) * kDim;  // O buffers alternate between tiles
          for (int j = 0; j < n_kv && !fail; ++j, ++g) {
            prefetch_ids();  // the next request's block ids land while this step runs
            // softmax step g done: P written into S buffer g & 1 (the barrier's
            // next phase, step g + 2, needs P.V of this step first, so the
            // parity cannot alias)
            if (!mbar_wait(bar_p + (g & 1), (g >> 1) & 1)) {
              fail = true;
              break;
            }
            tc_fence_after();
            const uint64_t dvs = dv + static_cast<uint64_t>((g % kKvStages) * (kKvTile >> 4));
            const uint32_t pcol = tmem + kSCol + (g & 1) * kBN;
#pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk)
              umma_f16_ts(obuf, pcol + 8 * kk, dvs + 128 * kk, idesc_o, j > 0 || kk > 0);
            umma_commit(bar_pv + (g & 1));
            ++pv_issued;
            // the previous step's P.V (done in order before this one) frees its
            // stage for step g - 1 + kKvAhead
            if (g >= 1) {
              if (!mbar_wait(bar_pv + ((g - 1) & 1), ((g - 1) >> 1) & 1)) {
                fail = true;
                break;
              }
              ++pv_seen;
              request_kv(g - 1 + kKvAhead);
            }
          }
        }
        if (fail) {
          flag_error(p.err, PSB_DEVERR_TIMEOUT);
          // let copies and MMAs still in flight land before shared memory and TMEM are released
          for (int t = pv_seen; t < pv_issued; ++t) (void)mbar_wait(bar_pv + (t & 1), (t >> 1) & 1);
          for (int t = 0; t < kKvStages && t < rg; ++t) {
            const int last = rg - 1 - ((rg - 1 - t) % kKvStages);  // the newest request of stage t
            (void)mbar_wait(bar_kv + t, (last / kKvStages) & 1);
          }
        }
      }
    }
  } else {
    // ---- softmax warps ------------------------------------------------------
    const int row = warp * 32 + lane;  // tile row = TMEM lane
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float sc = p.scale_log2;
    // output rows 16-byte aligned: whole-row vector stores
    const bool out16 = reinterpret_cast<uintptr_t>(p.out) % 16 == 0 && p.ost % 8 == 0 && p.osh % 8 == 0;
    // A tile's output is written after the next tile's first step (or at the
    // end): by then its last P.V is normally done, so the softmax does not
    // wait for it, and the tensor core has the next tile's work meanwhile.
    // The next tile accumulates into the other O buffer; the tile after that
    // overwrites this one only after P of its first step, which this thread
    // writes after the output below.
    int pend_k = -1;   // the tile whose output is pending (-1: none)
    float pend_l = 0.f;  // its row sum
    // the output of tile pk, whose last step was global step pg
    auto write_pending = [&](int pk, int pg) -> bool {
      if (!mbar_wait(bar_pv + (pg & 1), (pg >> 1) & 1)) return false;
      tc_fence_after();
      const uint32_t t_po = t_lane + kOCol + (pk & 1) * kDim;
      const TileInfo pt = tile_of(pk);
      const int prow = pt.qblk * kBM + row;
      const float inv = pend_l > 0.f ? 1.f / pend_l : 0.f;
      const int64_t tok0 = static_cast<int64_t>(pt.q0) + pt.qblk * kBM + warp * 32;  // token of warp row 0
      T* const out_h = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(pt.head) * p.osh;
      uint8_t* stg = smem + kOffOut + warp * kOutStageWarp;
      const int rl = lane >> 2, cl = lane & 3;
      // half a row (32 columns) at a time
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t ot[32];
        tmem_ld32(t_po + 32 * h, ot);
        tmem_wait_ld();
        uint32_t ob[16];  // the half row rounded to T, two values per word
#pragma unroll
        for (int d = 0; d < 32; d += 2)
          ob[d / 2] = pack2<T>(__uint_as_float(ot[d]) * inv, __uint_as_float(ot[d + 1]) * inv);
        if (out16) {
          // through this warp's staging area: lane r writes row r's four
          // 16-byte chunks (chunk c at slot c ^ ((r >> 1) & 3): no bank
          // conflicts), then lanes 4 r .. 4 r + 3 store the chunks of row
          // 8 i + r, so a quarter-warp writes two whole 64-byte segments
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(stg + lane * 64 + ((c ^ ((lane >> 1) & 3)) * 16)) =
                make_uint4(ob[4 * c], ob[4 * c + 1], ob[4 * c + 2], ob[4 * c + 3]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = 8 * i + rl;
            const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 64 + ((cl ^ ((rr >> 1) & 3)) * 16));
            if (pt.qblk * kBM + warp * 32 + rr < pt.len && tok0 + rr < p.total)
              *reinterpret_cast<uint4*>(out_h + (tok0 + rr) * p.ost + 32 * h + 8 * cl) = v;
          }
          __syncwarp();
        } else if (prow < pt.len && pt.q0 + prow < p.total) {
          T* op = out_h + static_cast<int64_t>(pt.q0 + prow) * p.ost + 32 * h;
#pragma unroll
          for (int d = 0; d < 32; d += 2) *reinterpret_cast<uint32_t*>(op + d) = ob[d / 2];
        }
      }
      tc_fence_before();
      pend_k = -1;
      return true;
    };
    int g = 0;
    for (int k = 0; k < my_tiles && !fail; ++k) {
      const TileInfo ti = tile_of(k);
      const int qrow = ti.qblk * kBM + row;  // position in the sequence
      const uint32_t t_o = t_lane + kOCol + (k & 1) * kDim;  // this tile's O buffer, this warp's lanes
      float ms = -INFINITY, l_run = 0.f;     // row max used for the exponents (scaled by sc), row sum
      // step j of this tile (global step g); false when a wait ran out
      auto step = [&](int j) -> bool {
        if (!mbar_wait(bar_s + (g & 1), (g >> 1) & 1)) return false;
        tc_fence_after();
        uint32_t sr[kBN];
        tmem_ld32(t_lane + kSCol + (g & 1) * kBN, sr);
        tmem_ld32(t_lane + kSCol + (g & 1) * kBN + 32, sr + 32);
        tmem_wait_ld();
        if (PAGED && j == ti.n_kv - 1 && row < kBN && j * kBN + row >= ti.ctx) {
          // V rows past the context (stale or never loaded) must not reach
          // P.V, where 0 * NaN would be NaN: zero them before this thread's
          // arrival lets P.V read the stage (the Q.K^T just read, and it
          // followed the stage's copies)
          const uint32_t vrow = s_base + kOffV + (g % kKvStages) * kKvTile + row * 128;
#pragma unroll
          for (int c = 0; c < 128; c += 16) st_shared_zero16(vrow + c);
          fence_proxy_async_smem();  // visible to the tensor core
        }
        // keys past this row's position or past the context only occur in the last steps
        const int lim = min(ti.start + qrow, ti.ctx - 1) - j * kBN;  // last valid key column
        if (lim < kBN - 1) {
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (c > lim) sr[c] = __float_as_uint(-INFINITY);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int c = 0; c < kBN; c += 4) {
          mx0 = fmax3(mx0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
          mx1 = fmax3(mx1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
        }
        const float mx = fmaxf(mx0, mx1);
        // lazy max: move it (and rescale O and the sum) only when the row max
        // grew by more than 2^kRescaleLog2; the warp's TMEM access is collective
        const float mxs = mx * sc;
        const bool grow = mxs > ms + kRescaleLog2;
        if (__any_sync(0xffffffffu, grow)) {
          const float ms_new = grow ? mxs : ms;
          const float alpha = ms == -INFINITY ? 0.f : ex2_approx(ms - ms_new);  // 1 where the max stays
          if (j > 0) {  // O holds P.V of the earlier steps once the last of them is done
            if (!mbar_wait(bar_pv + ((g - 1) & 1), ((g - 1) >> 1) & 1)) return false;
            tc_fence_after();
            uint32_t ot[kDim];
            tmem_ld32(t_o, ot);
            tmem_ld32(t_o + 32, ot + 32);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < kDim; ++d) ot[d] = __float_as_uint(__uint_as_float(ot[d]) * alpha);
            tmem_st32(t_o, ot);
            tmem_st32(t_o + 32, ot + 32);
            tmem_wait_st();
          }
          l_run *= alpha;
          ms = ms_new;
        }
        const float mu = ms == -INFINITY ? 0.f : ms;  // rows with nothing valid yet stay zero
        uint32_t pk[kBN / 2];
        const uint64_t sc2 = pk2(sc, sc), nmu2 = pk2(-mu, -mu);
        uint64_t rs2 = pk2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < kBN; c += 2) {
          const float2 a = up2(ffma2(pk2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2, nmu2));
          const float x0 = ex2_approx(a.x);
          const float x1 = ex2_approx(a.y);
          rs2 = fadd2(rs2, pk2(x0, x1));
          pk[c / 2] = pack2<T>(x0, x1);
        }
        const float2 rsp = up2(rs2);
        const float rs = rsp.x + rsp.y;
        l_run += rs;
        // P over the first half of this step's S buffer (this lane's S is in
        // registers; the buffer takes S of step g + 2 only after P.V of this step)
        tmem_st32(t_lane + kSCol + (g & 1) * kBN, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p + (g & 1));
        return true;
      };
      // The first step, then the previous tile's output (outside the step
      // loop, whose registers it would otherwise crowd), then the rest.
      if (!step(0)) {
        fail = true;
        break;
      }
      if (pend_k >= 0 && !write_pending(pend_k, g - 1)) {
        fail = true;
        break;
      }
      ++g;
      for (int j = 1; j < ti.n_kv; ++j, ++g) {
        if (!step(j)) {
          fail = true;
          break;
        }
      }
      if (fail) break;
      pend_k = k;
      pend_l = l_run;
    }
    if (!fail && pend_k >= 0 && !write_pending(pend_k, g - 1)) fail = true;
    if (fail && lane == 0) flag_error(p.err, PSB_DEVERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

size_t tc_smem_bytes(int max_level, int num_seqs, int max_cta_tiles) {
  return 1024 + kSmemTiles + kSmemBars + kSmemOut +
         sizeof(int32_t) * (3 * (static_cast<size_t>(max_level) + 1) + num_seqs) +
         16 + 2 * sizeof(int4) * static_cast<size_t>(max_cta_tiles);
}

// An upper bound of the tiles: sum over sequences of ceil(len / 128), times the heads.
int64_t tc_tiles_bound(const PrefillParams& p) { return (static_cast<int64_t>(p.total) / kBM + p.num_seqs) * p.hq; }

// Tiles per CTA that any persistent grid of at least one CTA per SM (or one
// CTA per tile, when there are fewer tiles) can deal to one CTA.
int tc_max_cta_tiles(const PrefillParams& p, int sms) {
  const int64_t tiles = tc_tiles_bound(p);
  return static_cast<int>(std::min<int64_t>(tiles, (tiles + sms - 1) / std::max(sms, 1) + 1));
}

}  // namespace

bool prefill_tc_supported(const PrefillParams& p, int dtype) {
  if (!(dtype == PSB_BF16 || dtype == PSB_F16) || p.head_dim != kDim) return false;
  if (p.paged && p.block_size != kPoolBlock) return false;
  auto al16 = [](const void* x) { return reinterpret_cast<uintptr_t>(x) % 16 == 0; };
  // TMA: 16-byte aligned bases and strides (the pools are contiguous); 4-byte output pairs
  const bool kv_strides = p.paged || (p.kst % 8 == 0 && p.ksh % 8 == 0 && p.vst % 8 == 0 && p.vsh % 8 == 0 &&
                                      p.kst > 0 && p.vst > 0);
  const bool strides = p.qst % 8 == 0 && p.qsh % 8 == 0 && kv_strides && p.ost % 2 == 0 && p.osh % 2 == 0 &&
                       p.qst > 0;
  const int max_level = (p.max_seqlen + kBM - 1) / kBM;
  const int sms = device_sm_count();
  if (sms <= 0) return false;
  return strides && al16(p.q) && al16(p.k) && al16(p.v) && reinterpret_cast<uintptr_t>(p.out) % 4 == 0 &&
         max_level <= kMaxLevels && p.num_seqs <= kMaxTcSeqs &&
         tc_smem_bytes(max_level, p.num_seqs, tc_max_cta_tiles(p, sms)) <= 227 * 1024;
}

int prefill_tc_launch(const PrefillParams& p_in, int dtype, cudaStream_t s) {
  PrefillParams p = p_in;
  const CUtensorMapDataType dt = dtype == PSB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  if (!encode_rows_map(&tq, p.q, p.total, p.hq, kDim, p.qst, p.qsh, kBM, dt)) return PSB_ERR_CUDA;
  if (p.paged) {
    // the pools as (layer, block, kv head) tiles of 16 x 64
    const int64_t tiles = static_cast<int64_t>(p.num_layers_total) * p.num_blocks * p.hkv;
    if (!encode_pool_map(&tk, p.k, tiles, kPoolBlock, kDim, dt) || !encode_pool_map(&tv, p.v, tiles, kPoolBlock, kDim, dt))
      return PSB_ERR_CUDA;
  } else if (!encode_rows_map(&tk, p.k, p.total, p.hkv, kDim, p.kst, p.ksh, kBN, dt) ||
             !encode_rows_map(&tv, p.v, p.total, p.hkv, kDim, p.vst, p.vsh, kBN, dt)) {
    return PSB_ERR_CUDA;
  }
  const int max_level = (p.max_seqlen + kBM - 1) / kBM;
  const int64_t tiles = tc_tiles_bound(p);
  if (tiles == 0) return PSB_OK;
  if (tiles >= (int64_t(1) << 31)) return PSB_ERR_UNSUPPORTED;
  const int sms = device_sm_count();
  if (sms <= 0) return PSB_ERR_CUDA;
  p.max_cta_tiles = tc_max_cta_tiles(p, sms);
  const size_t smem = tc_smem_bytes(max_level, p.num_seqs, p.max_cta_tiles);
  const auto bf = p.paged ? prefill_tc_kernel<__nv_bfloat16, true> : prefill_tc_kernel<__nv_bfloat16, false>;
  const auto hf = p.paged ? prefill_tc_kernel<__half, true> : prefill_tc_kernel<__half, false>;
  const void* kern = dtype == PSB_BF16 ? reinterpret_cast<const void*>(bf) : reinterpret_cast<const void*>(hf);
  int occ = 0;
  if (!kernel_occupancy(kern, kTcThreads, smem, &occ) || occ < 1) return PSB_ERR_CUDA;
  const int64_t grid = std::min<int64_t>(tiles, static_cast<int64_t>(sms) * occ);  // persistent
  discard_stale_error();
  cudaError_t e;
  if (dtype == PSB_BF16)
    e = launch_pdl(bf, dim3(static_cast<unsigned>(grid)), dim3(kTcThreads), smem, s, p, tq, tk, tv);
  else
    e = launch_pdl(hf, dim3(static_cast<unsigned>(grid)), dim3(kTcThreads), smem, s, p, tq, tk, tv);
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}

}  // namespace psb
