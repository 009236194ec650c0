// Packed ragged causal prefill on the 5th-generation tensor cores (sm_100a).
//
// Replaces the reference's one-request-at-a-time prefill attention
// (pagedserve/attention/qwen_paged_attention.py:121-128 calling
// pagedserve/attention/paged_attention.py:239-305) for bf16/f16, head_dim 64:
// q [T, Hq, 64], k/v [T, Hkv, 64], sequence i = rows cu[i] .. cu[i+1], causal
// within each sequence, q head h reads kv head h / (Hq / Hkv).
//
// One CTA (five warps, 80 KB of shared memory, 256 TMEM columns, two CTAs
// per SM) takes a tile of 128 query rows of one q head.  Tiles are numbered
// heaviest first (a tile of query block i needs 2 (i + 1) key tiles), with
// the q heads of a tile adjacent so they share K/V through L2.  Warp 4 is the
// producer: one lane issues every TMA copy and every tcgen05.mma.  Warps 0-3
// (thread r = TMEM lane r = query row r) do the softmax.  They meet only on
// mbarriers, so the tensor core works while the softmax runs.  Per key tile
// j of 64 keys, streamed through a 4-stage TMA ring (128-byte swizzle):
//   producer: S_{j+1} = Q K_{j+1}^T (four tcgen05.mma, M 128, N 64, K 16;
//   fp32 into one of two TMEM buffers) as soon as K_{j+1} lands;
//   softmax: thread r loads its row of S_j, masks keys past its own position
//   or past the sequence and stores P = exp2(S - m) rounded to the input type
//   (as the reference rounds the probabilities before P.V,
//   paged_attention.py:291-302) to its TMEM lane, two keys per column.  m is a lazily updated row max: only when a row's max grows by
//   more than 2^8 is the O accumulated so far in TMEM rescaled (so P stays
//   below 256 and most steps touch no O at all);
//   producer: O += P_j V_j (four tcgen05.mma with P read from TMEM, N 64, V as
//   an MN-major operand, accumulating in TMEM across tiles), then requests K/V
//   tile j + 3 into the stage P.V_{j-1} freed.
// Every mbarrier wait is bounded; on a timeout the CTA records
// PSB_DEVERR_TIMEOUT, waits (bounded) for its copies in flight, frees TMEM and
// returns.
#include "common.cuh"
#include "host_util.h"
#include "varlen_prefill.h"

namespace psb {
namespace {

constexpr int kSoftmaxThreads = 128;  // warps 0-3: warp w <-> TMEM lanes and tile rows 32 w .. 32 w + 31
constexpr int kTcThreads = kSoftmaxThreads + 32;  // warp 4: TMA and MMA issue
constexpr int kBM = 128;         // query rows per tile
constexpr int kBN = 64;          // keys per tile
constexpr int kDim = 64;
constexpr uint32_t kTile = kBM * kDim * 2;   // bytes of the Q tile and of P (16 KB)
constexpr uint32_t kKvTile = kBN * kDim * 2;  // bytes of one K or V tile (8 KB)
constexpr int kKvStages = 4;                 // K/V ring depth
constexpr uint32_t kTmemCols = 256;  // S buffers: cols [0, 64), [64, 128); O: [128, 192); P: [192, 224)
constexpr uint32_t kPCol = 192;
constexpr float kRescaleLog2 = 8.f;  // rescale O when a row max grows by more than 2^8
constexpr uint32_t kSCol = 0, kOCol = 128;
// dynamic shared memory (1024-byte aligned): Q | K ring | V ring
constexpr uint32_t kOffQ = 0, kOffK = kTile, kOffV = kTile + kKvStages * kKvTile;
constexpr uint32_t kSmemTiles = kTile + 2 * kKvStages * kKvTile;
constexpr int kMaxLevels = 1024;  // query blocks per sequence (128 K tokens)

// Length of sequence s; 0 unless 0 <= cu[s] <= cu[s+1] <= total (a malformed
// batch is reported by the caller's check and must not be read out of bounds).
__device__ __forceinline__ int seq_len(const PrefillParams& p, int s) {
  const int a = p.cu[s], b = p.cu[s + 1];
  if (a < 0 || b < a || b > p.total) return 0;
  return min(b - a, p.max_seqlen);
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 2)
    prefill_tc_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar_q = reinterpret_cast<uint64_t*>(smem + kSmemTiles);
  uint64_t* bar_kv = bar_q + 1;  // [kKvStages]
  uint64_t* bar_s = bar_q + 5;   // [2]
  uint64_t* bar_o = bar_q + 7;
  uint64_t* bar_p = bar_q + 8;   // softmax step done: P written, S and the O tile read
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar_q + 9);
  int32_t* s_info = reinterpret_cast<int32_t*>(bar_q + 10);   // seq, level
  int32_t* s_count = reinterpret_cast<int32_t*>(bar_q + 11);  // [max_level + 1] sequences per top level

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hq = p.hq, group = p.hq / p.hkv;
  const int head = static_cast<int>(blockIdx.x % hq);
  const int tile = static_cast<int>(blockIdx.x / hq);
  // cu_seqlens, q, k and v may come from the stream predecessor
  pdl_wait();

  // ---- tile -> (sequence, query block), heaviest blocks first ------------
  const int max_level = (p.max_seqlen + kBM - 1) / kBM;
  for (int i = tid; i <= max_level; i += kTcThreads) s_count[i] = 0;
  __syncthreads();
  for (int s = tid; s < p.num_seqs; s += kTcThreads) {
    const int nb = (seq_len(p, s) + kBM - 1) / kBM;
    if (nb > 0) atomicAdd(&s_count[nb - 1], 1);  // sequences whose top level is nb - 1
  }
  __syncthreads();
  if (warp == 0) {
    // tiles at level i = sequences with more than i blocks = suffix sum of s_count
    int level = -1, rank = 0, run = 0, above = 0;
    for (int i = max_level - 1; i >= 0 && level < 0; --i) {
      above += s_count[i];  // sequences reaching level i
      if (tile < run + above) {
        level = i;
        rank = tile - run;
      }
      run += above;
    }
    int seq = -1;
    if (level >= 0) {  // the rank-th sequence (by index) with more than ``level`` blocks
      int seen = 0;
      for (int s0 = 0; s0 < p.num_seqs && seq < 0; s0 += 32) {
        const int s = s0 + lane;
        bool hit = false;
        if (s < p.num_seqs) hit = (seq_len(p, s) + kBM - 1) / kBM > level;
        const uint32_t m = __ballot_sync(0xffffffffu, hit);
        const int c = __popc(m);
        if (rank < seen + c) {
          uint32_t mm = m;
          for (int k = 0; k < rank - seen; ++k) mm &= mm - 1;
          seq = s0 + __ffs(mm) - 1;
        }
        seen += c;
      }
    }
    if (lane == 0) {
      s_info[0] = seq;
      s_info[1] = level;
    }
  }
  __syncthreads();
  const int seq = s_info[0], qblk = s_info[1];
  if (seq < 0) return;  // grid is sized for an upper bound of the tiles

  const int q0 = p.cu[seq];
  const int len = seq_len(p, seq);
  const int kvh = head / group;
  const int n_kv = min(2 * (qblk + 1), (len + kBN - 1) / kBN);
  const uint32_t s_base = smem_u32(smem);

  // ---- set-up: barriers, TMEM ----------------------------------------------
  if (tid == 0) {
    mbar_init(bar_q, 1);
    for (int i = 0; i < kKvStages; ++i) mbar_init(bar_kv + i, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_s + 1, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_p, kSoftmaxThreads);
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

  if (warp == 4) {
    // ---- producer: one lane issues every copy and MMA ----------------------
    if (lane == 0) {
      const uint32_t fmt = Elem<T>::code == PSB_BF16 ? 1u : 0u;
      const uint32_t idesc_s = umma_idesc_f16(fmt, kBM, kBN, 0, 0);
      const uint32_t idesc_o = umma_idesc_f16(fmt, kBM, kDim, 0, 1);
      auto load_kv = [&](int t) {
        const int st = t % kKvStages;
        mbar_arrive_expect_tx(bar_kv + st, 2 * kKvTile);
        tma_load_3d(smem + kOffK + st * kKvTile, &tm_k, 0, kvh, q0 + t * kBN, bar_kv + st);
        tma_load_3d(smem + kOffV + st * kKvTile, &tm_v, 0, kvh, q0 + t * kBN, bar_kv + st);
      };
      // descriptors of stage 0; a k-step of 16 elements advances the
      // address field (bytes >> 4) by 2, a K/V stage by kKvTile >> 4, a V
      // k-step of 16 keys by 2048 >> 4
      const uint64_t dq = umma_desc_sw128(s_base + kOffQ, 1024, 16);
      const uint64_t dk = umma_desc_sw128(s_base + kOffK, 1024, 16);
      const uint64_t dv = umma_desc_sw128(s_base + kOffV, 1024, 8192);
      auto issue_qk = [&](int t) {  // K_t landed, S buffer t & 1 read by the softmax of t - 2
        tc_fence_after();
        const uint64_t dks = dk + static_cast<uint64_t>((t % kKvStages) * (kKvTile >> 4));
#pragma unroll
        for (int k = 0; k < kDim / 16; ++k)
          umma_f16_ss(tmem + kSCol + (t & 1) * kBN, dq + 2 * k, dks + 2 * k, idesc_s, k > 0);
        umma_commit(bar_s + (t & 1));
      };
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(bar_q, kTile);
      tma_load_3d(smem + kOffQ, &tm_q, 0, head, q0 + qblk * kBM, bar_q);
      int kv_req = 0, kv_seen = 0, qk_issued = 0, pv_issued = 0, pv_seen = 0, p_seen = 0;
      for (; kv_req < min(n_kv, kKvStages - 1); ++kv_req) load_kv(kv_req);
      bool q_ok = mbar_wait(bar_q, 0);
      if (q_ok && mbar_wait(bar_kv, 0)) {
        kv_seen = 1;
        issue_qk(0);
        qk_issued = 1;
      } else {
        fail = true;
      }
      for (int j = 0; j < n_kv && !fail; ++j) {
        // S_{j+1}: its buffer held S_{j-1}, read by the softmax step j - 1 seen last time
        if (j + 1 < n_kv) {
          if (!mbar_wait(bar_kv + (j + 1) % kKvStages, ((j + 1) / kKvStages) & 1)) {
            fail = true;
            break;
          }
          ++kv_seen;
          issue_qk(j + 1);
          ++qk_issued;
        }
        // softmax step j done: P_j written, S_j and O_{j-1} read
        if (!mbar_wait(bar_p, j & 1)) {
          fail = true;
          break;
        }
        ++p_seen;
        // P.V_{j-1} done (waited before P.V_j is issued, so the parity cannot
        // alias): the stage of tile j - 1 is free for tile j + 3
        if (j > 0) {
          if (!mbar_wait(bar_o, (j - 1) & 1)) {
            fail = true;
            break;
          }
          ++pv_seen;
        }
        if (kv_req < n_kv && kv_req <= j + kKvStages - 1) load_kv(kv_req++);
        tc_fence_after();
        const uint64_t dvs = dv + static_cast<uint64_t>((j % kKvStages) * (kKvTile >> 4));
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k)
          umma_f16_ts(tmem + kOCol, tmem + kPCol + 8 * k, dvs + 128 * k, idesc_o, j > 0 || k > 0);
        umma_commit(bar_o);
        ++pv_issued;
      }
      if (fail) {
        flag_error(p.err, PSB_DEVERR_TIMEOUT);
        // let copies and MMAs still in flight land before shared memory and TMEM are released
        if (!q_ok) (void)mbar_wait(bar_q, 0);
        for (int t = kv_seen; t < kv_req; ++t) (void)mbar_wait(bar_kv + t % kKvStages, (t / kKvStages) & 1);
        for (int t = pv_seen; t < pv_issued; ++t) (void)mbar_wait(bar_o, t & 1);
        (void)qk_issued;
        (void)p_seen;
      }
    }
  } else {
    // ---- softmax warps ------------------------------------------------------
    const int row = warp * 32 + lane;   // tile row = TMEM lane
    const int qrow = qblk * kBM + row;  // position in the sequence
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float sc = p.scale_log2;
    float ms = -INFINITY, l_run = 0.f;  // row max used for the exponents (scaled by sc), row sum
    for (int j = 0; j < n_kv && !fail; ++j) {
      if (!mbar_wait(bar_s + (j & 1), (j >> 1) & 1)) {
        fail = true;
        break;
      }
      tc_fence_after();
      uint32_t sr[kBN];
      tmem_ld32(t_lane + kSCol + (j & 1) * kBN, sr);
      tmem_ld32(t_lane + kSCol + (j & 1) * kBN + 32, sr + 32);
      tmem_wait_ld();
      // keys past this row's position or past the sequence only occur in the last tiles
      const int lim = min(qrow, len - 1) - j * kBN;  // last valid key column
      const bool interior = lim >= kBN - 1;
      float mx = -INFINITY;
      if (interior) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) mx = fmaxf(mx, __uint_as_float(sr[c]));
      } else {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          if (c > lim) sr[c] = __float_as_uint(-INFINITY);
          mx = fmaxf(mx, __uint_as_float(sr[c]));
        }
      }
      // lazy max: move it (and rescale O and the sum) only when the row max
      // grew by more than 2^kRescaleLog2; the warp's TMEM access is collective
      const float mxs = mx * sc;
      const bool grow = mxs > ms + kRescaleLog2;
      if (__any_sync(0xffffffffu, grow)) {
        const float ms_new = grow ? mxs : ms;
        const float alpha = ms == -INFINITY ? 0.f : ex2_approx(ms - ms_new);  // 1 where the max stays
        if (j > 0) {  // O holds P.V of the earlier tiles once the last of them is done
          if (!mbar_wait(bar_o, (j - 1) & 1)) {
            fail = true;
            break;
          }
          tc_fence_after();
          uint32_t ot[kDim];
          tmem_ld32(t_lane + kOCol, ot);
          tmem_ld32(t_lane + kOCol + 32, ot + 32);
          tmem_wait_ld();
#pragma unroll
          for (int d = 0; d < kDim; ++d) ot[d] = __float_as_uint(__uint_as_float(ot[d]) * alpha);
          tmem_st32(t_lane + kOCol, ot);
          tmem_st32(t_lane + kOCol + 32, ot + 32);
          tmem_wait_st();
        }
        l_run *= alpha;
        ms = ms_new;
      }
      const float mu = ms == -INFINITY ? 0.f : ms;  // rows with nothing valid yet stay zero
      float rs = 0.f;
      uint32_t pk[kBN / 2];
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        const float x0 = ex2_approx(fmaf(__uint_as_float(sr[c]), sc, -mu));
        const float x1 = ex2_approx(fmaf(__uint_as_float(sr[c + 1]), sc, -mu));
        rs += x0 + x1;
        pk[c / 2] = pack2<T>(x0, x1);
      }
      l_run += rs;
      // P_j overwrites P_{j-1} in TMEM: wait for P.V_{j-1} (issued right after step
      // j - 1, so normally long done; P.V_j cannot start before this thread's
      // arrival below, so the parity cannot alias)
      if (j > 0) {
        if (!mbar_wait(bar_o, (j - 1) & 1)) {
          fail = true;
          break;
        }
      }
      tmem_st32(t_lane + kPCol, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p);
    }
    if (!fail && !mbar_wait(bar_o, (n_kv - 1) & 1)) fail = true;  // the last P.V
    if (fail) {
      if (lane == 0) flag_error(p.err, PSB_DEVERR_TIMEOUT);
    } else {
      tc_fence_after();
      uint32_t ot[kDim];
      tmem_ld32(t_lane + kOCol, ot);
      tmem_ld32(t_lane + kOCol + 32, ot + 32);
      tmem_wait_ld();
      if (qrow < len && q0 + qrow < p.total) {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        T* op = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(q0 + qrow) * p.ost +
                static_cast<int64_t>(head) * p.osh;
#pragma unroll
        for (int d = 0; d < kDim; d += 2)
          *reinterpret_cast<uint32_t*>(op + d) =
              pack2<T>(__uint_as_float(ot[d]) * inv, __uint_as_float(ot[d + 1]) * inv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

size_t tc_smem_bytes(int max_level) { return 1024 + kSmemTiles + 88 + sizeof(int32_t) * (max_level + 2); }

}  // namespace

bool prefill_tc_supported(const PrefillParams& p, int dtype) {
  if (!(dtype == PSB_BF16 || dtype == PSB_F16) || p.head_dim != kDim) return false;
  auto al16 = [](const void* x) { return reinterpret_cast<uintptr_t>(x) % 16 == 0; };
  // TMA: 16-byte aligned bases and strides; 4-byte output pairs
  const bool strides = p.qst % 8 == 0 && p.qsh % 8 == 0 && p.kst % 8 == 0 && p.ksh % 8 == 0 && p.vst % 8 == 0 &&
                       p.vsh % 8 == 0 && p.ost % 2 == 0 && p.osh % 2 == 0 && p.qst > 0 && p.kst > 0 && p.vst > 0;
  const int max_level = (p.max_seqlen + kBM - 1) / kBM;
  return strides && al16(p.q) && al16(p.k) && al16(p.v) && reinterpret_cast<uintptr_t>(p.out) % 4 == 0 &&
         max_level <= kMaxLevels && tc_smem_bytes(max_level) <= 227 * 1024;
}

int prefill_tc_launch(const PrefillParams& p, int dtype, cudaStream_t s) {
  const CUtensorMapDataType dt = dtype == PSB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tk, tv;
  if (!encode_rows_map(&tq, p.q, p.total, p.hq, kDim, p.qst, p.qsh, kBM, dt) ||
      !encode_rows_map(&tk, p.k, p.total, p.hkv, kDim, p.kst, p.ksh, kBN, dt) ||
      !encode_rows_map(&tv, p.v, p.total, p.hkv, kDim, p.vst, p.vsh, kBN, dt))
    return PSB_ERR_CUDA;
  const int max_level = (p.max_seqlen + kBM - 1) / kBM;
  // an upper bound of the tiles: sum over sequences of ceil(len / 128)
  const int64_t tiles = static_cast<int64_t>(p.total) / kBM + p.num_seqs;
  const int64_t grid = tiles * p.hq;
  if (grid == 0) return PSB_OK;
  if (grid >= (int64_t(1) << 31)) return PSB_ERR_UNSUPPORTED;
  const size_t smem = tc_smem_bytes(max_level);
  const void* kern = dtype == PSB_BF16 ? reinterpret_cast<const void*>(prefill_tc_kernel<__nv_bfloat16>)
                                       : reinterpret_cast<const void*>(prefill_tc_kernel<__half>);
  int occ = 0;
  if (!kernel_occupancy(kern, kTcThreads, smem, &occ) || occ < 1) return PSB_ERR_CUDA;
  discard_stale_error();
  cudaError_t e;
  if (dtype == PSB_BF16)
    e = launch_pdl(prefill_tc_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(grid)), dim3(kTcThreads), smem, s, p,
                   tq, tk, tv);
  else
    e = launch_pdl(prefill_tc_kernel<__half>, dim3(static_cast<unsigned>(grid)), dim3(kTcThreads), smem, s, p, tq, tk,
                   tv);
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}

}  // namespace psb
