// Packed ragged causal prefill on the 5th-generation tensor cores (sm_100a).
//
// Replaces the reference's one-request-at-a-time prefill attention
// (pagedserve/attention/qwen_paged_attention.py:121-128 calling
// pagedserve/attention/paged_attention.py:239-305) for bf16/f16, head_dim 64:
// q [T, Hq, 64], k/v [T, Hkv, 64], sequence i = rows cu[i] .. cu[i+1], causal
// within each sequence, q head h reads kv head h / (Hq / Hkv).
//
// One CTA (4 warps, one persistent TMEM allocation) takes a tile of 128
// query rows of one q head.  Tiles are numbered heaviest first (a tile of
// query block i needs i + 1 key tiles), with the q heads of a tile adjacent so
// they share K/V through L2.  Per key tile j:
//   TMA (128-byte swizzle) brings K_j and V_j into a double-buffered ring;
//   S = Q K_j^T: four tcgen05.mma (M 128, N 128, K 16), fp32 in TMEM cols 0-127;
//   thread r (TMEM lane r) loads its row of S, masks keys past its own
//   position or past the sequence, keeps the running max, writes
//   P = exp2(S - max) rounded to the input type (as the reference rounds the
//   probabilities before P.V, paged_attention.py:291-302) to shared memory in
//   the swizzled K-major layout the next MMA reads;
//   O_j = P V_j: eight tcgen05.mma (N 64, V as an MN-major operand) into TMEM
//   cols 128-191, which thread r folds into its register row of O with the
//   online-softmax rescale.
// Every mbarrier wait is bounded; on a timeout the CTA records
// PSB_DEVERR_TIMEOUT, waits (bounded) for its copies in flight, frees TMEM and
// returns.
#include "common.cuh"
#include "host_util.h"
#include "varlen_prefill.h"

namespace psb {
namespace {

constexpr int kTcThreads = 128;  // warp w <-> TMEM lanes and tile rows 32 w .. 32 w + 31
constexpr int kBM = 128;         // query rows per tile
constexpr int kBN = 128;         // keys per tile
constexpr int kDim = 64;
constexpr uint32_t kTile = kBM * kDim * 2;  // bytes of one Q, K or V tile (16 KB)
constexpr uint32_t kTmemCols = 256;         // S: cols [0, 128), O tile: [128, 192)
constexpr uint32_t kSCol = 0, kOCol = 128;
// dynamic shared memory (1024-byte aligned): Q | K0 | K1 | V0 | V1 | P (2 x 16 KB k-blocks)
constexpr uint32_t kOffQ = 0, kOffK = kTile, kOffV = 3 * kTile, kOffP = 5 * kTile;
constexpr uint32_t kSmemTiles = 7 * kTile;
constexpr int kMaxLevels = 1024;  // query blocks per sequence (128 K tokens)

// Length of sequence s; 0 unless 0 <= cu[s] <= cu[s+1] <= total (a malformed
// batch is reported by the caller's check and must not be read out of bounds).
__device__ __forceinline__ int seq_len(const PrefillParams& p, int s) {
  const int a = p.cu[s], b = p.cu[s + 1];
  if (a < 0 || b < a || b > p.total) return 0;
  return min(b - a, p.max_seqlen);
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar_q = reinterpret_cast<uint64_t*>(smem + kSmemTiles);
  uint64_t* bar_kv = bar_q + 1;  // [2]
  uint64_t* bar_s = bar_q + 3;
  uint64_t* bar_o = bar_q + 4;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar_q + 5);
  int32_t* s_info = reinterpret_cast<int32_t*>(bar_q + 6);  // seq, level
  int32_t* s_count = reinterpret_cast<int32_t*>(bar_q + 8);  // [kMaxLevels + 1] tiles per level

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
  const int n_kv = qblk + 1;
  const uint32_t s_base = smem_u32(smem);

  // ---- set-up: barriers, TMEM, first loads ---------------------------------
  if (tid == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_kv, 1);
    mbar_init(bar_kv + 1, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
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
  if (tid == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    mbar_arrive_expect_tx(bar_q, kTile);
    tma_load_3d(smem + kOffQ, &tm_q, 0, head, q0 + qblk * kBM, bar_q);
    mbar_arrive_expect_tx(bar_kv, 2 * kTile);
    tma_load_3d(smem + kOffK, &tm_k, 0, kvh, q0, bar_kv);
    tma_load_3d(smem + kOffV, &tm_v, 0, kvh, q0, bar_kv);
  }

  const uint32_t fmt = Elem<T>::code == PSB_BF16 ? 1u : 0u;
  const uint32_t idesc_s = umma_idesc_f16(fmt, kBM, kBN, 0, 0);
  const uint32_t idesc_o = umma_idesc_f16(fmt, kBM, kDim, 0, 1);

  const int row = warp * 32 + lane;     // tile row = TMEM lane
  const int qrow = qblk * kBM + row;    // position in the sequence
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  float o[kDim];
#pragma unroll
  for (int d = 0; d < kDim; ++d) o[d] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  uint32_t ph_s = 0, ph_o = 0;
  int kv_issued = 1, kv_waited = 0;  // K/V tiles whose loads were issued / waited for
  bool fail = false;

  const bool q_ok = mbar_wait(bar_q, 0);
  fail = __syncthreads_or(!q_ok);
  for (int j = 0; j < n_kv && !fail; ++j) {
    const int buf = j & 1;
    if (mbar_wait(bar_kv + buf, (j >> 1) & 1))
      ++kv_waited;
    else
      fail = true;
    if (__syncthreads_or(fail)) {
      fail = true;
      break;
    }
    if (tid == 0) {
      tc_fence_after();
      const uint32_t q_addr = s_base + kOffQ, k_addr = s_base + kOffK + buf * kTile;
#pragma unroll
      for (int k = 0; k < kDim / 16; ++k)
        umma_f16_ss(tmem + kSCol, umma_desc_sw128(q_addr + 32 * k, 1024, 16), umma_desc_sw128(k_addr + 32 * k, 1024, 16),
                    idesc_s, k > 0);
      umma_commit(bar_s);
      // next K/V into the other buffer (its last reader, the P.V of tile j - 1, is complete)
      if (j + 1 < n_kv) {
        mbar_arrive_expect_tx(bar_kv + (buf ^ 1), 2 * kTile);
        tma_load_3d(smem + kOffK + (buf ^ 1) * kTile, &tm_k, 0, kvh, q0 + (j + 1) * kBN, bar_kv + (buf ^ 1));
        tma_load_3d(smem + kOffV + (buf ^ 1) * kTile, &tm_v, 0, kvh, q0 + (j + 1) * kBN, bar_kv + (buf ^ 1));
      }
    }
    if (tid == 0 && j + 1 < n_kv) ++kv_issued;
    if (!mbar_wait(bar_s, ph_s)) fail = true;
    ph_s ^= 1;
    tc_fence_after();

    // ---- softmax of row ``row`` over keys 128 j .. 128 j + 127 ------------
    const int key0 = j * kBN;
    const int lim = min(qrow, len - 1) - key0;  // last valid key column (may be < 0 for padding rows)
    float sv[kBN];
#pragma unroll
    for (int c = 0; c < kBN; c += 32) tmem_ld32_sync(t_lane + kSCol + c, sv + c);
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < kBN; ++c) {
      sv[c] = c <= lim ? sv[c] * p.scale_log2 : -INFINITY;
      mx = fmaxf(mx, sv[c]);
    }
    const float m_new = fmaxf(m_run, mx);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;  // fully masked padding rows stay zero
    const float alpha = exp2f(m_run - m_use);                // 0 on the first tile
    float rs = 0.f;
    uint8_t* prow = smem + kOffP + row * 128;
#pragma unroll
    for (int c8 = 0; c8 < kBN / 8; ++c8) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a = exp2f(sv[c8 * 8 + 2 * e] - m_use), b = exp2f(sv[c8 * 8 + 2 * e + 1] - m_use);
        rs += a + b;
        w[e] = pack2<T>(a, b);
      }
      // k-block c8 / 8, 16-byte chunk c8 % 8 of the 128-byte row, swizzled by row % 8
      uint8_t* dst = prow + (c8 >> 3) * kTile + (((c8 & 7) ^ (row & 7)) << 4);
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    l_run = l_run * alpha + rs;
    m_run = m_new;
    fence_proxy_async_smem();  // P visible to the tensor core
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t p_addr = s_base + kOffP, v_addr = s_base + kOffV + buf * kTile;
#pragma unroll
      for (int k = 0; k < kBN / 16; ++k)
        umma_f16_ss(tmem + kOCol, umma_desc_sw128(p_addr + (k >> 2) * kTile + 32 * (k & 3), 1024, 16),
                    umma_desc_sw128(v_addr + 2048 * k, 1024, 8192), idesc_o, k > 0);
      umma_commit(bar_o);
    }
    if (!mbar_wait(bar_o, ph_o)) fail = true;
    ph_o ^= 1;
    tc_fence_after();
    float ot[kDim];
    tmem_ld32_sync(t_lane + kOCol, ot);
    tmem_ld32_sync(t_lane + kOCol + 32, ot + 32);
#pragma unroll
    for (int d = 0; d < kDim; ++d) o[d] = fmaf(o[d], alpha, ot[d]);
    tc_fence_before();
    if (__syncthreads_or(fail)) fail = true;  // S, the O tile, P and K/V[buf] are free again
  }

  if (fail) {
    if (tid == 0) {
      flag_error(p.err, PSB_DEVERR_TIMEOUT);
      // let copies still in flight land before the shared memory is released
      if (!q_ok) (void)mbar_wait(bar_q, 0);
      for (int k = kv_waited; k < kv_issued; ++k) (void)mbar_wait(bar_kv + (k & 1), (k >> 1) & 1);
    }
  } else if (qrow < len) {
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    T* op = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(q0 + qrow) * p.ost + static_cast<int64_t>(head) * p.osh;
#pragma unroll
    for (int d = 0; d < kDim; d += 2) *reinterpret_cast<uint32_t*>(op + d) = pack2<T>(o[d] * inv, o[d + 1] * inv);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

size_t tc_smem_bytes(int max_level) { return 1024 + kSmemTiles + 64 + sizeof(int32_t) * (max_level + 2); }

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
