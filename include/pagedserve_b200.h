/*
 * pagedserve_b200 - C ABI of the B200 (sm_100a) paged-attention hot path.
 *
 * One shared library, libpagedserve_b200.so.  Every entry point takes raw
 * device pointers, element strides (int64), sizes (int32/int64) and a CUDA
 * stream, returns an int status (PSB_OK or a negative PSB_ERR_*), never
 * throws, never allocates device memory and is asynchronous on the given
 * stream.  The caller owns every buffer.
 *
 * KV pool layout (unchanged from PagedServe, pagedserve/engine/kv_cache.py:10-16,51-69):
 *     k_cache, v_cache : [num_layers, num_blocks, num_kv_heads, block_size, head_dim], contiguous
 * so (layer, block, kv_head) is one contiguous block_size x head_dim tile.
 *
 * Device-detected problems (a block id outside the pool, a slot outside the
 * pool, a context longer than its block table, an exhausted wait) never trap:
 * the offending access is skipped and a PSB_DEVERR_* bit is OR-ed into the
 * optional int32 word ``error_flag`` (device memory; may be NULL).
 */
#ifndef PAGEDSERVE_B200_H_
#define PAGEDSERVE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* psb_stream_t;

/* element types (the reference supports these three: triton_paged_decode.py:110) */
enum { PSB_F32 = 0, PSB_F16 = 1, PSB_BF16 = 2 };

/* host-side status codes */
enum {
  PSB_OK = 0,
  PSB_ERR_INVALID = -1,     /* bad shape, stride, pointer or size argument */
  PSB_ERR_WORKSPACE = -2,   /* workspace smaller than *_workspace_size() */
  PSB_ERR_UNSUPPORTED = -3, /* geometry/dtype the library has no kernel for */
  PSB_ERR_CUDA = -4         /* a CUDA runtime/driver call failed (see psb_last_cuda_error) */
};

/* device-side error bits written to *error_flag */
enum {
  PSB_DEVERR_BLOCK_RANGE = 1,   /* block id from a table outside [0, num_blocks) */
  PSB_DEVERR_SLOT_RANGE = 2,    /* slot outside [0, num_blocks * block_size) */
  PSB_DEVERR_CONTEXT = 4,       /* context length > table width * block_size, or < 0 */
  PSB_DEVERR_WORKSPACE = 8,     /* split-K work exceeded the workspace */
  PSB_DEVERR_TIMEOUT = 16,      /* an async copy / MMA wait exceeded its bound */
  PSB_DEVERR_SEQLENS = 32,      /* cu_seqlens not non-decreasing within [0, total] */
  PSB_DEVERR_LIMIT = 64         /* psb_select_tokens: a row had no tokens left to generate */
};

/* per-row status bits written by psb_select_tokens */
enum {
  PSB_SELECT_DONE = 1,  /* the request finishes with this token (EOS, or its last allowed token) */
  PSB_SELECT_EOS = 2,   /* the token is one of the EOS ids */
  PSB_SELECT_LIMIT = 4  /* the row had no tokens left on entry: nothing was counted (flagged) */
};

/* Library version string, e.g. "pagedserve_b200 0.1.0 sm_100a". */
const char* psb_version(void);

/* Text for a PSB_* status code. */
const char* psb_status_string(int status);

/* Last CUDA error code seen by the library on this thread (0 if none). */
int psb_last_cuda_error(void);

/*
 * reshape_and_cache: slot-mapped scatter of new tokens' K/V into the pools.
 *
 * Replaces PagedKVCache.write_token (pagedserve/engine/paged_kv_cache.py:148-200),
 * which the reference calls once per token per layer
 * (pagedserve/attention/batched_paged_attention.py:115-124,
 *  pagedserve/attention/qwen_paged_attention.py:110-119).  For token t with
 * slot s = slot_mapping[t] (int64): block = s / block_size, offset = s % block_size,
 *     k_cache[layer, block, h, offset, :] = key[t, h, :]   (and v likewise)
 * bit-exactly.  A negative slot writes nothing (padding row).  key/value are
 * [num_tokens, num_kv_heads, head_dim] with element strides (stride_t,
 * stride_h) and unit stride along head_dim.  Launched as a programmatic
 * dependent: it may start before its stream predecessor ends (it waits for
 * it before touching memory) and lets the kernel after it start at once.
 */
int psb_reshape_and_cache(const void* key, int64_t key_stride_t, int64_t key_stride_h, const void* value,
                          int64_t value_stride_t, int64_t value_stride_h, void* k_cache, void* v_cache,
                          const int64_t* slot_mapping, int32_t num_tokens, int32_t layer, int32_t num_layers,
                          int64_t num_blocks, int32_t num_kv_heads, int32_t block_size, int32_t head_dim,
                          int32_t dtype, int32_t* error_flag, psb_stream_t stream);

/*
 * Workspace bytes psb_paged_decode needs for ``batch`` sequences whose
 * contexts are at most ``max_context`` tokens: split-K partials (fixed
 * ~7.7 MB on the bf16/f16 path, which splits the pool blocks evenly over at
 * most 160 CTAs) or, on the CUDA-core path, per-chunk partials plus one
 * arrival counter per (sequence, kv head).  Returns the larger of the two,
 * 0 for an invalid geometry.  The workspace needs no initialisation: each
 * call clears what it relies on.
 */
size_t psb_paged_decode_workspace_size(int32_t batch, int32_t q_heads, int32_t num_kv_heads, int32_t head_dim,
                                       int32_t block_size, int32_t max_context, int32_t dtype);

/* Zero the arrival-counter region of a workspace (async memset on
 * ``stream``).  Optional: psb_paged_decode clears what it relies on itself;
 * this is for callers that want a freshly allocated workspace in a known
 * state before its first use. */
int psb_paged_decode_workspace_init(void* workspace, size_t workspace_bytes, int32_t batch, int32_t num_kv_heads,
                                    psb_stream_t stream);

/*
 * paged_decode: single-token GQA decode attention over the paged pool.
 *
 * Replaces the reference's _paged_decode_kernel launch
 * (pagedserve/attention/triton_paged_decode.py:10-95, launched at :161-172)
 * and, numerically, vectorized_paged_attention
 * (pagedserve/attention/vectorized_batched_attention.py:79-159):
 *     out[b, h, :] = softmax(scale * q[b, h, :] . K_b^T) V_b
 * over the first context_lens[b] tokens of sequence b, read through
 * block_tables[b, :] (int32, row stride ``table_stride`` elements); q head h
 * reads kv head h / (q_heads / num_kv_heads).  query/out are [batch, q_heads,
 * head_dim] with element strides (stride_b, stride_h) and unit stride along
 * head_dim, in the pool's dtype.  Softmax and accumulation are fp32.
 * ``max_context`` bounds every context_lens[b] (host-known, e.g. table width
 * x block_size).  bf16/f16 with head_dim 64 and block_size 16 split the
 * pool blocks of all sequences evenly over the SMs and merge the partials of
 * sequences that span several warps in a second kernel on the same stream;
 * other geometries run a CUDA-core kernel.  Context lengths and block tables
 * are read before the kernel waits on its stream predecessor (programmatic
 * dependent launch), possibly while the kernels this library launched just
 * before (reshape_and_cache, decode, combine, varlen_prefill) still run:
 * they must be written by an earlier kernel that is not one of those (an
 * ordinary launch such as pack_step's, or a host copy).  Calls sharing one
 * workspace must not overlap on the GPU.
 */
int psb_paged_decode(const void* query, int64_t q_stride_b, int64_t q_stride_h, void* out, int64_t o_stride_b,
                     int64_t o_stride_h, const void* k_cache, const void* v_cache, const int32_t* block_tables,
                     int64_t table_stride, const int32_t* context_lens, int32_t batch, int32_t q_heads,
                     int32_t layer, int32_t num_layers, int64_t num_blocks, int32_t num_kv_heads,
                     int32_t block_size, int32_t head_dim, int32_t dtype, int32_t max_context, float scale,
                     void* workspace, size_t workspace_bytes, int32_t* error_flag, psb_stream_t stream);

/*
 * rope_reshape_and_cache: rotary position embedding of q and k fused with the
 * slot-mapped K/V write.
 *
 * Replaces the transformers Qwen2 apply_rotary_pos_emb the reference applies
 * in its decode glue (pagedserve/attention/batched_paged_attention.py:105-112,
 * imported at :8) followed by the per-row write_token loop (:115-124):
 *     q'[t, h] = q[t, h] * cos[t] + rotate_half(q[t, h]) * sin[t]   (k' likewise),
 *     rotate_half(x) = cat(-x[D/2:], x[:D/2]),
 * then, for slot s = slot_mapping[t] >= 0, k'[t] and value[t] stored as
 * psb_reshape_and_cache stores them.  cos/sin are per-token rows
 * [num_tokens, head_dim] (row stride ``cs_stride_t`` elements; the engine's
 * position embeddings, pagedserve/model/engine.py:572-575).  Products and sums
 * are evaluated in fp32 and rounded to ``dtype`` as PyTorch evaluates that
 * expression, so query_out, key_out and the pool bytes are bit-identical to
 * the reference's.  query [num_tokens, num_q_heads, head_dim] -> query_out
 * (either query itself, for in place, or not overlapping it); key_out may be
 * null (the rotated keys then go only to the pool).  head_dim must be even.
 * A slot past the pool is skipped and flagged (PSB_DEVERR_SLOT_RANGE).  A
 * programmatic dependent launch, like psb_reshape_and_cache.
 */
int psb_rope_reshape_and_cache(const void* query, int64_t q_stride_t, int64_t q_stride_h, void* query_out,
                               int64_t qo_stride_t, int64_t qo_stride_h, const void* key, int64_t k_stride_t,
                               int64_t k_stride_h, void* key_out, int64_t ko_stride_t, int64_t ko_stride_h,
                               const void* value, int64_t v_stride_t, int64_t v_stride_h, const void* cos,
                               const void* sin, int64_t cs_stride_t, void* k_cache, void* v_cache,
                               const int64_t* slot_mapping, int32_t num_tokens, int32_t num_q_heads, int32_t layer,
                               int32_t num_layers, int64_t num_blocks, int32_t num_kv_heads, int32_t block_size,
                               int32_t head_dim, int32_t dtype, int32_t* error_flag, psb_stream_t stream);

/*
 * paged_decode_append: the decode step's cache write and attention in one
 * launch.  Equivalent to writing row b's new key/value
 * ([batch, num_kv_heads, head_dim], element strides (stride_b, stride_h),
 * unit stride along head_dim) at position context_lens[b] - 1 of sequence
 * b - located through block_tables as PagedKVCache.write_token does
 * (pagedserve/engine/paged_kv_cache.py:187-200), the per-row loop of
 * pagedserve/attention/batched_paged_attention.py:115-124 - followed by
 * psb_paged_decode over the first context_lens[b] tokens, which include it.
 * The pool bytes written and the outputs are identical to that sequence.
 * Rows with context_lens[b] == 0 write nothing.  Each row's last block must
 * belong to that row alone (no two rows share it), as with any decode step.
 * Arguments, workspace, results and error behaviour are otherwise
 * psb_paged_decode's.
 */
int psb_paged_decode_append(const void* query, int64_t q_stride_b, int64_t q_stride_h, void* out,
                            int64_t o_stride_b, int64_t o_stride_h, void* k_cache, void* v_cache,
                            const void* new_key, int64_t key_stride_b, int64_t key_stride_h,
                            const void* new_value, int64_t value_stride_b, int64_t value_stride_h,
                            const int32_t* block_tables, int64_t table_stride, const int32_t* context_lens,
                            int32_t batch, int32_t q_heads, int32_t layer, int32_t num_layers, int64_t num_blocks,
                            int32_t num_kv_heads, int32_t block_size, int32_t head_dim, int32_t dtype,
                            int32_t max_context, float scale, void* workspace, size_t workspace_bytes,
                            int32_t* error_flag, psb_stream_t stream);

/*
 * paged_decode_args: psb_paged_decode / psb_paged_decode_append with the
 * arguments that stay the same for every layer call of one decode iteration
 * (pools, block table, lengths, geometry, scale, workspace, error flag)
 * passed as one caller-owned struct, filled once per batch; only the query,
 * output, new rows, layer and stream are passed per call.  new_key and
 * new_value both null: psb_paged_decode; both set: psb_paged_decode_append;
 * one of them null: PSB_ERR_INVALID.  Results, checks and error behaviour
 * are those of the two calls.  No counterpart in the reference: it exists so
 * an FFI host pays the marshalling of 14 arguments per layer call instead of
 * 32 (psb_decode_args_size() gives sizeof(psb_decode_args), for bindings to
 * check their layout).
 */
typedef struct psb_decode_args {
  void* k_cache;
  void* v_cache;
  const int32_t* block_tables;
  int64_t table_stride;
  const int32_t* context_lens;
  int64_t num_blocks;
  void* workspace;
  size_t workspace_bytes;
  int32_t* error_flag;
  int32_t batch;
  int32_t q_heads;
  int32_t num_layers;
  int32_t num_kv_heads;
  int32_t block_size;
  int32_t head_dim;
  int32_t dtype;
  int32_t max_context;
  float scale;
  int32_t reserved;  /* zero */
} psb_decode_args;

size_t psb_decode_args_size(void);

int psb_paged_decode_args(const psb_decode_args* args, const void* query, int64_t q_stride_b, int64_t q_stride_h,
                          void* out, int64_t o_stride_b, int64_t o_stride_h, const void* new_key,
                          int64_t key_stride_b, int64_t key_stride_h, const void* new_value,
                          int64_t value_stride_b, int64_t value_stride_h, int32_t layer, psb_stream_t stream);

/*
 * paged_decode_static: psb_paged_decode without a caller workspace.  It has
 * no counterpart in the reference (whose Triton decode needs no scratch); it
 * exists for callers that cannot allocate device memory where they launch
 * decode (a pre-carved memory pool, an FFI host that owns no CUDA memory).
 *
 * The split-K scratch is a file-scope device array of
 * psb_paged_decode_static_capacity() bytes (32 MiB) per device, reserved when
 * its module loads; the call allocates nothing.  Only the scratch of the path
 * the call takes is checked against that: the bf16/f16 head_dim-64 path needs
 * a fixed ~10.8 MB whatever the batch (256 sequences of up to 8192 tokens
 * fit); the CUDA-core path needs per-chunk partials that grow with batch x
 * max_context, and a call whose need exceeds the array returns
 * PSB_ERR_WORKSPACE.
 *
 * Set-up: the first call on each device looks up the array's address with
 * that device current (and may load the module); make that first call before
 * any stream capture.  Decode clears what it relies on itself (the CUDA-core
 * path zeroes its arrival counters at the start of every call; the fast
 * path's partial slots are written before they are read).  The scratch is
 * shared by every caller on a device and keeps the last call's contents:
 * calls that overlap on the GPU (other streams, other threads) race and must
 * be serialised by the caller.
 * Arguments, results and error behaviour are otherwise psb_paged_decode's.
 */
int psb_paged_decode_static(const void* query, int64_t q_stride_b, int64_t q_stride_h, void* out,
                            int64_t o_stride_b, int64_t o_stride_h, const void* k_cache, const void* v_cache,
                            const int32_t* block_tables, int64_t table_stride, const int32_t* context_lens,
                            int32_t batch, int32_t q_heads, int32_t layer, int32_t num_layers, int64_t num_blocks,
                            int32_t num_kv_heads, int32_t block_size, int32_t head_dim, int32_t dtype,
                            int32_t max_context, float scale, int32_t* error_flag, psb_stream_t stream);

/* Bytes of the per-device scratch behind psb_paged_decode_static. */
size_t psb_paged_decode_static_capacity(void);

/*
 * varlen_prefill: packed ragged causal attention over freshly projected
 * q [total, q_heads, D], k/v [total, num_kv_heads, D] (element strides
 * (stride_t, stride_h), unit stride along D).  Sequence i owns rows
 * cu_seqlens[i] .. cu_seqlens[i+1] and is causal within itself.
 *
 * Replaces the reference's one-request-at-a-time prefill attention
 * (pagedserve/attention/qwen_paged_attention.py:121-128 calling
 *  pagedserve/attention/paged_attention.py:10-146 with query_start_position 0).
 * bf16/f16 with head_dim 64 run on tcgen05 tensor cores with TMEM
 * accumulators fed by TMA; other geometries use a CUDA-core kernel.
 */
int psb_varlen_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k, int64_t k_stride_t,
                       int64_t k_stride_h, const void* v, int64_t v_stride_t, int64_t v_stride_h, void* out,
                       int64_t o_stride_t, int64_t o_stride_h, const int32_t* cu_seqlens, int32_t num_seqs,
                       int32_t total_tokens, int32_t max_seqlen, int32_t q_heads, int32_t num_kv_heads,
                       int32_t head_dim, int32_t dtype, float scale, int32_t* error_flag, psb_stream_t stream);

/*
 * paged_prefill: prefix-aware (chunked) causal prefill over the paged pool.
 *
 * The reference's paged_attention(query [Hq, S, D], cache, request_id, layer,
 * query_start_position) (pagedserve/attention/paged_attention.py:10-146), for
 * a packed batch: q [total_tokens, q_heads, head_dim] holds each sequence's
 * new rows, sequence i owning rows cu_seqlens[i] .. cu_seqlens[i+1] (n_i of
 * them); the sequence has context_lens[i] tokens in the pool, read through
 * block_tables[i, :], its query rows being the last n_i of them (their K/V
 * already written).  Row j attends to positions 0 .. context_lens[i] - n_i + j
 * (GQA, fp32 softmax, probabilities rounded to the input type before P.V).
 * With context_lens == n the result equals psb_varlen_prefill on the same
 * keys.  bf16/f16 with head_dim 64 and block_size 16 run the tcgen05 kernel
 * (pool tiles loaded by TMA through the table); other geometries a CUDA-core
 * kernel.  A context shorter than its query rows or longer than max_context,
 * and block ids outside the pool, are flagged (PSB_DEVERR_CONTEXT /
 * PSB_DEVERR_BLOCK_RANGE) instead of read.
 */
int psb_paged_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache,
                      const void* v_cache, const int32_t* block_tables, int64_t table_stride,
                      const int32_t* context_lens, void* out, int64_t o_stride_t, int64_t o_stride_h,
                      const int32_t* cu_seqlens, int32_t num_seqs, int32_t total_tokens, int32_t max_seqlen,
                      int32_t max_context, int32_t q_heads, int32_t layer, int32_t num_layers, int64_t num_blocks,
                      int32_t num_kv_heads, int32_t block_size, int32_t head_dim, int32_t dtype, float scale,
                      int32_t* error_flag, psb_stream_t stream);

/*
 * select_tokens: greedy next-token selection and the stop check of one decode
 * step, for every row of the batch, in one launch.
 *
 * Replaces the reference's
 *     tokens = logits[:, -1, :].argmax(dim=-1, keepdim=True)
 * followed by its per-row host loop - token.item(), add_generated_token
 * (which raises when no tokens remain), and the finish test
 * ``token_id in eos_ids or request.remaining_tokens == 0``
 * (pagedserve/engine/continuous_batcher.py:333-360, pagedserve/engine/request.py:84-106).
 *
 * logits     [batch, vocab] of ``dtype``, row stride ``row_stride`` elements
 *            (>= vocab when batch > 1), unit element stride; for the
 *            reference's [B, S, V] output pass the last position's rows
 *            (base + (S-1)*V, row_stride = S*V).
 * eos_ids    [num_eos] int64 (num_eos <= 64; may be NULL when 0)
 * remaining  [batch] int32, in/out: tokens each request may still generate
 *            (max_new_tokens - generated); decremented by one per row.
 * tokens     [batch] int64, out: argmax index (first maximum; NaN counts as
 *            the largest value, as torch.argmax does; -0.0 == +0.0)
 * status     [batch] uint8, out: PSB_SELECT_* bits
 * ctas_per_row  0 = chosen by the library, else 1..8 CTAs (one thread-block
 *            cluster) per row.
 * A row whose ``remaining`` is <= 0 on entry keeps it, gets
 * PSB_SELECT_DONE | PSB_SELECT_LIMIT and raises PSB_DEVERR_LIMIT.
 * Launched with programmatic dependent launch: a kernel that consumes
 * ``tokens`` must wait (griddepcontrol.wait) before reading them.
 */
int psb_select_tokens(const void* logits, int64_t row_stride, int32_t batch, int32_t vocab, int32_t dtype,
                      const int64_t* eos_ids, int32_t num_eos, int32_t* remaining, int64_t* tokens, uint8_t* status,
                      int32_t ctas_per_row, int32_t* error_flag, psb_stream_t stream);

/*
 * pack_step: GPU-side ragged-batch packer for one engine step.
 *
 * Inputs (device): for each of ``batch`` scheduled requests, ``req_rows[b]``
 * (its row in the device-resident block-table store ``table_store``
 * [store_rows, store_width] int32), ``starts[b]`` (position of its first new
 * token) and ``query_lens[b]`` (new tokens this step: 1 for decode, the prompt
 * length for prefill).  Outputs (device):
 *     cu_seqlens   [batch + 1] int32   exclusive prefix sum of query_lens
 *     context_lens [batch]     int32   starts + query_lens  (= position + 1 for decode)
 *     slot_mapping [total]     int64   table[pos / BS] * BS + pos % BS per new token
 *     positions    [total]     int64   absolute position of every new token (RoPE input)
 *     block_tables [batch, out_width] int32  the requests' table rows, zero padded
 * ``total`` must equal sum(query_lens) (the host knows it from the step plan).
 * Replaces the reference's host-side metadata build
 * (pagedserve/attention/triton_paged_decode.py:134-154) and the per-token
 * slot arithmetic of write_token (pagedserve/engine/paged_kv_cache.py:187-192).
 */
int psb_pack_step(const int32_t* table_store, int64_t store_width, int32_t store_rows, const int32_t* req_rows,
                  const int32_t* starts, const int32_t* query_lens, int32_t batch, int32_t total, int32_t block_size,
                  int32_t* cu_seqlens, int32_t* context_lens, int64_t* slot_mapping, int64_t* positions,
                  int32_t* block_tables, int32_t out_width, int32_t* error_flag, psb_stream_t stream);

/*
 * add_rms_norm: a Qwen2 decoder layer's residual add fused with RMSNorm.
 *
 * Replaces ``residual + x`` followed by Qwen2RMSNorm (transformers' module,
 * called by the reference's model runner at pagedserve/model/engine.py:577-598
 * for decode and :628-648 for prefill).  With ``residual`` non-null, for every
 * row: residual = round(residual + x) (in place), out = RMSNorm(residual);
 * with ``residual`` null, out = RMSNorm(x).  RMSNorm(r) = round(weight *
 * round(r * rsqrt(mean(r^2) + eps))), the mean over ``hidden`` in fp32.
 * x, residual, out are [rows, hidden] with row strides in elements and unit
 * element stride; weight is [hidden]; all of ``dtype``.
 */
int psb_add_rms_norm(const void* x, int64_t x_stride, void* residual, int64_t residual_stride, const void* weight,
                     void* out, int64_t out_stride, int32_t rows, int32_t hidden, float eps, int32_t dtype,
                     psb_stream_t stream);

/*
 * silu_and_mul: the Qwen2 MLP's activation, act_fn(gate_proj(x)) * up_proj(x)
 * (transformers' Qwen2MLP, called at pagedserve/model/engine.py:595 and :645),
 * over a fused [rows, 2 * intermediate] gate|up projection:
 *     out[r, j] = round(round(silu(gate_up[r, j])) * gate_up[r, intermediate + j])
 * silu evaluated in fp32.  Row strides in elements, unit element stride.
 */
int psb_silu_and_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride, int32_t rows,
                     int32_t intermediate, int32_t dtype, psb_stream_t stream);

/*
 * bounded_wait_check: a self-test with no counterpart in the reference.  One
 * warp waits, with the same bounded wait the library's kernels use, on a
 * barrier that nothing completes; after the wall-clock bound (2 s) it gives
 * up, ORs PSB_DEVERR_TIMEOUT (16) into *error_flag and returns.  A host uses
 * it to see that a wait that cannot finish ends with a status on its stream
 * rather than a hang, and that the device stays usable afterwards.
 */
int psb_bounded_wait_check(int32_t* error_flag, psb_stream_t stream);

/* Number of SMs of the current device (for callers sizing persistent grids). */
int psb_device_sm_count(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* PAGEDSERVE_B200_H_ */
