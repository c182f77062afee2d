/*
 * unicache_b200 -- C ABI of the B200 (sm_100a) physical-engine hot path of
 * UniCache (Superone77/UniCache): KIVI quantize/pack, dequantize, packed-KV
 * decode attention, LSE merge, H2O scoring/selection/compaction and dense-cache
 * compaction.
 *
 * Conventions
 *  - Every pointer argument named *_dev is device memory; sizes and strides are
 *    in elements unless the name says bytes.  No entry point allocates memory;
 *    workspaces are passed in.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Return value: UCB_OK (0) or a negative UCB_ERR_* code; ucb_last_error()
 *    returns the message of the last failure on the calling thread.
 *  - Layout "b200" of a packed KIVI segment (per layer, per sequence):
 *        key_code    int32 [H, T/fk, D]   (uint8 [H, T, D] for 8-bit)
 *        key_scale   stat  [H, T/G, D]    key_minimum same
 *        value_code  int32 [H, T, D/fv]   (uint8 [H, T, D] for 8-bit)
 *        value_scale stat  [H, T, D/G]    value_minimum same
 *    with f = 32/bits codes per word, code i of a word in bits [i*b, i*b+b).
 *    It is the reference layout of unicache/storage/physical.py:228-332 with its
 *    first two axes swapped; the int32 words are identical.
 */
#ifndef UNICACHE_B200_H
#define UNICACHE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define UCB_API __attribute__((visibility("default")))
#else
#define UCB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define UCB_OK 0
#define UCB_ERR_INVALID (-1)     /* bad argument: shape, size, alignment    */
#define UCB_ERR_UNSUPPORTED (-2) /* valid request this library does not do  */
#define UCB_ERR_CUDA (-3)        /* CUDA runtime / launch failure           */
#define UCB_ERR_DEVICE (-4)      /* a kernel raised its device error flag   */

#define UCB_BF16 0
#define UCB_F16 1
#define UCB_F32 2

/* Message of the last failed call on this thread ("" if none). */
UCB_API const char* ucb_last_error(void);

/* ABI version (major*100 + minor). */
UCB_API int ucb_version(void);

/* Read and clear the device error word of the current device.  *flags gets the
 * bits kernels set instead of trapping (1 = a bounded wait timed out,
 * 2 = an invalid descriptor was met).  Synchronises `stream`. */
UCB_API int ucb_device_status(unsigned int* flags, void* stream);

/* ------------------------------------------------------------------ KIVI pack
 * Replaces the quantize-and-pack step of PackedKIVICache.from_dense
 * (unicache/storage/physical.py:291-304 -> _quantize_grouped :139-175 and
 * _pack_codes :66-85; on CUDA the KIVI Triton packer, kivi_cuda.py:157-190).
 * Bit-exact with the reference CPU path: per group mn/mx in fp32,
 * scale = max((mx-mn)/(2^b-1), FLT_EPSILON), code = clamp(rint((x-mn)/scale)),
 * scale and minimum stored in the input dtype.
 *
 * x_dev: [tokens, heads, head_dim] with strides (stride_token, stride_head, 1).
 * Key: groups of group_size consecutive tokens per (head, channel);
 *      tokens % group_size == 0.  Outputs in the b200 layout above.
 * Value: groups of group_size consecutive channels per (token, head);
 *      head_dim % group_size == 0.
 * bits in {2,4,8}; group_size % (32/bits) == 0 for 2/4-bit keys;
 * head_dim in {64, 128}. */
UCB_API int ucb_kivi_pack_key(const void* x_dev, int dtype, int64_t tokens, int64_t heads, int64_t head_dim,
                      int64_t stride_token, int64_t stride_head, int bits, int group_size,
                      void* codes_dev, void* scale_dev, void* minimum_dev, void* stream);
UCB_API int ucb_kivi_pack_value(const void* x_dev, int dtype, int64_t tokens, int64_t heads, int64_t head_dim,
                        int64_t stride_token, int64_t stride_head, int bits, int group_size,
                        void* codes_dev, void* scale_dev, void* minimum_dev, void* stream);

/* Keys and values of one segment in ONE launch (the whole pack step of
 * PackedKIVICache.from_dense, unicache/storage/physical.py:291-304), with
 * results identical to ucb_kivi_pack_key + ucb_kivi_pack_value on the same
 * inputs.  Built for dtype UCB_BF16, head_dim 128 and group_size 32 with
 * 16-byte-aligned value rows; any other case returns UCB_ERR_UNSUPPORTED and
 * the caller uses the two separate entries.  Key and value inputs may have
 * different strides; both are [tokens, heads, 128]. */
UCB_API int ucb_kivi_pack_kv(const void* key_dev, const void* value_dev, int dtype, int64_t tokens, int64_t heads,
                             int64_t head_dim, int64_t key_stride_token, int64_t key_stride_head,
                             int64_t value_stride_token, int64_t value_stride_head, int k_bits, int v_bits,
                             int group_size, void* key_codes_dev, void* key_scale_dev, void* key_minimum_dev,
                             void* value_codes_dev, void* value_scale_dev, void* value_minimum_dev, void* stream);

/* Batched ucb_kivi_pack_kv: one launch packs every job of a device table of
 * ucb_kivi_pack_job_bytes() bytes each (no counterpart in the reference,
 * which packs one segment per call).  A job is, in order: the key side
 * {input, token stride, head stride (int64, elements), codes, scale, minimum}
 * and the value side in the same form, then int32 tokens, key_blocks =
 * ceil(tokens/32 * heads / 2), blocks = key_blocks + ceil(tokens * heads *
 * 128/32 / 256), and one int32 of padding.  Every job satisfies the
 * conditions of ucb_kivi_pack_kv (bf16, head_dim 128, group 32, tokens a
 * multiple of 32, 16-byte-aligned value rows) with the same bits and heads;
 * max_blocks is the largest job's `blocks`.  Validation of the table's
 * contents is the caller's (the Python wrapper builds it from checked
 * tensors). */
UCB_API int64_t ucb_kivi_pack_job_bytes(void);
UCB_API int ucb_kivi_pack_kv_batched(const void* jobs_dev, int num_jobs, int max_blocks, int64_t heads, int k_bits,
                                     int v_bits, int group_size, void* stream);

/* ------------------------------------------------------------------ KIVI dequantize
 * Replaces PackedKIVICache.dequantize (physical.py:379-423 -> _dequantize_grouped
 * :178-201) and dequantize_kivi_chunk (unicache/storage/kivi_cuda.py:58-93 ->
 * kivi_triton.py:690-770).  Bit-exact: out = round_dtype(fp32(code*scale) + minimum).
 * Dequantizes quantized tokens [token_begin, token_end) of one segment into
 * out_dev rows [0, token_end-token_begin) with strides (out_stride_token,
 * out_stride_head, 1); out_dtype may differ from stat_dtype. */
UCB_API int ucb_kivi_dequant_key(const void* codes_dev, const void* scale_dev, const void* minimum_dev,
                         int stat_dtype, int64_t quantized_tokens, int64_t heads, int64_t head_dim,
                         int bits, int group_size, int64_t token_begin, int64_t token_end,
                         void* out_dev, int out_dtype, int64_t out_stride_token,
                         int64_t out_stride_head, void* stream);
UCB_API int ucb_kivi_dequant_value(const void* codes_dev, const void* scale_dev, const void* minimum_dev,
                           int stat_dtype, int64_t quantized_tokens, int64_t heads, int64_t head_dim,
                           int bits, int group_size, int64_t token_begin, int64_t token_end,
                           void* out_dev, int out_dtype, int64_t out_stride_token,
                           int64_t out_stride_head, void* stream);

/* ------------------------------------------------------------------ fake quantization
 * Replaces asymmetric_fake_quant / kivi_fake_quant_key / kivi_fake_quant_value
 * (unicache/operators/builtin.py:31-65).  The tensor is viewed as
 * [outer, length, inner] (contiguous) and quantized in groups of group_size
 * along `length` (a partial last group allowed); scale = max(mx-mn, eps)/(2^b-1).
 * Bit-exact. bits in {2,3,4,8}. out_dev may equal x_dev. */
UCB_API int ucb_fake_quant(const void* x_dev, void* out_dev, int dtype, int64_t outer, int64_t length,
                   int64_t inner, int bits, int group_size, void* stream);

/* ------------------------------------------------------------------ decode attention
 * Replaces single-token attention over a sequence's [dense ‖ physical segments]:
 * packed_kivi_attention_parts + torch softmax + apply_value (kivi_cuda.py:238-329,
 * adapters/bagel.py:1201-1297), packed_kivi_quantized_attention_summary
 * (kivi_cuda.py:96-120) for q_len == 1, and _run_fused_h2o_attention
 * (bagel.py:1860-1901) without its per-step torch.cat.
 *
 * A decode batch is a set of (sequence, kv head) pairs; each pair owns spans:
 *  kind 0 (packed KIVI):  key_code..value_minimum point at this head's slice of a
 *                         b200-layout segment; `tokens` quantized tokens.
 *  kind 1 (dense):        key/value rows of `tokens` tokens for this head,
 *                         row i at key + i*key_stride (elements, bf16).
 * Spans are cut into units (64 packed or 8 dense tokens) numbered in span order
 * (spans sorted by pair; span.unit_begin = its first unit).  CTA i processes
 * units [ctas[i].unit_begin, ctas[i].unit_end), which touch pairs
 * [pair_begin, pair_begin + num_pairs) (at most 4); its warp w processes units
 * [warp_bounds[i*(W+1) + w], warp_bounds[i*(W+1) + w + 1]) where W comes from
 * ucb_decode_config, and each warp range may cross at most one segment
 * boundary (a change of pair or of span kind).  A warp writes the softmax state
 * (max, sum, unnormalised rows) of each segment it processed into a state slot
 * of ucb_decode_partial_bytes(head_dim) bytes: warp_slots_dev[2*(i*W + w)] for
 * its first segment when it crosses a boundary, warp_slots_dev[2*(i*W + w) + 1]
 * for its last segment (-1 where the warp has none).  The slots of pair p are
 * [pair.partial_begin, pair.partial_begin + pair.partial_count).  A merge
 * kernel launched after the decode grid on the same stream folds each pair's
 * states into out_dev [seq, q_head, :] (bf16) and
 * lse_dev [seq, q_head] (natural-log LSE, fp32; may be NULL).
 * Workspace: partials_dev >= ucb_decode_partial_bytes(head_dim) * (number of
 * slots) bytes; every slot the merge reads is written by the same call, so
 * nothing needs zeroing.  Calls sharing a workspace must not overlap. */
typedef struct ucb_span {
  const void* key_code;      /* packed: int32/uint8 codes; dense: key rows    */
  const void* key_scale;     /* packed: key scales; dense: NULL, or a device
                                int32 live length (a growing decode suffix:
                                the decode kernel reads min(tokens, *it)
                                rows, so one plan sized for the capacity
                                serves every step)                            */
  const void* key_minimum;   /* packed only                                   */
  const void* value_code;    /* packed: codes; dense: value rows              */
  const void* value_scale;   /* packed only                                   */
  const void* value_minimum; /* packed only                                   */
  int64_t key_stride;        /* dense only: elements between key rows         */
  int64_t value_stride;      /* dense only                                    */
  int32_t kind;              /* 0 packed, 1 dense                             */
  int32_t tokens;
  int32_t pair;              /* owning (sequence, kv head) pair               */
  int32_t unit_begin;        /* first unit of this span                       */
} ucb_span;

typedef struct ucb_decode_cta {
  int32_t unit_begin;
  int32_t unit_end;
  int32_t span_begin;        /* span containing unit_begin                    */
  int32_t pair_begin;
  int32_t num_pairs;         /* 1..4                                          */
  int32_t reserved[3];       /* [0]: span_end, one past the last span (<= span_begin + 16) */
} ucb_decode_cta;

typedef struct ucb_decode_pair {
  int32_t seq;
  int32_t kv_head;
  int32_t partial_begin;
  int32_t partial_count;     /* warp-state slots of this pair                 */
  int32_t cta_first;         /* first CTA touching this pair (informational)  */
  int32_t reserved[3];
} ucb_decode_pair;

UCB_API int64_t ucb_decode_partial_bytes(int head_dim);

/* query_dev: bf16 rows [seq, q_head, head_dim], row (seq, h) at
 * query_dev + seq*query_stride + h*head_dim.  out likewise with out_stride.
 * All packed spans of one call share (k_bits, v_bits, group_size, stat_dtype).
 * softmax_scale: multiplier of q.k (1/sqrt(head_dim) in the reference). */
UCB_API int ucb_decode_attention(const void* query_dev, int64_t query_stride, int num_q_heads, int num_kv_heads,
                         int head_dim, const ucb_span* spans_dev, int num_spans, const ucb_decode_cta* ctas_dev,
                         int num_ctas, const int32_t* warp_bounds_dev, const ucb_decode_pair* pairs_dev,
                         int num_pairs, int k_bits,
                         int v_bits, int group_size, int stat_dtype, float softmax_scale,
                         void* partials_dev, const int32_t* warp_slots_dev, void* out_dev, int64_t out_stride,
                         float* lse_dev, void* stream);

/* Allocation-free variant of ucb_decode_attention; no counterpart in the
 * reference.  For callers that may not allocate device memory when they
 * decode (an engine that owns the whole HBM pool, a host that forbids library
 * allocations): the warp-state slots come from one static device array of
 * 2,129,920 bytes that the library holds on every GPU it is loaded on until
 * exit, so the plan may use at most 512 slots (num_partials = sum of
 * partial_count); larger plans get UCB_ERR_INVALID.  Every slot index in
 * warp_slots_dev and every pair's [partial_begin, partial_begin +
 * partial_count) must lie below num_partials: the kernels check each index
 * against it, and one that does not is skipped and sets flag 2 (an invalid
 * descriptor, read with ucb_device_status) instead of writing past the array.  The caller
 * still passes the plan tables, the query and the outputs.  It calls no cudaMalloc or
 * cudaFree.  The first call on a device looks up the array's address (set-up);
 * make that call before any stream capture.  Every call shares the one array
 * (each slot it reads is written earlier in the same call, so nothing needs
 * clearing): calls that overlap on the GPU (other streams, other host
 * threads) race. */
UCB_API int ucb_decode_attention_noalloc(const void* query_dev, int64_t query_stride, int num_q_heads,
                         int num_kv_heads, int head_dim, const ucb_span* spans_dev, int num_spans,
                         const ucb_decode_cta* ctas_dev, int num_ctas, const int32_t* warp_bounds_dev,
                         const ucb_decode_pair* pairs_dev, int num_pairs, const int32_t* warp_slots_dev,
                         int num_partials, int k_bits, int v_bits, int group_size, int stat_dtype,
                         float softmax_scale, void* out_dev, int64_t out_stride, float* lse_dev, void* stream);

/* Diagnostics: when trace_dev (device memory, 32 uint64 per CTA) is not
 * NULL, later ucb_decode_attention calls record per CTA word 0 = start,
 * word 4 = SM id, word 6 + w = the time warp w finished (state written) and
 * word 18 + w = the time warp w spent waiting for its copies (global timer,
 * ns).  NULL switches it off. */
UCB_API int ucb_decode_set_trace(void* trace_dev);

/* Launch shape of ucb_decode_attention on the current device: CTAs that run at
 * once (one per SM) and warps per CTA for the given packed configuration. */
UCB_API int ucb_decode_config(int k_bits, int v_bits, int group_size, int stat_dtype, int* ctas,
                              int* warps_per_cta);

/* ------------------------------------------------------------------ long-query attention
 * Replaces the q_len > 1 branch of the fused mixed physical attention
 * (unicache/adapters/bagel.py:1598-1858: dequantized workspace, then
 * flash_attn_func(..., causal=False) at :1796-1801) for all KV heads at once,
 * on the tcgen05 tensor cores.  Per KV head h (non-causal):
 *   out[h, m, :] = softmax(q[h, m, :] . k[h, :n_tokens, :]^T * softmax_scale) v
 *   lse[h, m]    = natural-log log-sum-exp of the scaled logits (may be NULL)
 * q_dev bf16 [heads, m_rows, 128] (the query rows of one KV head: (position,
 * head-in-group) pairs), k_dev bf16 [heads, n_padded, 128], vt_dev bf16
 * [heads, 128, n_padded] (V transposed), out_dev bf16 [heads, m_rows, 128],
 * lse_dev fp32 [heads, m_rows].  n_padded >= n_tokens, a multiple of 8; key
 * and value padding tokens must be finite (zeros).  Operands 16-byte aligned. */
UCB_API int ucb_prefill_attention(const void* q_dev, const void* k_dev, const void* vt_dev, int heads, int m_rows,
                                  int n_tokens, int n_padded, float softmax_scale, void* out_dev, float* lse_dev,
                                  void* stream);

/* Batched variant: one launch over several problems (samples) that share the
 * tensors q_dev [heads, m_rows, 128], k_dev [heads, n_padded, 128],
 * vt_dev [heads, 128, n_padded], out_dev, lse_dev.  items_dev: device array of
 * num_items ucb_prefill_item records, one per CTA; CTA i computes query rows
 * [q_row0, q_row0 + q_rows) (q_rows <= 256) of KV head `head` against keys
 * [k_row0, k_row0 + n_tokens) of that head.  k_row0 must be a multiple of 64;
 * key rows k_row0 + n_tokens .. k_row0 + 128*ceil(n_tokens/128) - 1 that lie
 * inside n_padded must be finite (zeros or another problem's keys); rows past
 * n_padded read as zeros.  Query rows q_row0 .. q_row0 + 255 must exist.
 * Replaces the single flash_attn_varlen_func(causal=False) call of
 * apply_static_physical_attention_batch (unicache/adapters/bagel.py:773-980)
 * for query blocks. */
typedef struct ucb_prefill_item {
  int32_t head, q_row0, q_rows, k_row0, n_tokens;
  int32_t mode; /* 0: write out/lse; 1: partial (see ucb_prefill_attention_items); 2: merge */
  int32_t slot; /* partial slot and flag index for modes 1 and 2 */
  int32_t reserved;
} ucb_prefill_item;

UCB_API int ucb_prefill_attention_batched(const void* q_dev, const void* k_dev, const void* vt_dev, int heads,
                                          int m_rows, int n_padded, const void* items_dev, int num_items,
                                          float softmax_scale, void* out_dev, float* lse_dev, void* stream);

/* Batched variant whose items may split a row block's keys in two, to fill
 * every SM when a problem has fewer row blocks than SMs (no counterpart in
 * the reference, whose varlen FlashAttention call schedules itself).  The
 * mode-1 item (keys [k_row0, k_row0 + n_tokens) of the second part) writes
 * its normalised fp32 rows and log2 LSE to partials_dev slot `slot`
 * (ucb_prefill_partial_bytes() each) and then adds 1 to flags_dev[slot]
 * (making it odd); the mode-2 item of the same rows (the first part) waits
 * for the flag to be odd (bounded: on expiry it sets the device error word),
 * merges the two results by LSE into out/lse and adds 1 again.  Both items add
 * exactly once per launch, a timed-out one included, so flags_dev must be even
 * (e.g. zero) before the first launch and is even again after every launch,
 * and a partial that lands late in a failed launch is never mistaken for the
 * next launch's.  Mode-2 items must be
 * fewer than the SMs, so that their partners always find an SM; list them
 * first so they start first.  partials_dev and flags_dev may be NULL when no
 * item uses modes 1 or 2. */
UCB_API int ucb_prefill_attention_items(const void* q_dev, const void* k_dev, const void* vt_dev, int heads,
                                        int m_rows, int n_padded, const void* items_dev, int num_items,
                                        float softmax_scale, void* out_dev, float* lse_dev, float* partials_dev,
                                        unsigned int* flags_dev, void* stream);
UCB_API int64_t ucb_prefill_partial_bytes(void);

/* Long-query attention that reads the physical segments in place (replaces
 * the bf16 workspace that unicache/adapters/bagel.py:1410-1450 assembles and
 * the dequantize + flash_attn_func(causal=False) calls of bagel.py:1598-1858
 * and :773-980).  q_dev and out_dev: bf16 [positions, num_q_heads, 128] in the
 * caller's own layout; lse_dev: fp32 [num_q_heads, positions] (natural log).
 * The query rows of KV head h are the (position, head-in-group) pairs: row m
 * of an item is position pos0 + m / grp and query head h * grp + m % grp
 * (grp = num_q_heads / num_kv_heads).  Each item (one CTA) covers rows
 * [q_row0, q_row0 + q_rows) (<= 256) of KV head `head` against tokens
 * [k_row0, k_row0 + n_tokens) of the concatenation of spans
 * spans_dev[span_begin .. span_begin + span_count): span s holds `tokens`
 * tokens starting at token `unit_begin` of that concatenation (the spans of
 * an item are ordered and contiguous).  A dense span (kind 1) is bf16 rows of
 * this KV head: row t at key_code + t*key_stride (value_code likewise), rows
 * 16-byte aligned.  A packed span (kind 0) is one KV head's b200-layout KIVI
 * tensors (key codes [T/f, 128], key statistics [T/G, 128], value codes
 * [T, 128/f], value statistics [T, 128/G], bf16 statistics), restored inside
 * the kernel as code * scale + minimum with one rounding to bf16 directly
 * into the tensor-core operand tiles in shared memory.  All packed spans of a
 * call share (k_bits in {2,4}, v_bits in {2,4}, group_size in {32,64,128}).
 * mode / slot: as for ucb_prefill_attention_items (key splits need
 * partials_dev and flags_dev). */
typedef struct ucb_lq_item {
  int32_t head;
  int32_t q_row0;
  int32_t q_rows;
  int32_t k_row0;
  int32_t n_tokens;
  int32_t mode;
  int32_t slot;
  int32_t span_begin;
  int32_t span_count;
  int32_t pos0;              /* first query position of the item's sample     */
  int32_t reserved[2];
} ucb_lq_item;

UCB_API int ucb_long_query_attention(const void* q_dev, int positions, int num_q_heads, int num_kv_heads,
                                     const void* items_dev, int num_items, const ucb_span* spans_dev, int num_spans,
                                     int k_bits, int v_bits, int group_size, float softmax_scale, void* out_dev,
                                     float* lse_dev, float* partials_dev, unsigned int* flags_dev, void* stream);

/* Staging job of a staged long-query launch: one key space (the keys of one
 * KV head of one sample, i.e. the span list its items read) gathered into
 * workspace rows [ws_row0, ws_row0 + rows) of KV head `head`; tokens
 * [tokens, rows) are written as zeros.  ws_row0 and rows are multiples of
 * 128, rows >= tokens. */
typedef struct ucb_lq_stage_job {
  int32_t head;
  int32_t span_begin;
  int32_t span_count;
  int32_t tokens;
  int32_t ws_row0;
  int32_t rows;
  int32_t reserved[2];
} ucb_lq_stage_job;

/* Gathers every job's key space into a bf16 workspace: k_ws [heads, ws_rows,
 * 128] (token rows) and vt_ws [heads, 128, ws_rows] (values transposed).
 * Dense spans are copied; packed spans are restored as code * scale +
 * minimum with one rounding to bf16, the values ucb_long_query_attention
 * restores in its operand tiles.  Grid: max_chunks x num_jobs blocks of 32
 * tokens (max_chunks * 32 >= the largest `rows`; ws_rows a multiple of 128). */
/* Diagnostics: when trace_dev (device memory, 32 uint64 per CTA) is not
 * NULL, later long-query and prefill launches record per CTA (global timer,
 * ns): word 0 = kernel entry, 1 = set-up done, 2 = SM id, 3 = exit, 4 = items
 * run, and for its first 12 items i: word 6 + 2i = the softmax warps start
 * the item (its query rows loaded), 7 + 2i = the item's results written;
 * word 30 = the MMA thread's total wait for K/V tiles, 31 = its total wait
 * for the softmax warps' P tiles (ns).  NULL switches it off. */
UCB_API int ucb_prefill_set_trace(void* trace_dev);

UCB_API int ucb_long_query_stage(const ucb_span* spans_dev, int num_spans, const void* jobs_dev, int num_jobs,
                                 int max_chunks, int k_bits, int v_bits, int group_size, void* k_ws_dev,
                                 void* vt_ws_dev, int64_t ws_rows, void* stream);

/* ucb_long_query_attention with its keys and values staged first
 * (ucb_long_query_stage, then the tensor-core kernel streaming both by TMA):
 * same arguments and results, plus the staging jobs and workspace; each
 * item's key space starts at workspace row reserved[0] of the item (the
 * ws_row0 of its job), so items keep k_row0 relative to their key space.
 * Each packed tile is restored once per launch instead of once per row block.
 *
 * cta_items_dev NULL: one CTA per item, as ucb_long_query_attention.
 * Otherwise a persistent launch of num_ctas CTAs: CTA b runs items
 * [cta_items_dev[b], cta_items_dev[b + 1]) one after the other (int32,
 * num_ctas + 1 entries, non-decreasing, ending at num_items), so work can be
 * split evenly over the SMs in (row block, key tile) units.  A row block cut
 * into pieces runs its first piece as a merge item (mode 2, listed last in
 * its CTA) and the others as partial items (mode 1, each the first item of
 * its CTA) in consecutive slots [slot, slot + reserved[1]) of the merge item
 * (reserved[1] >= 1); every item settles its flags once per launch as for
 * ucb_prefill_attention_items.  num_ctas must not exceed the number of SMs
 * that can hold one CTA each (merge items wait for partials). */
UCB_API int ucb_long_query_attention_staged(const void* q_dev, int positions, int num_q_heads, int num_kv_heads,
                                            const void* items_dev, int num_items, const int32_t* cta_items_dev,
                                            int num_ctas, const ucb_span* spans_dev, int num_spans,
                                            const void* jobs_dev, int num_jobs, int max_chunks, int k_bits,
                                            int v_bits, int group_size, float softmax_scale, void* k_ws_dev,
                                            void* vt_ws_dev, int64_t ws_rows, void* out_dev, float* lse_dev,
                                            float* partials_dev, unsigned int* flags_dev, void* stream);

/* ---- element-wise steps of the configuration-5 decoder (the workload that
 * drives the decode path at Qwen2-7B shape; no counterpart in the path's
 * reference code).  All bf16, contiguous rows.
 * ucb_rms_norm: out[r] = bf16(bf16(x[r] * rsqrt(mean(x[r]^2) + eps)) * w).
 * ucb_qkv_rope_append: qkv [batch, (hq + 2*hkv) * head_dim] (query, key, value
 * heads); slot = *length - 1 (device int32), position = prompt + slot; the
 * query heads, rotated (half-split rotary embedding with angles position *
 * inv_freq[i], fp32 inv_freq [head_dim/2]), go to q_out [batch, hq,
 * head_dim]; the rotated key heads and the value heads are written to row
 * `slot` of suffix_k / suffix_v [batch, capacity, hkv, head_dim].  A slot
 * outside [0, capacity) appends nothing and sets device error flag 2.
 * ucb_silu_mul: gate_up [rows, 2*ffn] -> out [rows, ffn] =
 * bf16(bf16(silu(gate)) * up). */
UCB_API int ucb_rms_norm(const void* x_dev, const void* weight_dev, int rows, int hidden, float eps, void* out_dev,
                         void* stream);
UCB_API int ucb_qkv_rope_append(const void* qkv_dev, int batch, int hq, int hkv, int head_dim,
                                const int32_t* length_dev, int prompt, const float* inv_freq_dev, void* q_out_dev,
                                void* suffix_k_dev, void* suffix_v_dev, int capacity, void* stream);
UCB_API int ucb_silu_mul(const void* gate_up_dev, int rows, int ffn, void* out_dev, void* stream);

/* ---- sequence-split merge over NVLink peer memory (no counterpart in the
 * reference, which decodes one sequence on one device).  Each rank allocates
 * one exchange buffer of ucb_peer_buffer_bytes(rows) bytes
 * (ucb_peer_buffer_alloc: cudaMalloc'd, zeroed, with a 64-byte CUDA IPC
 * handle), shares the handle with its peers (for example through the process
 * group) and maps theirs with ucb_peer_buffer_open.  ucb_split_merge_peer then
 * replaces the all-gather + ucb_lse_merge of a split decode step: rank `rank`
 * sends its summary (out_local [rows, 128] bf16, lse_local [rows] fp32,
 * natural log; rows = B * Hq) into every peer's buffer as 8-byte peer stores
 * that each carry 4 data bytes and the step's epoch, reads the peers' words
 * from its own buffer as their epochs arrive (at most 1 s; on expiry it sets
 * the device error word and leaves out/lse unwritten) and merges the world
 * summaries in rank order as ucb_lse_merge does into out/lse, which must not
 * alias out_local/lse_local (UCB_ERR_INVALID).
 * bufs: host array of `world` buffer addresses as mapped in this process
 * (bufs[rank] is the local one); world <= 8.  Every rank must make the same
 * sequence of calls; one call per buffer at a time. */
UCB_API int64_t ucb_peer_buffer_bytes(int64_t rows);
UCB_API int ucb_peer_buffer_alloc(int64_t bytes, void** ptr, void* handle_out);
UCB_API int ucb_peer_buffer_open(const void* handle, void** ptr);
UCB_API int ucb_peer_buffer_close(void* ptr);
UCB_API int ucb_peer_buffer_free(void* ptr);
UCB_API int ucb_split_merge_peer(int rank, int world, void* const* bufs, const void* out_local,
                                 const float* lse_local, int64_t rows, int head_dim, void* out, float* lse,
                                 void* stream);

/* ------------------------------------------------------------------ LSE merge
 * Replaces merge_attention_summaries (unicache/adapters/bagel.py:57-72).
 * n summaries, summary i: out_ptrs[i] -> [rows, heads, head_dim] (dtype),
 * lse_ptrs[i] -> fp32 [heads, rows].  Pointer arrays are HOST arrays.
 * Writes out_dev [rows, heads, head_dim] (dtype) and lse_out_dev fp32
 * [heads, rows]. n <= 64. */
UCB_API int ucb_lse_merge(int n, const void* const* out_ptrs, const float* const* lse_ptrs, int dtype,
                  int64_t rows, int64_t heads, int64_t head_dim, void* out_dev, float* lse_out_dev,
                  void* stream);

/* ------------------------------------------------------------------ H2O
 * Per-KV-head heavy-hitter selection (GQAH2OCache.from_dense / trim,
 * unicache/storage/physical.py:508-532 and :624-649): for each of `heads` rows
 * of scores_dev (fp32, row stride score_stride), keep the heavy_k largest scores
 * among the first history_end entries (ties: lower index first) in ascending
 * index order, followed by the recent window [tokens-recent, tokens).
 * index_out_dev: int64 [heads, heavy_k + recent]. tokens <= 1<<24. */
UCB_API int ucb_h2o_select(const float* scores_dev, int64_t score_stride, int heads, int64_t tokens,
                   int64_t history_end, int64_t heavy_k, int64_t recent, int64_t* index_out_dev,
                   void* stream);

/* Gather rows by per-head indices (physical.py:533-542 and :650-654):
 * src row (h, i) at src + h*src_stride_head + i*src_stride_token (elements of
 * elem_bytes each row of row_elems), dst [heads, keep, row_elems] contiguous.
 * Used for K/V (row_elems = head_dim), logical ids (int64, row_elems = 1) and
 * scores (fp32, row_elems = 1). */
UCB_API int ucb_gather_rows(const void* src_dev, int64_t src_stride_head, int64_t src_stride_token,
                    int64_t row_elems, int elem_bytes, const int64_t* index_dev, int heads,
                    int64_t keep, void* dst_dev, void* stream);

/* H2O score accumulation from materialised probabilities
 * (physical.py:598-610, unicache/operators/physical.py:63-65):
 * probs_dev fp32/bf16 [q_heads, queries, tokens] -> scores_dev[kv, t] (+)=
 * sum over the kv head's query heads and all queries.  accumulate=0 overwrites. */
UCB_API int ucb_h2o_accumulate_probs(const void* probs_dev, int dtype, int q_heads, int64_t queries,
                             int64_t tokens, int kv_heads, float* scores_dev, int accumulate,
                             void* stream);

/* A packed segment's generic attention parts (kivi_cuda.py:238-329 /
 * physical.py:452-475 of the reference): the caller materialises the softmax.
 * Tokens are the segment's quantized prefix followed by its residual rows.
 * Packed tensors of one KV head start at codes + kv*codes_head_stride
 * (elements of the code dtype: int32 words, uint8 at 8 bits) and
 * stats + kv*stats_head_stride (bf16 statistics); residual row t of head kv
 * is at residual + t*res_token_stride + kv*res_head_stride (bf16, 16-byte
 * aligned rows).  Codes are restored as the reference's dequantize() does
 * (code * scale + minimum in fp32, one rounding to bf16).
 *   logits: query bf16 [queries, q_heads, 128] -> logits fp32
 *           [q_heads, queries, quantized + residual], scaled by softmax_scale.
 *   apply:  probs [q_heads, queries, quantized + residual] (bf16, f16 or f32;
 *           rounded to bf16 as the reference casts them to the value dtype)
 *           -> out bf16 [q_heads, queries, 128]. */
UCB_API int ucb_kivi_attention_logits(const void* query_dev, int64_t queries, int q_heads, int kv_heads,
                                      const void* key_code_dev, const void* key_scale_dev,
                                      const void* key_minimum_dev, int64_t codes_head_stride,
                                      int64_t stats_head_stride, const void* residual_key_dev,
                                      int64_t res_token_stride, int64_t res_head_stride, int64_t quantized_tokens,
                                      int64_t residual_tokens, int bits, int group_size, float softmax_scale,
                                      float* logits_dev, void* stream);
UCB_API int ucb_kivi_attention_apply(const void* probs_dev, int probs_dtype, int64_t queries, int q_heads,
                                     int kv_heads, const void* value_code_dev, const void* value_scale_dev,
                                     const void* value_minimum_dev, int64_t codes_head_stride,
                                     int64_t stats_head_stride, const void* residual_value_dev,
                                     int64_t res_token_stride, int64_t res_head_stride, int64_t quantized_tokens,
                                     int64_t residual_tokens, int bits, int group_size, void* out_dev, void* stream);

/* Fused H2O scoring without materialised probabilities (adapters/bagel.py:1845-1856):
 * scores[kv, t] (+)= sum_{g, q} exp(scale * q_{kv*G+g, q} . k_t - lse[kv*G+g, q]).
 * query_dev bf16 [queries, q_heads, head_dim]; key rows bf16, row (t, kv) at
 * key_dev + t*key_stride_token + kv*key_stride_head; lse_dev fp32 [q_heads, queries]
 * (natural log). */
UCB_API int ucb_h2o_scores_from_lse(const void* query_dev, int64_t queries, int q_heads, const void* key_dev,
                            int64_t key_stride_token, int64_t key_stride_head, int64_t tokens,
                            int kv_heads, int head_dim, const float* lse_dev, float softmax_scale,
                            float* scores_dev, int accumulate, void* stream);

/* The same reduction (operators/physical.py:51-101 and GQAH2OCache.update_scores,
 * storage/physical.py:598-610, without the [Hq, Lq, T] probabilities) for
 * bf16 (tensor cores, mma.sync) or fp32 (CUDA cores) query and keys of one
 * dtype.  lse_dev NULL: the attention covers exactly these keys and the LSE of
 * every row is computed first into lse_workspace_dev (8-byte aligned,
 * ucb_h2o_scores_workspace_floats(queries, q_heads, tokens) floats: the
 * LSE [q_heads, queries] first, then per-64-token-block partial maxima and
 * sums).  bf16 needs a 16-byte aligned query and 4-byte aligned key rows. */
UCB_API int64_t ucb_h2o_scores_workspace_floats(int64_t queries, int q_heads, int64_t tokens);
UCB_API int ucb_h2o_scores(const void* query_dev, int dtype, int64_t queries, int q_heads, const void* key_dev,
                           int64_t key_stride_token, int64_t key_stride_head, int64_t tokens, int kv_heads,
                           int head_dim, const float* lse_dev, float* lse_workspace_dev, float softmax_scale,
                           float* scores_dev, int accumulate, void* stream);

/* ------------------------------------------------------------------ dense compaction
 * Replaces TensorCacheStorageBackend.compact's per-sample boolean gather
 * (unicache/storage/tensor_backend.py:54-100).  mask_dev uint8 [rows];
 * rows with mask != 0 are copied in order to dst (row_bytes each, 16-byte
 * aligned rows), and to types_out (int64) when types_dev is not NULL.
 * prefix_dev: int64 workspace of rows+1 entries; *kept_host receives the
 * number of kept rows (synchronises `stream`). */
UCB_API int ucb_compact_rows(const void* src_dev, int64_t row_bytes, const uint8_t* mask_dev, int64_t rows,
                     const int64_t* types_dev, void* dst_dev, int64_t* types_out_dev,
                     int64_t* prefix_dev, int64_t* kept_host, void* stream);

/* ------------------------------------------------------------------ self test
 * Checks on the current device that mma.sync f16 consumes fp16 subnormal
 * operands exactly (the decode kernel feeds small integer codes as subnormals).
 * *max_abs_err receives the largest deviation from an fp32 reference. */
UCB_API int ucb_selftest_mma_subnormal(float* max_abs_err, void* stream);

/* ------------------------------------------------------------------ host transfers
 * No counterpart in the reference (its engine copies with torch).  Per-step
 * host <-> device transfers of small buffers (a decode query, its output and
 * LSE) done by a kernel over mapped pinned host memory instead of a DMA copy.
 * ucb_host_device_pointer: device-visible address of pinned host memory
 * (cudaHostGetDevicePointer); UCB_ERR_INVALID when the memory is not mapped.
 * ucb_copy_ranges: one kernel copies n (1..8) ranges, bytes[i] from src[i]
 * to dst[i], all device-visible (device memory or such mapped host
 * addresses) and 16-byte aligned, on `stream`; the pointer and size arrays
 * are host arrays. */
UCB_API int ucb_host_device_pointer(const void* host, void** dev);
UCB_API int ucb_copy_ranges(int n, void* const* dst_dev, const void* const* src_dev, const int64_t* bytes,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* UNICACHE_B200_H */
