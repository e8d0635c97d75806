/*
 * kvb.h -- C ABI of libkvb.so, the B200 (sm_100a) kernels of the quantised
 * decoder-layer hot path of KernelVerse.
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are raw DEVICE pointers to contiguous row-major
 *     buffers; sizes are element counts.  No torch types cross this boundary.
 *   - The caller owns all memory (inputs, outputs and any workspace); entry
 *     points never allocate and never synchronise the host.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); all work is
 *     stream-ordered on it.
 *   - The return value is KVB_OK (0) or a positive KVB_E_* status; the message
 *     for the calling thread's last failure is kvb_last_error().
 *   - Every reference interface an entry point replaces is cited as
 *     path:line inside the KernelVerse tree.
 */
#ifndef KVB_H_
#define KVB_H_

#include <stddef.h>
#include <stdint.h>

#if defined(KVB_BUILD) && defined(__GNUC__)
#define KVB_API __attribute__((visibility("default")))
#else
#define KVB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define KVB_OK 0
#define KVB_E_ARG 1        /* null pointer / bad enum / negative size */
#define KVB_E_SHAPE 2      /* shape outside what the kernel supports */
#define KVB_E_ALIGN 3      /* pointer or stride alignment violated */
#define KVB_E_DTYPE 4      /* unsupported dtype combination */
#define KVB_E_LAUNCH 5     /* CUDA launch / driver error */
#define KVB_E_TIMEOUT 6    /* a bounded device-side wait gave up */
#define KVB_E_WORKSPACE 7  /* workspace missing or too small */
#define KVB_E_DEVICE 8     /* device is not sm_100 */
#define KVB_E_INDEX 9      /* an out-of-range index was skipped on the device */

/* element types */
#define KVB_F32 0
#define KVB_F16 1
#define KVB_BF16 2
#define KVB_I8 3
#define KVB_U8 4
#define KVB_I32 5
#define KVB_I64 6
#define KVB_E4M3 7         /* float8_e4m3fn codes (OCP FP8 E4M3, no inf, max 448) */

/* Message for the last non-zero status returned on this host thread. */
KVB_API const char* kvb_last_error(void);
/* ABI version: bumped on any signature change. */
KVB_API int kvb_abi_version(void);

/*
 * Diagnostics (no reference counterpart).  kvb_device_status synchronises the
 * current device and returns the OR of the library's device status words:
 * bit 0 = a bounded device-side wait gave up (its kernel drained and exited
 * early; outputs of that launch are invalid); bit 1 = a slot or block-table entry out of
 * range was skipped; bit 2 = a prefill indptr range out of range was skipped.  reset != 0
 * clears the words.
 * Returns 0x80000000 if the device itself reports an error.
 */
KVB_API unsigned int kvb_device_status(int reset);
/*
 * kvb_device_status as a status code (no reference counterpart): synchronises the current
 * device and returns KVB_E_TIMEOUT when bit 0 is set, KVB_E_INDEX when bit 1 or 2 is set,
 * KVB_E_LAUNCH when the device reports an error, else KVB_OK; the message is in
 * kvb_last_error().  Entry points never synchronise, so a wait that gives up inside a launch
 * surfaces here, not in the entry point's return value.  reset != 0 clears the words.
 */
KVB_API int kvb_check_device(int reset);
/*
 * Sets the bound of every device-side wait, in nanoseconds of %globaltimer (0 restores the
 * default, 2 s), on the current device (no reference counterpart).  Not stream-ordered: call
 * it while none of the library's kernels run.
 */
KVB_API int kvb_set_wait_limit_ns(uint64_t limit_ns);
/*
 * Test hook of the bounded wait (no reference counterpart): one thread bulk-copies 16 bytes from
 * src16 (device, 16-byte aligned) into shared memory, then waits on an mbarrier on which nothing
 * ever arrives.  The wait gives up after the current limit and sets bit 0 of
 * kvb_device_status; the kernel then drains its copy and returns.  out[3] (device int32):
 * out[0] = the first copied int32, out[1] = 1 if the wait gave up, out[2] = 1 if the copy
 * completed.
 */
KVB_API int kvb_selftest_wait_timeout(const void* src16, int* out, void* stream);
/* out[i] = a[i] / b[i] through the kernels' FMA-corrected division (test hook). */
KVB_API int kvb_selftest_div_rn(const float* a, const float* b, float* out, int64_t n, void* stream);

/* ---------------------------------------------------------------- quantisation */

/* Bytes of workspace kvb_dynamic_scaled_int8_quant needs (a 256-byte-aligned block). */
KVB_API size_t kvb_dynamic_scaled_int8_quant_workspace_size(void);

/*
 * Per-tensor dynamic int8 quantisation.
 * Replaces operators/quantization/dynamic_scaled_int8_quant/dynamic_scaled_int8_quant.py:21-26
 * (constants helpers.py:7-8):
 *   scale = max(float32(dtype(amax|x| / 127)), 1/(448*512));
 *   q = round_half_even(clamp(x / scale, -127, 127)); azp = 0.
 * x: `numel` elements of x_dtype (KVB_F32/F16/BF16).  q: numel int8.  scale: 1 float.
 * azp: 1 int32 (may be NULL).  workspace: >= kvb_dynamic_scaled_int8_quant_workspace_size()
 * bytes of device memory (the running amax); it is re-initialised on every call.
 * Two kernels are launched (amax, then quantise) after a 4-byte memset.
 */
KVB_API int kvb_dynamic_scaled_int8_quant(const void* x, int x_dtype, int64_t numel,
                                  int8_t* q, float* scale, int32_t* azp,
                                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Per-token, per-group dynamic int8 quantisation.
 * Replaces operators/quantization/per_token_group_quant_int8/per_token_group_quant_int8.py:23-32:
 *   scales[t, g] = max(amax|x[t, g*G:(g+1)*G]| / 127, eps)   (float32)
 *   q = clamp(round_half_even(x / scales), -127, 127)
 * x: [tokens, hidden] of x_dtype; hidden % group_size == 0.  q: [tokens, hidden] int8;
 * scales: [tokens, hidden / group_size] float32.  group_size == hidden gives per-token
 * quantisation (the BASELINE first config).
 */
KVB_API int kvb_per_token_group_quant_int8(const void* x, int x_dtype, int64_t tokens, int64_t hidden,
                                   int64_t group_size, float eps, int8_t* q, float* scales,
                                   void* stream);

/*
 * Static-scale int8 quantisation.
 * Replaces operators/quantization/static_scaled_int8_quant/static_scaled_int8_quant.py:28-32
 * (MIN_SCALE at helpers.py:8), float32 arithmetic (the reference's correctness mode):
 *   q = clamp(round_half_even(x / max(scale, 1/(448*512)) + azp), -127, 127).
 * x: `numel` elements of x_dtype (KVB_F32/F16/BF16); scale: 1 float32 and azp: 1 int32 (may
 * be NULL: 0), both in device memory; q: numel int8.  One kernel, no host synchronisation.
 */
KVB_API int kvb_static_scaled_int8_quant(const void* x, int x_dtype, int64_t numel, const float* scale,
                                         const int32_t* azp, int8_t* q, void* stream);

/* ---------------------------------------------------------------- residual add + RMSNorm */

/*
 * out = dtype((s * rsqrt(mean(s^2) + eps)) * w), s = x + residual, all in float32.
 * Replaces operators/normalization/add_rmsnorm/add_rmsnorm.py:24-35 (correctness
 * compute mode, :17-22).  x, residual, out: [rows, hidden] of `dtype`; weight: [hidden].
 */
KVB_API int kvb_add_rmsnorm(const void* x, const void* residual, const void* weight, int dtype,
                    int64_t rows, int64_t hidden, float eps, void* out, void* stream);

/*
 * Fused residual add + RMSNorm + dynamic per-row quantisation (one HBM pass).
 * No single reference operator: composes add_rmsnorm.py:24-35 with the per-row
 * quantisation of the BASELINE second config.
 *   residual_out = dtype(x + residual)                     (may alias `residual`)
 *   y = (s * rsqrt(mean(s^2) + eps)) * w                   (float32)
 *   scales[r] = max(amax|y_r| / Q, 1/(448*512)),  Q = 448 (KVB_E4M3) or 127 (KVB_I8)
 *   codes = e4m3fn(clamp(y / scale, +-448))  or  clamp(round_half_even(y / scale), +-127)
 * residual_out may be NULL (not written).  codes: [rows, hidden] bytes; scales: [rows].
 * Exactness: residual_out is bit-exact.  y is a float32 computation whose sum of squares is
 * reduced in the kernel's own order, so y (and with it the scale and the codes) can differ
 * from a float64- or differently-ordered reference by about one float32 rounding: codes are
 * within one step (one e4m3 ulp, or +-1 for int8) of the reference's, >= 99.9 % of them
 * identical, and scales within a relative 1e-6.  The standalone quantisers
 * (kvb_per_token_group_quant_int8 etc.) take their scale from the input and are bit-exact.
 */
KVB_API int kvb_add_rmsnorm_quant(const void* x, const void* residual, const void* weight, int dtype,
                          int64_t rows, int64_t hidden, float eps, void* residual_out,
                          void* codes, int code_dtype, float* scales, void* stream);

/* ---------------------------------------------------------------- W8A8 int8 GEMM */

/* Bytes of workspace kvb_w8a8_scaled_mm needs (0-sized needs still take a 256-byte block). */
KVB_API size_t kvb_w8a8_workspace_size(int64_t M, int64_t N, int64_t K, int b_layout, int has_azp);

/*
 * W8A8 GEMM on tcgen05 tensor cores (int32 accumulation in TMEM).
 * Replaces operators/gemm/int8_scaled_mm_azp/int8_scaled_mm_azp.py:61-85 (whose float
 * dequantise-then-matmul is computed exactly in integers here) and implements the BASELINE
 * third config:
 *   acc[m, n] = sum_k a[m, k] * B(n, k)                 (exact int32)
 *   acc      -= azp[n] * sum_k a[m, k]                  (when azp != NULL; azp holds integers)
 *   out[m, n] = ((float(acc) * a_scales[m]) * b_scales[n] + azp_adj[n]) + bias[n]
 *             (each term only when its pointer is non-NULL; one float32 rounding per step)
 * out_dtype KVB_BF16 / KVB_F16 / KVB_F32, or KVB_I32 for the raw accumulator (scales unused).
 * a [M, K] int8 row-major.  b_layout 0: b [N, K] (K contiguous); 1: b [K, N] (the reference's
 * layout, transposed into the workspace first).  out [M, ldo] row-major.  K % 16 == 0;
 * a (and b for layout 0) 16-byte aligned.  Workspace: kvb_w8a8_workspace_size() bytes when
 * b_layout == 1 or azp != NULL, else may be NULL.
 */
KVB_API int kvb_w8a8_scaled_mm(const int8_t* a, const int8_t* b, int b_layout, const float* a_scales,
                               const float* b_scales, const void* bias, int bias_dtype, const float* azp,
                               const float* azp_adj, int64_t M, int64_t N, int64_t K, void* out, int out_dtype,
                               int64_t ldo, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Column-sharded tensor-parallel W8A8 GEMM with the all-gather fused into its epilogue
 * (BASELINE fifth config; no reference counterpart -- the reference has no multi-GPU code).
 * Rank `rank` of `world` (<= 8) holds b_shard [N_shard, K] (columns rank*N_shard ... of the
 * full weight), its b_scales_shard / bias_shard, and the replicated a [M, K], a_scales [M].
 * out_ptrs[r] is rank r's output buffer [M, ldo] (ldo >= world * N_shard), mapped into this
 * process (e.g. symmetric memory); every finished tile is stored into all `world` buffers at
 * columns rank*N_shard + n with plain peer stores over NVLink, then fenced at system scope.
 * The caller must order the kernels of all ranks before reading (e.g. a small collective on
 * the same stream after the call).  Same epilogue and exactness as kvb_w8a8_scaled_mm.
 */
KVB_API int kvb_w8a8_scaled_mm_allgather(const int8_t* a, const int8_t* b_shard, const float* a_scales,
                                         const float* b_scales_shard, const void* bias_shard, int bias_dtype,
                                         int64_t M, int64_t N_shard, int64_t K, void* const* out_ptrs, int world,
                                         int rank, int64_t ldo, int out_dtype, void* stream);

/*
 * W8A8 GEMM with a gated-activation epilogue: the gate+up projection of an MLP followed by
 * SwiGLU in one kernel (operators/activation/swiglu/swiglu.py:24-28 and
 * operators/activation/mul_and_silu/mul_and_silu.py:24-29 applied to this GEMM's output).
 * b_nk [N, K] holds the two operand weights with their rows interleaved in blocks of 128:
 * rows [256 j, 256 j + 128) are rows [128 j, 128 j + 128) of the first operand's weight and
 * rows [256 j + 128, 256 j + 256) the same rows of the second's; b_scales and bias [N] follow
 * the same order.  With f = (acc * a_scales[m]) * b_scales[n] + bias[n] rounded to out_dtype
 * (exactly what kvb_w8a8_scaled_mm would store), output column c of row m is
 *   act 1: silu(f_first) * f_second      (SwiGLU: gate first)
 *   act 2: f_first * silu(f_second)      (mul-and-silu: value first)
 * in float32 (silu(x) = x * rcp(1 + e^-x) with the fast exponential: within a few float32
 * ulps), rounded to out_dtype.  out: [M, N / 2] (pitch ldo).
 * N must be a multiple of 256; out_dtype KVB_BF16, KVB_F16 or KVB_F32.
 */
KVB_API int kvb_w8a8_scaled_mm_act(const int8_t* a, const int8_t* b_nk, const float* a_scales, const float* b_scales,
                                   const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K, int act,
                                   void* out, int out_dtype, int64_t ldo, void* stream);

/*
 * kvb_w8a8_scaled_mm_act, column-sharded over `world` ranks with the all-gather fused into the
 * epilogue as in kvb_w8a8_scaled_mm_allgather: rank `rank` holds the interleaved rows of its
 * N_shard / 2 output columns (N_shard a multiple of 256) and stores them at columns
 * rank * N_shard / 2 of every rank's [M, ldo] buffer (ldo >= world * N_shard / 2).  The
 * gathered bytes are half those of gathering the gate+up output.
 */
KVB_API int kvb_w8a8_scaled_mm_act_allgather(const int8_t* a, const int8_t* b_shard, const float* a_scales,
                                             const float* b_scales_shard, const void* bias_shard, int bias_dtype,
                                             int64_t M, int64_t N_shard, int64_t K, int act, void* const* out_ptrs,
                                             int world, int rank, int64_t ldo, int out_dtype, void* stream);

/* ---------------------------------------------------------------- paged KV-cache writes */

/*
 * Replaces operators/kv_cache/paged_kv_cache_update/paged_kv_cache_update.py:21-31:
 * kv_cache_out = copy of kv_cache_in (skipped when kv_cache_in is NULL or equal to
 * kv_cache_out), then for every token i with slot_mapping[i] >= 0, flat slot
 * slot_mapping[i] of kv_cache_out ([num_slots, slot_elems], num_slots = blocks * block_size)
 * receives to_cache[i] ([num_tokens, slot_elems]).  All of `dtype`; slot_mapping is
 * KVB_I32 or KVB_I64.  Slots >= num_slots are skipped and flagged in kvb_device_status.
 */
KVB_API int kvb_paged_kv_cache_update(const void* to_cache, const void* kv_cache_in, void* kv_cache_out,
                                      const void* slot_mapping, int index_dtype, int dtype, int64_t num_tokens,
                                      int64_t num_slots, int64_t slot_elems, void* stream);

/*
 * FP8 paged KV write (BASELINE fourth config; slot placement as paged_kv_cache_update.py:27-30):
 * cache[slot_mapping[i], h, :] = e4m3(clamp(x_new[i, h, :] / head_scales[h], +-448)).
 * x_new [num_tokens, num_heads, head_dim] (x_dtype); cache [num_slots, num_heads, head_dim]
 * e4m3 codes; negative slots are skipped.
 */
KVB_API int kvb_paged_fp8_kv_write(const void* x_new, int x_dtype, void* cache, const void* slot_mapping,
                                   int index_dtype, const float* head_scales, int64_t num_tokens, int64_t num_slots,
                                   int num_heads, int head_dim, void* stream);

/*
 * KV-cache write into [batch, heads, max_seq_len, head_dim] caches.
 * Replaces operators/kv_cache/kv_cache_write/kv_cache_write.py:24-58: k_cache_out / v_cache_out
 * become copies of k_cache_in / v_cache_in (no copy when an input is NULL or equals its output),
 * then k_cache_out[b, h, pos(b, w), :] = key[b, h, w, :] and likewise for V, with
 * pos(b, w) = positions[w] (per_batch == 0, positions [write_len]) or positions[b, w]
 * (per_batch != 0, [batch, write_len]), KVB_I32 or KVB_I64.  A negative position counts from
 * the end as torch indexing does; positions outside [-max_seq_len, max_seq_len) are skipped
 * and flagged in kvb_device_status.  key/value: [batch, heads, write_len, head_dim]; all
 * tensors of `dtype`.  Launches one copy per cache and one scatter kernel.
 */
KVB_API int kvb_kv_cache_write(const void* key, const void* value, const void* k_cache_in, const void* v_cache_in,
                               void* k_cache_out, void* v_cache_out, const void* positions, int index_dtype,
                               int per_batch, int dtype, int64_t batch, int64_t heads, int64_t max_seq_len,
                               int64_t write_len, int64_t head_dim, void* stream);

/* ---------------------------------------------------------------- paged decode attention */

/* Bytes of workspace kvb_paged_attention needs (float32 split-KV partials). */
KVB_API size_t kvb_paged_attention_workspace_size(int batch, int num_q_heads, int head_dim, int max_partitions);

/*
 * The partition size kvb_paged_attention uses for partition_size 0: 512 tokens, halved down to
 * 64 while sequences * ceil(max_seq_len / size) is below two per SM of the current device.
 * A caller sizes the workspace with ceil(max_seq_len / that size) partitions.
 */
KVB_API int kvb_paged_attention_auto_partition(int sequences, int64_t max_seq_len);

/*
 * GQA decode attention over a paged KV cache, split over partitions of the sequence.
 * Replaces operators/attention/paged_attention_v1/paged_attention_v1.py:27-92 and, with the
 * v2 outputs, operators/attention/paged_attention_v2/paged_attention_v2.py:28-175.
 *
 * query [B, Hq, D] (q_dtype); key_cache / value_cache [num_blocks, block_size, Hkv, D] of
 * cache_dtype (KVB_E4M3 with per-KV-head float32 k_scale / v_scale [Hkv], or KVB_F16 /
 * KVB_BF16 with NULL scales): token t of sequence b is row t % block_size of block
 * block_table[b * bt_stride + t / block_size] -- the memory order in which the reference
 * gathers and reshapes its cache (paged_attention_v1.py:64-69).  block_table == NULL means
 * block b holds all of sequence b (dense [B, L, Hkv, D] caches,
 * operators/attention/batched_decode_attention/batched_decode_attention.py:30-52).
 * seq_lens [B] (KVB_I32 / KVB_I64); max_seq_len >= every seq_len (sizes the grid).
 * out[b, h] = softmax(K q * sm_scale) V with q-head h reading KV head h / (Hq / Hkv).
 *
 * k_new / v_new [B, Hkv, D] (new_dtype, optional, e4m3 caches only): each sequence's newest
 * token (position seq_len - 1) is first quantised (e4m3(clamp(x / scale[h]))) and written
 * to its slot, and the attention uses the written codes.
 * partition_size: tokens per split-KV partition (multiple of 16; 0 = automatic:
 * kvb_paged_attention_auto_partition(batch, max_seq_len), or 512 when the workspace was
 * sized for 512-token partitions).
 * exp_sums, max_logits [B, Hq, max_partitions] and tmp_out [B, Hq, max_partitions, D]
 * (out_dtype, optional, all or none): the v2 partition outputs; then out uses the v2
 * normalisation (global_sum + 1e-6) and max_partitions must equal
 * ceil(max_seq_len / partition_size).
 * D in {32, 64, 128} (float32 caches: any multiple of 4); any block_size; Hkv * ceil(group / 8) <= 16.
 */
KVB_API int kvb_paged_attention(const void* query, int q_dtype, const void* key_cache, const void* value_cache,
                                int cache_dtype, const float* k_scale, const float* v_scale, const void* seq_lens,
                                int seq_lens_dtype, const int32_t* block_table, int64_t bt_stride, int batch,
                                int num_q_heads, int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                int64_t max_seq_len, float sm_scale, const void* k_new, const void* v_new,
                                int new_dtype, int partition_size, void* out, int out_dtype, void* exp_sums,
                                void* max_logits, void* tmp_out, int max_partitions, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Bytes of workspace kvb_flash_attn_with_kvcache needs. */
KVB_API size_t kvb_flash_attn_with_kvcache_workspace_size(int batch, int seq_len_q, int num_heads, int head_dim,
                                                          int64_t seq_len_k);

/*
 * Attention of seq_len_q query tokens per sequence over a dense KV cache.
 * Replaces operators/attention/flash_attn_with_kvcache/flash_attn_with_kvcache.py:29-56:
 * q [batch, seq_len_q, num_heads, D]; k_cache / v_cache [batch, seq_len_k, num_kv_heads, D];
 * cache_seqlens [batch] (KVB_I32 or KVB_I64, each <= seq_len_k): every query token of
 * sequence b attends to its first cache_seqlens[b] keys (no causal mask), query head h to KV
 * head h / (num_heads / num_kv_heads), logits scaled by softmax_scale, float32 softmax.
 * out [batch, seq_len_q, num_heads, D] in `dtype`; softmax_lse [batch, num_heads, seq_len_q]
 * float32, the natural-log sum of exp of the scaled logits (may be NULL).  q, caches and out
 * share `dtype` (KVB_F32, KVB_F16 or KVB_BF16; D = 32, 64 or 128 for the 16-bit types).  Runs
 * the split-KV decode kernels with one query row per (sequence, query token); KV heads whose
 * query tiles exceed 16 warps are split across CTAs.  workspace: >=
 * kvb_flash_attn_with_kvcache_workspace_size() bytes.
 */
KVB_API int kvb_flash_attn_with_kvcache(const void* q, const void* k_cache, const void* v_cache, int dtype,
                                       const void* cache_seqlens, int seqlens_dtype, int batch, int seq_len_q,
                                       int64_t seq_len_k, int num_heads, int num_kv_heads, int head_dim,
                                       float softmax_scale, void* out, float* softmax_lse, void* workspace,
                                       size_t workspace_bytes, void* stream);

/*
 * Packed variable-length causal prefill.  Replaces
 * operators/attention/batched_prefill_attention/batched_prefill_attention.py:30-73:
 * q [total_q, num_q_heads, D]; k / v [total_kv, num_kv_heads, D]; qo_indptr / kv_indptr int32
 * [batch + 1] (device): request b owns query rows [qo_indptr[b], qo_indptr[b+1]) and keys
 * [kv_indptr[b], kv_indptr[b+1]); with q_len <= kv_len its query row i is at position
 * kv_len - q_len + i and attends keys 0..that position (causal), query head h using KV head
 * h / (num_q_heads / num_kv_heads); logits scaled by softmax_scale; float32 softmax state.
 * out [total_q, num_q_heads, D] in `dtype` (KVB_F32, KVB_F16 or KVB_BF16, shared by q, k, v).
 * D a multiple of 8, at most 128.  An indptr range outside [0, total_q] / [0, total_kv] skips
 * its request and sets bit 2 of kvb_device_status.  No workspace, no host synchronisation.
 */
KVB_API int kvb_batched_prefill_attention(const void* q, const void* k, const void* v, int dtype,
                                          const int32_t* qo_indptr, const int32_t* kv_indptr, int batch,
                                          int64_t total_q, int64_t total_kv, int num_q_heads, int num_kv_heads,
                                          int head_dim, float softmax_scale, void* out, void* stream);
/*
 * The same with the kernel chosen (test hook, no reference counterpart): variant 0 = automatic
 * (tcgen05 for f16 / bf16 with head_dim a multiple of 16 in [64, 128], at least 128 query and
 * key tokens and a 16-byte-aligned out; otherwise the mma.sync kernel), 1 = the mma.sync
 * kernel, 2 = the tcgen05 kernel with one 128-row query tile per CTA, 3 = the tcgen05 kernel
 * with two query tiles per CTA (KVB_E_SHAPE where tcgen05 does not apply).
 */
KVB_API int kvb_batched_prefill_attention_variant(const void* q, const void* k, const void* v, int dtype,
                                                  const int32_t* qo_indptr, const int32_t* kv_indptr, int batch,
                                                  int64_t total_q, int64_t total_kv, int num_q_heads,
                                                  int num_kv_heads, int head_dim, float softmax_scale, void* out,
                                                  int variant, void* stream);

/*
 * Allocation-free variant of kvb_paged_attention (no counterpart in the reference).
 * Some callers cannot allocate device memory: a plugin that its host framework hands only
 * input and output buffers, or a serving loop that must not call cudaMalloc (which can
 * synchronise the device) on its hot path.  This entry point takes the same arguments as
 * kvb_paged_attention minus the workspace and keeps its split-KV partials in a static
 * device array of KVB_PAGED_ATTENTION_NOALLOC_SCRATCH_BYTES (16 MiB), which every GPU that
 * loads the library holds until the process exits.  It allocates and frees nothing.
 *   - Calls needing more scratch than that (batch * num_q_heads * ceil(max_seq_len /
 *     partition_size) * (head_dim + 2) * 4 + 256 bytes) fail with KVB_E_WORKSPACE; a larger
 *     partition_size shrinks the need.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *     with that device current; make that first call before any stream capture.
 *   - All calls on a device share the array and it keeps the last call's contents; calls
 *     whose work overlaps on the GPU (different streams or host threads) race on it.
 */
#define KVB_PAGED_ATTENTION_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
KVB_API int kvb_paged_attention_noalloc(const void* query, int q_dtype, const void* key_cache,
                                        const void* value_cache, int cache_dtype, const float* k_scale,
                                        const float* v_scale, const void* seq_lens, int seq_lens_dtype,
                                        const int32_t* block_table, int64_t bt_stride, int batch, int num_q_heads,
                                        int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                        int64_t max_seq_len, float sm_scale, const void* k_new, const void* v_new,
                                        int new_dtype, int partition_size, void* out, int out_dtype,
                                        void* exp_sums, void* max_logits, void* tmp_out, int max_partitions,
                                        void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* KVB_H_ */
