/*
 * ntb200.h -- C ABI of the B200 (sm_100a) operator backend behind the vllm_nt plugin.
 *
 * Every entry point takes plain device pointers, element counts and element strides
 * (strides are in ELEMENTS, never bytes), launches its kernels on `stream` (a
 * cudaStream_t passed as void*), never synchronises the host, never allocates, and
 * returns NTB200_OK (0) or a negative NTB200_ERR_* status.  The caller owns all memory;
 * the only scratch an op needs (split-K partials of the paged decode) is passed in as
 * `workspace` and sized by the matching *_workspace_size() query.  No lock is taken on a
 * launch path beyond one-time per-device set-ups (error word, SM count, shared-memory limits,
 * the no-allocation decode's scratch address); the per-thread error message is thread-local.
 *
 * Each function names the reference (vllm_nt) interface it replaces.  Citations are
 * paths inside the vllm_nt project.
 */
#ifndef NTB200_H_
#define NTB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
enum {
  NTB200_DTYPE_F32 = 0,
  NTB200_DTYPE_BF16 = 1,
  NTB200_DTYPE_F16 = 2,
  NTB200_DTYPE_I32 = 3,
  NTB200_DTYPE_I64 = 4
};

/* host-side status codes */
enum {
  NTB200_OK = 0,
  NTB200_ERR_INVALID_ARGUMENT = -1, /* null pointer, negative size, bad stride */
  NTB200_ERR_UNSUPPORTED_DTYPE = -2,
  NTB200_ERR_MISALIGNED = -3,       /* pointer/stride not aligned for the vector path */
  NTB200_ERR_WORKSPACE = -4,        /* workspace missing or too small */
  NTB200_ERR_CUDA = -5,             /* a CUDA runtime/driver call failed */
  NTB200_ERR_UNSUPPORTED_SHAPE = -6,
  NTB200_ERR_DEVICE = -7            /* reported by ntb200_read_device_error */
};

/* bits of the device-side error word (see ntb200_read_device_error) */
enum {
  NTB200_DEVERR_WAIT_TIMEOUT = 1,   /* a bounded mbarrier wait gave up; the kernel returned early */
  NTB200_DEVERR_INDEX_RANGE = 2     /* an id / slot / block id was out of range and was skipped */
};

int ntb200_version(void);
const char* ntb200_status_string(int status);
/* Detail of the last non-OK status returned on the calling thread. */
const char* ntb200_last_error(void);
/* Copies the device error word of the current device into *word (0 = clean) and clears it.
 * Synchronises `stream`. */
int ntb200_read_device_error(int* word, void* stream);

/* ---------------------------------------------------------------------------------------
 * RMS norm:  out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * weight   (fp32 statistics)
 * Replaces vllm_nt/_ntops/torch/rms_norm.py:10-33 (_fused_rms_norm_last_dim) and
 * vllm_nt/_ntops/kernels/fused_rms_norm.py:9-24.  weight may be NULL (all ones).
 * dtype: F32, BF16 or F16 (x, weight and out share it).
 */
int ntb200_rms_norm(void* out, const void* x, const void* weight, int64_t num_rows,
                    int64_t hidden, int64_t x_row_stride, int64_t out_row_stride, float eps,
                    int dtype, void* stream);

/* Fused residual add + RMS norm:  s = x + residual (fp32);  residual <- s (rounded to
 * dtype);  out = s * rsqrt(mean(s^2) + eps) * weight.  out may alias x.
 * Replaces vllm_nt/_ntops/oot_support.py:32-48 (norm with a residual) which vllm_nt's
 * RMSNorm hook reaches from vllm_nt/_ntops/patching.py:229-256. */
int ntb200_fused_add_rms_norm(void* out, void* residual, const void* x, const void* weight,
                              int64_t num_rows, int64_t hidden, int64_t x_row_stride,
                              int64_t residual_row_stride, int64_t out_row_stride, float eps,
                              int dtype, void* stream);

/* Gemma RMS norm:  out = round(x * rsqrt(mean(x^2) + eps) * (1 + weight))  with (1 + weight)
 * formed in fp32 and one rounding (of the product), as vLLM's GemmaRMSNorm.forward_native
 * (vllm/model_executor/layers/layernorm.py:153-170) computes it.  weight is the raw Gemma
 * parameter w (not 1 + w) and must not be NULL.
 * Replaces vllm_nt/_ntops/oot_support.py:32-48 (norm with gemma=True), which vllm_nt's
 * GemmaRMSNorm hook reaches from vllm_nt/_ntops/patching.py:259-288. */
int ntb200_gemma_rms_norm(void* out, const void* x, const void* weight, int64_t num_rows,
                          int64_t hidden, int64_t x_row_stride, int64_t out_row_stride, float eps,
                          int dtype, void* stream);

/* Gemma residual add + RMS norm:  s = x + residual in the input dtype (a bf16 sum is rounded
 * to bf16 before the statistics);  residual <- s;  out as ntb200_gemma_rms_norm(s).  F32 and
 * BF16 only: vLLM returns an fp32 residual for fp16 inputs, which the in-place fp16 residual
 * cannot hold (NTB200_ERR_UNSUPPORTED_DTYPE).  out may alias x. */
int ntb200_gemma_fused_add_rms_norm(void* out, void* residual, const void* x, const void* weight,
                                    int64_t num_rows, int64_t hidden, int64_t x_row_stride,
                                    int64_t residual_row_stride, int64_t out_row_stride, float eps,
                                    int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * out[r, i] = silu(x[r, i]) * x[r, d + i],  i < d.
 * Replaces vllm_nt/_ntops/oot_support.py:51-56 (act_and_mul with nt_silu),
 * vllm_nt/_ntops/torch/silu.py:7-17 and vllm_nt/_ntops/kernels/silu.py:9-18. */
int ntb200_silu_and_mul(void* out, const void* x, int64_t num_rows, int64_t d,
                        int64_t x_row_stride, int64_t out_row_stride, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * In-place NeoX rotary embedding of the first rotary_dim dims of every query/key head:
 *   c, s = cos_sin_cache[pos][:rot/2], cos_sin_cache[pos][rot/2:rot]
 *   x1' = x1*c - x2*s ;  x2' = x2*c + x1*s
 * key may be NULL.  positions: I64 or I32.  cos_sin_cache [num_cache_rows, >= rotary_dim]
 * has the dtype of query/key.  A token whose position is outside [0, num_cache_rows) is
 * left untouched and sets NTB200_DEVERR_INDEX_RANGE.
 * Replaces vllm_nt/_ntops/oot_support.py:134-204 (rope/_apply_rotary),
 * vllm_nt/_ntops/torch/rotary_emb.py:7-9 and vllm_nt/_ntops/kernels/rotary_emb.py:6-37. */
int ntb200_rotary_embedding_neox(const void* positions, int positions_dtype, void* query,
                                 void* key, const void* cos_sin_cache, int64_t num_tokens,
                                 int64_t num_q_heads, int64_t num_k_heads, int64_t head_size,
                                 int64_t rotary_dim, int64_t q_token_stride,
                                 int64_t q_head_stride, int64_t k_token_stride,
                                 int64_t k_head_stride, int64_t cache_row_stride,
                                 int64_t num_cache_rows, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * Paged KV-cache store (slot-mapped scatter; bit-exact copy):
 *   for t with slot = slot_mapping[t] >= 0:
 *     key_cache  [slot / block_size, slot % block_size, h, :] = key  [t, h, :]
 *     value_cache[slot / block_size, slot % block_size, h, :] = value[t, h, :]
 * Negative slots (vLLM padding) are skipped; slots >= num_slots are skipped and set
 * NTB200_DEVERR_INDEX_RANGE.  Both caches share the strides given.  elem_bytes: 1, 2 or 4.
 * slot_dtype: I64 or I32.
 * Replaces vllm_nt/_ntops/torch/kv_cache.py:7-21 (store_kvcache) and
 * vllm_nt/_ntops/kernels/kv_cache.py:4-45. */
int ntb200_reshape_and_cache(const void* key, const void* value, void* key_cache,
                             void* value_cache, const void* slot_mapping, int slot_dtype,
                             int64_t num_tokens, int64_t num_heads, int64_t head_size,
                             int64_t block_size, int64_t num_slots, int64_t key_token_stride,
                             int64_t key_head_stride, int64_t value_token_stride,
                             int64_t value_head_stride, int64_t cache_block_stride,
                             int64_t cache_page_stride, int64_t cache_head_stride,
                             int elem_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * NeoX RoPE fused with the paged KV-cache store, one pass over the step's q/k/v rows:
 *   q, k <- rotated in place exactly as ntb200_rotary_embedding_neox does;
 *   for t < num_store_tokens with slot = slot_mapping[t] >= 0:
 *     key_cache  [slot / block_size, slot % block_size, h, :] = rotated key[t, h, :]
 *     value_cache[slot / block_size, slot % block_size, h, :] = value[t, h, :]
 * The result is bit-identical to ntb200_rotary_embedding_neox followed by
 * ntb200_reshape_and_cache, in every case: negative slots (vLLM padding) only rotate; slots
 * >= num_slots only rotate and set NTB200_DEVERR_INDEX_RANGE; a position outside
 * [0, num_cache_rows) leaves the token's q/k unrotated (its unrotated k and its v are still
 * stored) and sets NTB200_DEVERR_INDEX_RANGE.  One fused kernel below 2048 tokens; from
 * 2048 tokens on, where the two kernels keep more bytes in flight, the pair is launched.
 * key and value rows have num_kv_heads heads of head_size; both caches share the strides
 * given and have the dtype of query/key/value (F32, BF16 or F16).  positions: I64 or I32,
 * num_tokens entries; slot_mapping: I64 or I32, num_store_tokens (<= num_tokens) entries;
 * rows past it (vLLM's padded rows) are rotated only.
 * Replaces the RoPE hook followed by the KV-store hook of one attention layer:
 * vllm_nt/_ntops/oot_support.py:134-204 with vllm_nt/_ntops/kernels/rotary_emb.py:6-37,
 * then vllm_nt/_ntops/torch/kv_cache.py:7-21 with vllm_nt/_ntops/kernels/kv_cache.py:4-45
 * (reached from vllm_nt/_ntops/patching.py:1323-1354 and 532-562); the reference has no
 * fused form. */
int ntb200_rope_and_cache(const void* positions, int positions_dtype, void* query, void* key,
                          const void* value, const void* cos_sin_cache, void* key_cache,
                          void* value_cache, const void* slot_mapping, int slot_dtype,
                          int64_t num_tokens, int64_t num_store_tokens, int64_t num_q_heads,
                          int64_t num_kv_heads,
                          int64_t head_size, int64_t rotary_dim, int64_t q_token_stride,
                          int64_t q_head_stride, int64_t k_token_stride, int64_t k_head_stride,
                          int64_t v_token_stride, int64_t v_head_stride, int64_t cache_row_stride,
                          int64_t num_cache_rows, int64_t block_size, int64_t num_slots,
                          int64_t cache_block_stride, int64_t cache_page_stride,
                          int64_t cache_head_stride, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * Embedding gather (bit-exact copy): out[t, :] = weight[ids[t], :].
 * Ids outside [0, num_embeddings) produce a zero row and set NTB200_DEVERR_INDEX_RANGE.
 * ids_dtype: I64 or I32.  elem_bytes: 1, 2 or 4.
 * Replaces vllm_nt/_ntops/torch/embedding.py:7-30 and vllm_nt/_ntops/kernels/wpe.py:11-67
 * (reached from vllm_nt/_ntops/patching.py:2661-2679). */
int ntb200_embedding(void* out, const void* ids, int ids_dtype, const void* weight,
                     int64_t num_tokens, int64_t num_embeddings, int64_t embedding_dim,
                     int64_t weight_row_stride, int64_t out_row_stride, int elem_bytes,
                     void* stream);

/* ---------------------------------------------------------------------------------------
 * Paged-attention decode (one query token per sequence), split-K over KV blocks:
 *   out[b, h] = softmax(scale * q[b, h] . K_b^T) V_b  over the seq_lens[b] cached tokens of
 *   sequence b, K/V head = h / (num_q_heads / num_kv_heads).  fp32 softmax/accumulate.
 * Cache layout [num_blocks, block_size, num_kv_heads, head_size] (vLLM flash layout, one
 * of K/V); block_tables [num_seqs, block_table_stride] int32; seq_lens [num_seqs] int32.
 * max_seq_len bounds every seq_lens[b] (<= 0: derived from max_blocks_per_seq).
 * dtype BF16 or F16; head_size 128; block_size 16 (the decode kernel's tile shape).
 * workspace: ntb200_paged_attention_decode_workspace_size(...) bytes, 256-byte aligned.
 * Sequences with seq_lens[b] == 0 produce zeros.
 * Replaces vllm_nt/_ntops/torch/attention.py:51-77 (flash_attn_with_kvcache) and
 * vllm_nt/_ntops/kernels/attention.py:97-197 (KvCache), reached from
 * vllm_nt/_ntops/oot_support.py:112-123. */
size_t ntb200_paged_attention_decode_workspace_size(int64_t num_seqs, int64_t num_q_heads,
                                                    int64_t num_kv_heads, int64_t head_size,
                                                    int64_t block_size, int64_t max_seq_len);
int ntb200_paged_attention_decode(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* seq_lens, const int32_t* block_tables, int64_t num_seqs,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int64_t block_size,
    int64_t num_blocks, int64_t max_blocks_per_seq, int64_t block_table_stride,
    int64_t max_seq_len, float scale, int64_t q_seq_stride, int64_t q_head_stride,
    int64_t out_seq_stride, int64_t out_head_stride, int64_t cache_block_stride,
    int64_t cache_page_stride, int64_t cache_head_stride, void* workspace,
    size_t workspace_bytes, int dtype, void* stream);

/* The same decode without a caller workspace, for callers that cannot allocate device
 * memory at the call: a serving loop that must not call cudaMalloc/cudaFree while decoding
 * (they can synchronise the device and take a process-wide lock), code being recorded
 * into a CUDA graph, or a host that binds only this C ABI and has no device allocator.
 * The split-K partials go to a fixed 64 MiB array compiled into the library, which a GPU
 * holds until the process exits once the library's device code is loaded on it (under the
 * default lazy module loading: on first use; with CUDA_MODULE_LOADING=EAGER: on every GPU
 * whose context loads the library).  A call that needs more scratch than that returns
 * NTB200_ERR_WORKSPACE without launching.  The first successful call on a device resolves
 * the array's address (cudaGetSymbolAddress), so make it before any stream capture; a
 * failed lookup is not remembered, and the next call retries it.  All calls on a device
 * share the array: calls that overlap on the GPU race; order them on one stream.  Arguments as ntb200_paged_attention_decode minus the
 * workspace.  This entry point has no counterpart in the reference. */
int ntb200_paged_attention_decode_noalloc(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* seq_lens, const int32_t* block_tables, int64_t num_seqs,
    int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int64_t block_size,
    int64_t num_blocks, int64_t max_blocks_per_seq, int64_t block_table_stride,
    int64_t max_seq_len, float scale, int64_t q_seq_stride, int64_t q_head_stride,
    int64_t out_seq_stride, int64_t out_head_stride, int64_t cache_block_stride,
    int64_t cache_page_stride, int64_t cache_head_stride, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * Varlen paged prefill attention (a flash-attention forward on the tcgen05 tensor cores):
 *   out[t, h] = softmax(scale * q[t, h] . K_b^T + mask) V_b
 * for the queries t of sequence b (rows query_start_loc[b] .. query_start_loc[b+1] of
 * query/out, [num_tokens, num_q_heads, head_size]) over the seq_lens[b] tokens cached for b
 * (the queries' own K/V included, as the last q_len of them), K/V head
 * h / (num_q_heads / num_kv_heads).  causal != 0: query i of a sequence with q_len queries
 * sits at position seq_lens[b] - q_len + i and sees keys up to that position (vLLM's
 * FlashAttention rule; it covers a cached prefix and chunked prefill).  fp32 softmax and
 * accumulation, P rounded to the input type for the P.V product.  Rows that see no key are
 * zero.  Caches and block tables as ntb200_paged_attention_decode; head_size 128,
 * block_size 16; dtype BF16 or F16; all pointers 16-byte aligned, strides multiples of 8.
 * max_query_len bounds every q_len.  Out-of-range page ids and context lengths set
 * NTB200_DEVERR_INDEX_RANGE (the pages read as zeros).  No workspace.
 * Replaces vllm_nt/_ntops/kernels/attention.py:10-94 (_VarLen) with the K/V gather of
 * vllm_nt/_ntops/torch/kv_cache.py:24-63, reached from vllm_nt/_ntops/patching.py:639-671. */
int ntb200_paged_attention_prefill(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* block_tables,
    int64_t num_seqs, int64_t num_tokens, int64_t num_q_heads, int64_t num_kv_heads,
    int64_t head_size, int64_t block_size, int64_t num_blocks, int64_t max_blocks_per_seq,
    int64_t block_table_stride, int64_t max_query_len, float scale, int causal,
    int64_t q_token_stride, int64_t q_head_stride, int64_t out_token_stride,
    int64_t out_head_stride, int64_t cache_block_stride, int64_t cache_page_stride,
    int64_t cache_head_stride, int dtype, void* stream);

/* Decode for the single-query sequences of a varlen batch: as ntb200_paged_attention_decode,
 * but sequence b's query and output row is query_start_loc[b] ([num_seqs + 1] int32) and
 * sequences whose query count is not 1 are left untouched.  Same workspace. */
int ntb200_paged_attention_decode_varlen(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* block_tables,
    int64_t num_seqs, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
    int64_t block_size, int64_t num_blocks, int64_t max_blocks_per_seq,
    int64_t block_table_stride, int64_t max_seq_len, float scale, int64_t q_token_stride,
    int64_t q_head_stride, int64_t out_token_stride, int64_t out_head_stride,
    int64_t cache_block_stride, int64_t cache_page_stride, int64_t cache_head_stride,
    void* workspace, size_t workspace_bytes, int dtype, void* stream);

/* A vLLM attention batch of any mix of decodes and (chunked) prefills, causal: the
 * single-query sequences through ntb200_paged_attention_decode_varlen, the others through
 * the prefill kernel (which skips the single-query ones).  Arguments as
 * ntb200_paged_attention_prefill plus max_seq_len (bounds seq_lens) and the decode
 * workspace (ntb200_paged_attention_decode_workspace_size(num_seqs, ...) bytes).
 * Replaces the prefill/decode split of vllm_nt/_ntops/patching.py:565-685. */
int ntb200_paged_attention_varlen(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* block_tables,
    int64_t num_seqs, int64_t num_tokens, int64_t num_q_heads, int64_t num_kv_heads,
    int64_t head_size, int64_t block_size, int64_t num_blocks, int64_t max_blocks_per_seq,
    int64_t block_table_stride, int64_t max_query_len, int64_t max_seq_len, float scale,
    int64_t q_token_stride, int64_t q_head_stride, int64_t out_token_stride,
    int64_t out_head_stride, int64_t cache_block_stride, int64_t cache_page_stride,
    int64_t cache_head_stride, void* workspace, size_t workspace_bytes, int dtype, void* stream);

/* The same attention over contiguous varlen K/V instead of the paged cache: key/value
 * [num_k_tokens, num_kv_heads, 128], sequence b's keys at rows cu_seqlens_k[b] ..
 * cu_seqlens_k[b+1] (its context), its queries at rows cu_seqlens_q[b] .. cu_seqlens_q[b+1]
 * of query/out; causal as above (aligned to the end of each context).
 * Replaces vllm_nt/_ntops/torch/attention.py:9-46 (flash_attn_varlen_func) and
 * vllm_nt/_ntops/kernels/attention.py:10-94, reached from
 * vllm_nt/_ntops/oot_support.py:88-109 (paged_attention_prefill). */
int ntb200_flash_attn_varlen(
    void* out, const void* query, const void* key, const void* value,
    const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int64_t num_seqs,
    int64_t num_q_tokens, int64_t num_k_tokens, int64_t num_q_heads, int64_t num_kv_heads,
    int64_t head_size, int64_t max_query_len, float scale, int causal, int64_t q_token_stride,
    int64_t q_head_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t v_token_stride, int64_t v_head_stride, int64_t out_token_stride,
    int64_t out_head_stride, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * Dense projection  out[M, N] = x[M, K] . weight[N, K]^T (+ bias[N]),  fp32 accumulate,
 * tcgen05/TMEM tensor cores fed by TMA.  dtype BF16 or F16; K a multiple of 8, rows 16-byte
 * aligned.  bias may be NULL.
 * Replaces vllm_nt/_ntops/torch/linear.py:7-21 and vllm_nt/_ntops/kernels/linear.py:9-85
 * (reached from vllm_nt/_ntops/oot_support.py:59-65). */
size_t ntb200_linear_workspace_size(int64_t M, int64_t N, int64_t K);
int ntb200_linear(void* out, const void* x, const void* weight, const void* bias, int64_t M,
                  int64_t N, int64_t K, int64_t x_row_stride, int64_t weight_row_stride,
                  int64_t out_row_stride, void* workspace, size_t workspace_bytes, int dtype,
                  void* stream);

/* ---------------------------------------------------------------------------------------
 * Fused gate_up projection + SiluAndMul:
 *   out[M, I] = silu(x . W[0:I]^T) * (x . W[I:2I]^T)
 * for vLLM's merged gate_up weight W [2I, K] (MergedColumnParallelLinear, gate rows then
 * up rows), with the rounding points of the unfused pair (each half rounded to the dtype,
 * silu(gate) rounded before the multiply), so the result equals ntb200_linear followed by
 * ntb200_silu_and_mul.  Replaces the MatMul hook on gate_up_proj followed by the
 * SiluAndMul hook (vllm_nt/_ntops/patching.py:2630-2658 and 291-316); the reference has
 * no fused form.  dtype BF16 or F16; K a multiple of 8, rows 16-byte aligned; no bias. */
int ntb200_linear_silu_and_mul(void* out, const void* x, const void* weight, int64_t M, int64_t I,
                               int64_t K, int64_t x_row_stride, int64_t weight_row_stride,
                               int64_t out_row_stride, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * Fused (residual-add) RMS norm + projection for decode batches of at most 16 tokens:
 *   s = x (+ residual) in fp32;  residual_out = s (rounded);
 *   out[m, n] = rsqrt(mean_k(s[m, k]^2) + eps) * sum_k round(s[m, k] * norm_weight[k]) W[n, k]
 * Replaces the RMSNorm hook followed by the MatMul hook of the next projection
 * (vllm_nt/_ntops/oot_support.py:32-48, then vllm_nt/_ntops/torch/linear.py:7-21), which
 * the reference runs as two kernels with the normalised rows written to and read back from
 * memory; here the GEMM input round(s * norm_weight) is formed in shared memory and never
 * written, and the per-row 1/rms scales the fp32 products (the projection is linear in
 * it), so the MMAs do not wait for the row statistics.  The rounding points therefore
 * differ from the unfused pair's (normalised value rounded, times the weight, rounded
 * again): one rounding of the input instead of two.  residual and residual_out
 * are both given or both null, and residual_out must not alias x or residual (other CTAs
 * still read them while it is written).  M <= 16 (NTB200_ERR_UNSUPPORTED_SHAPE above),
 * dtype BF16 or F16, K a multiple of 8, rows 16-byte aligned; at most 4096 columns of K per
 * CTA after the K split (NTB200_ERR_UNSUPPORTED_SHAPE otherwise). */
int ntb200_rms_norm_linear(void* out, void* residual_out, const void* x, const void* residual,
                           const void* norm_weight, float eps, const void* weight, int64_t M,
                           int64_t N, int64_t K, int64_t x_row_stride, int64_t residual_row_stride,
                           int64_t residual_out_row_stride, int64_t weight_row_stride,
                           int64_t out_row_stride, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * LM head + greedy argmax:  out_index[m] = argmax_v (x[m] . W[v])  over V vocabulary rows,
 * comparing the logits rounded to the dtype (what vLLM's greedy sampler compares: the LM
 * head writes dtype logits) with the first index winning ties, as torch.argmax does.  For
 * M <= 256 the GEMM epilogue reduces each tile and folds it into a per-token key with a
 * 64-bit atomicMax, so the [M, V] logits are never written; larger M computes the logits
 * into the workspace and reduces each row.  Replaces the LMHead hook (vllm_nt/_ntops/
 * patching.py:2682-2710) followed by the sampler's argmax (vllm:v1/sample/sampler.py
 * greedy_sample) for greedy decoding.  out_index: int64 [M].  workspace:
 * ntb200_linear_argmax_workspace_size(M, V, K) bytes, 256-byte aligned. */
size_t ntb200_linear_argmax_workspace_size(int64_t M, int64_t V, int64_t K);
int ntb200_linear_argmax(int64_t* out_index, const void* x, const void* weight, int64_t M, int64_t V,
                         int64_t K, int64_t x_row_stride, int64_t weight_row_stride, void* workspace,
                         size_t workspace_bytes, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * Top-k / top-p mask of fp32 logits [num_rows, vocab] (row stride row_stride), in place:
 * for each row b, with k = clamp(top_k[b], 1, vocab) and p = top_p[b],
 *   top-k: logits below the k-th largest logit of the row become -inf (ties with it kept);
 *   top-p: over the logits top-k kept, with probabilities exp(x - max) / Z, logits whose
 *          cumulative probability counted from the smallest upwards (themselves included)
 *          is <= 1 - p become -inf; the largest logit is always kept.
 * top_k (I32 or I64 per row, top_k_dtype) or top_p (fp32 per row) may be NULL to skip that
 * filter; both NULL is a no-op.  No sort: per row, radix selection of the two cut values
 * over order-preserving 32-bit keys, one CTA per row.  Equal to the reference's sort-based
 * mask except where a run of equal logits straddles the top-p cut (kept whole here; the
 * reference keeps the part its unstable sort happens to put last) or where the cumulative
 * probability at a logit is within fp32 summation error of 1 - p.
 * Replaces vllm_nt/_ntops/torch/sampler.py:4-31 (apply_top_k_top_p), reached from
 * vllm_nt/_ntops/patching.py:1446-1463 (the TopKTopP patch of vLLM's
 * topk_topp_sampler.apply_top_k_top_p). */
int ntb200_top_k_top_p(float* logits, int64_t num_rows, int64_t vocab, int64_t row_stride,
                       const void* top_k, int top_k_dtype, const float* top_p, void* stream);

/* Exponential-race sampling from fp32 probabilities: out[b] = argmax_i probs[b, i] / q[b, i]
 * (int64), q being the caller's Exp(1) draws, with the quotient rounded as IEEE division,
 * NaN ranked above every number and the first index winning ties (torch.argmax).  One pass
 * over probs and q; the [num_rows, vocab] quotient is never written.
 * Replaces vllm_nt/_ntops/torch/sampler.py:34-42 (random_sample: torch.div then argmax),
 * reached from vllm_nt/_ntops/patching.py:1466-1479 (the RandomSample patch). */
int ntb200_random_sample(int64_t* out, const float* probs, const float* q, int64_t num_rows,
                         int64_t vocab, int64_t probs_row_stride, int64_t q_row_stride,
                         void* stream);

/* ---------------------------------------------------------------------------------------
 * One-shot all-reduce over peer memory for the row-parallel projections of tensor
 * parallelism (o_proj and down under TP): replaces the NCCL all-reduce that vLLM's
 * RowParallelLinear issues after the GEMM (vllm:model_executor/layers/linear.py
 * RowParallelLinear.forward -> tensor_model_parallel_all_reduce); the reference plugin has
 * no counterpart of its own (it leaves the collective to vLLM).
 * Every rank owns a buffer of ntb200_allreduce_buffer_size(capacity, 2, world_size) bytes
 * that all ranks can address (e.g. torch symmetric memory), zero-filled once; capacity is
 * the largest element count it will reduce.  partial (numel <= capacity bf16/f16 elements,
 * this rank's GEMM output, ordinary device memory) is pushed into every rank's buffer and
 * out receives the elementwise sum of all ranks' partials (fp32 accumulation).
 * peer_buffers is a DEVICE array of world_size buffer addresses (index = rank, this rank's
 * own included).  Every rank must make the same sequence of calls on its buffer; the call
 * count lives in the buffer, so calls may be captured in a CUDA graph and replayed.  At
 * most 8 ranks.  Waits for peers are bounded (NTB200_DEVERR_WAIT_TIMEOUT after ~2 s). */
size_t ntb200_allreduce_buffer_size(int64_t capacity, int elem_bytes, int world_size);
int ntb200_allreduce_oneshot(void* out, const void* partial, const uint64_t* peer_buffers,
                             int64_t numel, int64_t capacity, int rank, int world_size, int dtype,
                             void* stream);

/* The same sum as a two-shot all-reduce (reduce-scatter, then all-gather) over the same
 * buffers: rank r pushes chunk d of its partial to rank d, sums the W pieces of chunk r, and
 * reads the other ranks' reduced chunks over NVLink.  Each rank moves 2 (W - 1) / W of the
 * message over NVLink instead of the one-shot's (W - 1), at the cost of a second barrier: the
 * form for messages of more than a few hundred KB.  numel must be a multiple of 8.  Calls of
 * the two kinds may alternate on one buffer (every rank in the same order). */
int ntb200_allreduce_twoshot(void* out, const void* partial, const uint64_t* peer_buffers,
                             int64_t numel, int64_t capacity, int rank, int world_size, int dtype,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NTB200_H_ */
