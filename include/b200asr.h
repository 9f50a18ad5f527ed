/*
 * b200asr -- B200 (sm_100a) kernels for the ragged continuous-batching path of the
 * qwen-asr-vllm engine (Qwen3-ASR). C ABI: plain device pointers, sizes and a CUDA
 * stream; no framework types. Every call is asynchronous on `stream`, launches only
 * kernels (no allocation, no host synchronisation), and may therefore be captured
 * in a CUDA graph. All tensors are device memory owned by the caller.
 *
 * Types: "bf16" = 16-bit bfloat16 element, passed as void*. Row strides are in
 * ELEMENTS. Every function returns B200ASR_OK (0) or an error code; the message of
 * the last failure on the calling thread is available from b200asr_last_error().
 *
 * Device-side index checks: where a kernel meets an index outside the caller's
 * declared bounds (a KV slot or block id outside the pool, a position outside the
 * RoPE table) it skips that access and ORs a bit into *error_flag (when non-NULL):
 *   B200ASR_DEVERR_SLOT 1, B200ASR_DEVERR_BLOCK 2, B200ASR_DEVERR_POSITION 4,
 *   B200ASR_DEVERR_LENGTH 8. The host reads the word after the step.
 *
 * Reference locations are paths inside the qwen-asr-vllm project.
 */
#ifndef B200ASR_H_
#define B200ASR_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define B200ASR_API __attribute__((visibility("default")))
#else
#define B200ASR_API
#endif

typedef struct CUstream_st *b200asr_stream_t; /* == cudaStream_t */

enum {
  B200ASR_OK = 0,
  B200ASR_ERR_INVALID = 1,     /* bad shape, stride, alignment or null pointer */
  B200ASR_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
  B200ASR_ERR_UNSUPPORTED = 3, /* configuration outside what the kernels handle */
  B200ASR_ERR_WORKSPACE = 4    /* caller workspace too small */
};

enum {
  B200ASR_DEVERR_SLOT = 1,
  B200ASR_DEVERR_BLOCK = 2,
  B200ASR_DEVERR_POSITION = 4,
  B200ASR_DEVERR_LENGTH = 8
};

/* Library version (major*10000 + minor*100 + patch) and last error message. */
B200ASR_API int b200asr_version(void);
B200ASR_API const char *b200asr_last_error(void);

/* Programmatic dependent launch (no reference counterpart; default off). When on,
 * the decode-path kernels (rmsnorm, qk_norm_rope_store, paged_decode, linear_small,
 * silu_mul, store_kvcache, greedy_argmax) are launched so that each may begin its
 * prologue -- shared-memory and TMEM set-up, tensor-map and weight loads -- while the
 * previous kernel in the stream finishes; each waits for that kernel's results before
 * reading them or writing global memory. A CUDA graph captured with it on keeps the
 * overlap. Process-wide; set it before capturing graphs.
 * Two reads happen before that wait, on data a decode step fixes before its decoder
 * kernels run: paged_decode with max_seqlen_k <= 512 reads cu_seqlens_k, block_tables
 * and the cached K/V rows of every position but each sequence's newest, and a
 * b200asr_l2_prefetch's K/V part reads cu_seqlens_k / block_tables.
 * With PDL on, those must have been written before the nearest preceding launch in the
 * stream that is not itself a PDL launch (the engine's embedding kernel follows the
 * step's packer); the newest row may be written by the kernel right before.          */
B200ASR_API void b200asr_set_pdl(int32_t enable);
B200ASR_API int32_t b200asr_pdl_enabled(void);

/* ---------------------------------------------------------------- packers ----
 * Replaces ModelRunner._prepare (engine/model_runner.py:183-233): builds the ragged
 * decoder metadata of a mixed prefill/decode batch on the GPU.
 *   req_start[b]  = num_computed_tokens, req_end[b] = len(request)
 *   table_off[b], table_len[b] index the concatenated block tables `tables`
 *   query_tokens  = concatenated token ids of every request's query span
 * Outputs: input_ids i64[T], positions i64[T], slot_mapping i32[T]
 * (= table[p / block_size] * block_size + p % block_size), cu_seqlens_q/k i32[B+1],
 * max_seqlen i32[2] (q, k), block_tables i32[B, width] padded with -1,
 * last_token_index i64[B] (= cu_seqlens_q[b+1] - 1). T = sum(end - start) must be
 * passed as total_tokens and width >= max(table_len).                              */
B200ASR_API int b200asr_pack_decoder(const int32_t *req_start, const int32_t *req_end,
                         const int32_t *table_off, const int32_t *table_len,
                         const int32_t *tables, const int32_t *query_tokens,
                         int32_t batch, int32_t total_tokens, int32_t width,
                         int32_t block_size, int64_t *input_ids, int64_t *positions,
                         int32_t *slot_mapping, int32_t *cu_seqlens_q, int32_t *cu_seqlens_k,
                         int32_t *max_seqlen, int32_t *block_tables,
                         int64_t *last_token_index, b200asr_stream_t stream);

/* Replaces GraphRunner.run host staging (engine/graph_runner.py:149-191): fills the
 * static decode buffers of a CUDA-graph bucket. Rows >= batch are padding: slot -1,
 * key length 1, all-zero block-table row, input id and position 0.
 *   lens[b] = len(request), last_ids[b] = last token id.
 * Outputs (sized for `bucket`): input_ids i64, positions i64, slot_mapping i32,
 * cu_seqlens_k i32[bucket+1], block_tables i32[bucket, max_blocks].              */
B200ASR_API int b200asr_pack_decode_bucket(const int32_t *lens, const int32_t *last_ids,
                               const int32_t *table_off, const int32_t *table_len,
                               const int32_t *tables, int32_t batch, int32_t bucket,
                               int32_t max_blocks, int32_t block_size, int64_t *input_ids,
                               int64_t *positions, int32_t *slot_mapping,
                               int32_t *cu_seqlens_k, int32_t *block_tables,
                               b200asr_stream_t stream);

/* Advances the first four descriptor arrays of b200asr_pack_decode_bucket by one
 * generated token, on the device: for rows with table_len > 0, lens += 1 and
 * last_ids = (int32) sampled (the greedy_argmax output). Used to replay a decode
 * graph several times in a row without a host round trip (the caller allocates the
 * blocks those steps write ahead of time); no reference counterpart.              */
B200ASR_API int b200asr_advance_decode_bucket(int32_t *lens, int32_t *last_ids,
                                  const int32_t *table_len, const int64_t *sampled,
                                  int32_t bucket, b200asr_stream_t stream);

/* Replaces the metadata of pack_audio_batch (audio/batcher.py:101-141) and
 * num_audio_tokens/chunk_lengths_for (audio/tokens.py:30-52).
 *   mel_frames[b] > 0 for each request.
 * Outputs: chunk_lengths i64[C], chunk_valid_lens i64[C], chunk_start i32[C]
 * (first mel frame of each chunk), audio_token_lens i32[B], cu_seqlens i32[W+1]
 * (attention windows of `window_tokens`), counts i32[3] = {C, W, max_seqlen}.
 * Capacities max_chunks / max_windows bound the outputs (B200ASR_DEVERR_LENGTH is
 * raised in *error_flag if exceeded).                                            */
B200ASR_API int b200asr_pack_audio(const int32_t *mel_frames, int32_t batch, int32_t chunk_frames,
                       int32_t window_tokens, int32_t max_chunks, int32_t max_windows,
                       int64_t *chunk_lengths, int64_t *chunk_valid_lens, int32_t *chunk_start,
                       int32_t *audio_token_lens, int32_t *cu_seqlens, int32_t *counts,
                       int32_t *error_flag, b200asr_stream_t stream);

/* Replaces AudioEncoder._chunk_and_pad (models/audio_encoder.py:130-143): packed
 * mel bf16[bins, total_frames] -> padded bf16[num_chunks, bins, chunk_frames] with
 * zeros past each chunk's length.                                                */
B200ASR_API int b200asr_audio_chunk_pad(const void *mel, int32_t bins, int32_t total_frames,
                            const int32_t *chunk_start, const int64_t *chunk_lengths,
                            int32_t num_chunks, int32_t chunk_frames, void *padded,
                            b200asr_stream_t stream);

/* Replaces the "conv.gather" step of AudioEncoder.forward
 * (models/audio_encoder.py:169-173): out[i] = bf16(embed[src] + pos[src % tokens_per_chunk]) with
 * src = token_index[i] for i < tokens (embed bf16[embed_rows, d], the conv_out rows of
 * every chunk; pos bf16[tokens_per_chunk, d]); rows [tokens, rows_out) of out are zero.
 * An index outside [0, embed_rows) raises B200ASR_DEVERR_LENGTH (its row is zeroed).  */
B200ASR_API int b200asr_audio_gather_pos(const void *embed, int64_t embed_rows, const void *pos,
                             int32_t tokens_per_chunk, const int64_t *token_index,
                             int32_t tokens, int32_t rows_out, int32_t d, void *out,
                             int32_t *error_flag, b200asr_stream_t stream);

/* ------------------------------------------------------------------ KV store ----
 * Replaces store_kvcache / _store_kvcache_kernel (layers/attention.py:31-67).
 * key/value: bf16 [T, num_kv_heads, head_dim] with row strides (elements) and a
 * contiguous [num_kv_heads * head_dim] row; caches: bf16 [num_slots, num_kv_heads *
 * head_dim]. slot_mapping[t] == -1 skips token t.                                 */
B200ASR_API int b200asr_store_kvcache(const void *key, int64_t key_row_stride, const void *value,
                          int64_t value_row_stride, void *k_cache, void *v_cache,
                          const int32_t *slot_mapping, int32_t num_tokens,
                          int32_t num_kv_heads, int32_t head_dim, int64_t num_slots,
                          int32_t *error_flag, b200asr_stream_t stream);

/* --------------------------------------------------------- norm + rope + store ----
 * Replaces Qwen3Attention.forward lines 43-48 (models/qwen3.py) plus the KV store:
 * from the fused qkv row [q | k | v] (bf16, row stride qkv_row_stride) computes
 * per-head RMSNorm of q and k (layers/layernorm.py:19-25, eps, bf16 weights), then
 * half-split RoPE (layers/rotary_embedding.py:9-32) at positions[t] using
 * cos_sin_cache fp32 [max_position, head_dim] = [cos | sin], writes q to q_out
 * (bf16 [T, num_heads, head_dim], row stride q_out_row_stride) and k, v into the
 * paged caches at slot_mapping[t] (-1 skips). If k_out is non-NULL the rotated k is
 * also written there (bf16 [T, num_kv_heads, head_dim], contiguous).               */
B200ASR_API int b200asr_qk_norm_rope_store(const void *qkv, int64_t qkv_row_stride,
                               const int64_t *positions, int32_t num_tokens,
                               int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                               const void *q_norm_weight, const void *k_norm_weight,
                               float eps, const float *cos_sin_cache, int32_t max_position,
                               void *q_out, int64_t q_out_row_stride, void *k_out,
                               void *k_cache, void *v_cache, const int32_t *slot_mapping,
                               int64_t num_slots, int32_t *error_flag,
                               b200asr_stream_t stream);

/* Replaces RMSNorm._norm / RMSNorm._add_norm (layers/layernorm.py:19-36).
 * x bf16 [rows, hidden]. With residual == NULL: out = norm(x) * w. Otherwise
 * s = x + residual (fp32); residual <- bf16(s) (in place); out = norm(s) * w.     */
B200ASR_API int b200asr_rmsnorm(const void *x, void *residual, const void *weight, float eps,
                    int32_t rows, int32_t hidden, void *out, b200asr_stream_t stream);

/* Replaces SiluAndMul (layers/activation.py:8-14): x bf16 [rows, 2*inner] ->
 * out bf16 [rows, inner] = silu(x[:, :inner]) * x[:, inner:].                    */
B200ASR_API int b200asr_silu_mul(const void *x, int32_t rows, int32_t inner, void *out,
                     b200asr_stream_t stream);

/* ---------------------------------------------------------------- attention ----
 * Split-K paged decode. Replaces the decode use of flash_attn_varlen_func with a
 * block table inside the CUDA-graph decode (layers/attention.py:96-107 with
 * max_seqlen_q = 1, engine/graph_runner.py:81-94). One query token per sequence:
 * q bf16 [batch, num_heads, head_dim] (row stride q_row_stride), context length of
 * sequence b = cu_seqlens_k[b+1] - cu_seqlens_k[b]; keys/values from the paged
 * caches bf16 [num_blocks, block_size, num_kv_heads, head_dim] through
 * block_tables i32 [batch, bt_stride]. out bf16 [batch, num_heads, head_dim].
 * Supported: head_dim 128, block_size 256, num_heads / num_kv_heads in {1,2,4,8},
 * num_kv_heads <= 8. workspace: device scratch of at least
 * b200asr_paged_decode_workspace_size(batch, max_seqlen_k, num_heads, head_dim)
 * bytes. max_seqlen_k <= 512 (with block_size % 64 == 0) selects a kernel with one CTA
 * per (sequence, KV head) and no split, the faster choice for short contexts; larger
 * bounds select the stream-K split over the whole batch.
 * Its first 4096 bytes hold per-sequence merge counters that must be zero
 * before the first call with that workspace; every completed call leaves them zero
 * (allocate it zero-filled once). A call that set an error bit in error_flag may
 * leave them non-zero: clear them before the workspace is used again. Calls sharing
 * a workspace must not overlap on the GPU.                                         */
B200ASR_API size_t b200asr_paged_decode_workspace_size(int32_t batch, int32_t max_seqlen_k,
                                           int32_t num_heads, int32_t head_dim);
B200ASR_API int b200asr_paged_decode(const void *q, int64_t q_row_stride, const void *k_cache,
                         const void *v_cache, int32_t num_blocks, int32_t block_size,
                         int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                         const int32_t *cu_seqlens_k, const int32_t *block_tables,
                         int32_t bt_stride, int32_t batch, int32_t max_seqlen_k, float scale,
                         void *out, int64_t out_row_stride, void *workspace,
                         size_t workspace_bytes, int32_t *error_flag, b200asr_stream_t stream);

/* Allocation-free variant of b200asr_paged_decode. No counterpart in the reference:
 * it exists for callers that cannot allocate device scratch -- an FFI host without a
 * CUDA allocator, a server whose memory pool is fully reserved up front, or code running
 * during CUDA-graph capture, where cudaMalloc is illegal. Same arguments and results as
 * b200asr_paged_decode minus the workspace: the split-K partials live in a static device
 * array of B200ASR_NOALLOC_SCRATCH_BYTES held by every GPU that loads the library.
 * Requests whose b200asr_paged_decode_workspace_size exceeds that limit are rejected
 * with B200ASR_ERR_WORKSPACE. The first call on each device resolves the array's address
 * (cudaGetSymbolAddress, with that device current): make it before any stream capture.
 * Every call clears the array's merge counters with cudaMemsetAsync on `stream` before
 * its kernel, so the clear is ordered with the launch on any stream and nothing a
 * failed call left behind reaches the next one. Every call shares the array, so calls
 * whose kernels overlap on the GPU race on it; serialise them (one stream, or one
 * replay at a time). Allocates nothing.                                             */
#define B200ASR_NOALLOC_SCRATCH_BYTES (12u << 20)
B200ASR_API int b200asr_paged_decode_noalloc(const void *q, int64_t q_row_stride,
                                 const void *k_cache, const void *v_cache, int32_t num_blocks,
                                 int32_t block_size, int32_t num_heads, int32_t num_kv_heads,
                                 int32_t head_dim, const int32_t *cu_seqlens_k,
                                 const int32_t *block_tables, int32_t bt_stride, int32_t batch,
                                 int32_t max_seqlen_k, float scale, void *out,
                                 int64_t out_row_stride, int32_t *error_flag,
                                 b200asr_stream_t stream);

/* Varlen causal GQA attention over the paged KV cache on tcgen05 tensor cores.
 * Replaces PagedAttention.forward (layers/attention.py:87-107) for prefill and mixed
 * batches: flash_attn_varlen_func(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k,
 * max_seqlen_q, max_seqlen_k, softmax_scale, causal=True, block_table) with the
 * causal mask aligned bottom-right (query i of a row with Lq queries and Lk keys
 * sees keys 0 .. Lk - Lq + i). Rows with one query are decode rows.
 * q bf16 [total_q, num_heads, head_dim]; out likewise. Supported: head_dim 128,
 * block_size a multiple of 64, num_heads == 2 * num_kv_heads.                     */
B200ASR_API int b200asr_paged_prefill(const void *q, int64_t q_row_stride, const void *k_cache,
                          const void *v_cache, int32_t num_blocks, int32_t block_size,
                          int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                          const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                          const int32_t *block_tables, int32_t bt_stride, int32_t batch,
                          int32_t total_q, int32_t max_seqlen_q, float scale, void *out,
                          int64_t out_row_stride, int32_t *error_flag,
                          b200asr_stream_t stream);

/* Bidirectional varlen attention inside segments on tcgen05 tensor cores. Replaces
 * VarlenSelfAttention.forward (layers/attention.py:121-139, called from
 * models/audio_encoder.py:58-67): flash_attn_varlen_func(q, k, v, cu_seqlens,
 * cu_seqlens, max_seqlen, max_seqlen, scale, causal=False).
 * q/k/v bf16 [total_tokens, num_heads, head_dim] with row strides (elements);
 * out bf16 likewise. Supported: head_dim 64, segments of at most 128 tokens
 * (the encoder's windows are 104).                                                */
B200ASR_API int b200asr_varlen_attention(const void *q, int64_t q_row_stride, const void *k,
                             int64_t k_row_stride, const void *v, int64_t v_row_stride,
                             const int32_t *cu_seqlens, int32_t num_segments,
                             int32_t total_tokens, int32_t max_seqlen, int32_t num_heads,
                             int32_t head_dim, float scale, void *out, int64_t out_row_stride,
                             int32_t *error_flag, b200asr_stream_t stream);

/* Element types of b200asr_pool_paged_decode. */
enum { B200ASR_DTYPE_BF16 = 0, B200ASR_DTYPE_F16 = 1, B200ASR_DTYPE_F32 = 2 };

/* One-token decode attention over a page pool in the TTS talker's layout, with the
 * current token's K/V written by the same launch. Replaces paged_attention_decode and
 * its Triton kernel (agent/qwen_tts_paged_attention.py:130-287, 383-516; the write of
 * its torch path, 519-532), as called by QwenPagedCache.paged_attention_decode
 * (agent/qwen_tts_outer_varlen.py:392-436).
 *   query       [batch, num_heads, 1, head_dim], strides q_stride_b / q_stride_h
 *   key_pool,
 *   value_pool  [num_pages, num_kv_heads, page_size, head_dim], strides kv_stride_p /
 *               kv_stride_h / kv_stride_s (shared by both pools)
 *   page_table  int64 [batch, table_stride]: row b's logical page p is physical page
 *               page_table[b][p], p < table_width (the padded width, the reference's
 *               kernel_page_count)
 *   seq_lens    int64 [batch], positive
 *   key_valid_mask  NULL or bool/uint8 [batch, valid_stride]: positions t < valid_len
 *               with a zero byte are not attended; positions >= valid_len are
 *   new_key,
 *   new_value   NULL, or [batch, num_kv_heads, 1, head_dim] with strides new_stride_b /
 *               new_stride_h (shared by both): stored at position seq_lens[b] - 1 of
 *               row b's pages and attended in the same pass
 *   out         [batch, num_heads, 1, head_dim], strides out_stride_b / out_stride_h
 * All strides in elements; head_dim is the unit stride. dtype B200ASR_DTYPE_* for
 * query, pools, new K/V and out alike; softmax and accumulation in fp32. Row b attends
 * positions < min(seq_lens[b], max_seq_len) (the reference's kernel_seq_len bound); a
 * row whose positions are all masked yields zeros. Supported: num_heads / num_kv_heads
 * in {1, 2, 4, 8}, head_dim * element size a multiple of 16 bytes and at most 1024,
 * 16-byte aligned query, pools and new K/V. tokens_per_cta: positions per CTA (0 =
 * chosen from the batch; else >= 64). workspace: at least
 * b200asr_pool_paged_decode_workspace_size(batch, num_heads, head_dim, max_seq_len)
 * bytes whose first bytes (merge counters) are zero before the first call; every call
 * leaves them zero, and calls sharing a workspace must not overlap on the GPU.
 * Device-side checks: a page outside the table or the pool raises
 * B200ASR_DEVERR_BLOCK (the position is skipped); seq_lens[b] <= 0 or > max_seq_len
 * raises B200ASR_DEVERR_LENGTH.                                                    */
B200ASR_API size_t b200asr_pool_paged_decode_workspace_size(int32_t batch, int32_t num_heads,
                                                int32_t head_dim, int32_t max_seq_len);
B200ASR_API int b200asr_pool_paged_decode(
    int32_t dtype, int32_t batch, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
    const void *query, int64_t q_stride_b, int64_t q_stride_h, void *key_pool, void *value_pool,
    int32_t num_pages, int32_t page_size, int64_t kv_stride_p, int64_t kv_stride_h,
    int64_t kv_stride_s, const int64_t *page_table, int64_t table_stride, int32_t table_width,
    const int64_t *seq_lens, const uint8_t *key_valid_mask, int64_t valid_stride,
    int32_t valid_len, const void *new_key, const void *new_value, int64_t new_stride_b,
    int64_t new_stride_h, void *out, int64_t out_stride_b, int64_t out_stride_h,
    int32_t max_seq_len, int32_t tokens_per_cta, float scale, void *workspace,
    size_t workspace_bytes, int32_t *error_flag, b200asr_stream_t stream);

/* ------------------------------------------------------------------ sampler ----
 * Replaces the greedy branch of Sampler.forward (layers/sampler.py:16-20):
 * out_ids[b] = argmax over logits[b, :vocab] (bf16, row stride in elements) in
 * fp32, first index on ties, NaN counted as the maximum.                          */
B200ASR_API int b200asr_greedy_argmax(const void *logits, int64_t row_stride, int32_t batch,
                          int32_t vocab, int64_t *out_ids, b200asr_stream_t stream);

/* -------------------------------------------------------- decode linears ----
 * The decoder's dense projections at decode batch sizes (qkv_proj / o_proj /
 * gate_up_proj + SiluAndMul / down_proj of models/qwen3.py:20-69 and
 * layers/activation.py:11-14, called from the CUDA-graph decode with 1..64 rows):
 *   y[r, j] = sum_k x[r, k] * w[j, k]   (bf16 in/out, fp32 accumulation), r < m <= 64
 * w is [n, k] row-major (k % 64 == 0, n % 128 == 0). With silu_inner = I > 0 the
 * weight is the fused [gate; up] of 2I rows (I % 64 == 0) and
 *   y[r, j] = bf16(bf16(silu(bf16(gate))) * bf16(up)),  j < I.
 * No workspace; launches thread-block clusters (split-K reduced on chip). A plain
 * projection with more 128-row tiles than two CTAs per SM (the lm_head) runs on a
 * persistent kernel that streams the tiles through one TMA ring; same results.       */
B200ASR_API int b200asr_linear_small(const void *x, int64_t x_row_stride, int32_t m, int32_t k,
                         const void *w, int32_t n, int32_t silu_inner, void *y,
                         int64_t y_row_stride, int32_t *error_flag, b200asr_stream_t stream);

/* ------------------------------------------- decode-step RMSNorm fusions ----
 * The decoder layer's add + RMSNorm (RMSNorm._add_norm / _norm, layers/layernorm.py:19-36)
 * split across the projections around it, for 1..64 rows. Between them a row is carried
 * as h (fp32, the pre-norm sum) plus ss[r][t] (fp32 [rows][hidden / 128], row-major): the
 * sum of h[r]^2 over columns 128t .. 128t + 127. The RMSNorm of that row is
 *   bf16(bf16(h * rsqrt(sum_t ss[r][t] / hidden + eps)) * weight)   (t summed in order).
 *
 * linear_small_add (o_proj / down_proj + the residual add of the next norm):
 *   h[r, j] = bf16(y[r, j]) + residual[r, j] (fp32), residual[r, j] <- bf16(h), h_out, ss_out
 *   with y = x w^T as in b200asr_linear_small (n % 128 == 0, n / 128 <= 64).
 * linear_small_norm (qkv_proj / gate_up_proj after the norm): y = RMSNorm(h) w^T, with
 *   silu_inner as in b200asr_linear_small; k = hidden, ss_tiles = hidden / 128 (hidden a
 *   multiple of 512 up to 4096: the normalised slice of each CTA must fit its ring).
 * linear_small_norm_qk_rope (qkv_proj + Qwen3Attention.forward's q/k norm and RoPE,
 *   models/qwen3.py:43-48, + the KV store of PagedAttention.forward, attention.py:90):
 *   the projection of RMSNorm(h), then per head exactly what b200asr_qk_norm_rope_store
 *   does (q heads to q_out, K and V into the cache at slot_mapping; slot -1 skipped);
 *   head_dim 128.
 * The three projections take an optional b200asr_l2_prefetch (NULL: none).
 * rms_stats: h and ss of x (+ residual, updated in place to bf16(x + residual)) -- the
 *   layer-0 input norm, whose input is the embedding.
 * norm_apply: out = RMSNorm of (h, ss) -- the model's final norm before lm_head.     */
/* Optional L2 prefetch issued by a fused projection before it waits on the previous
 * kernel (no reference counterpart; pure performance hint, results are unchanged):
 * the cached K/V rows (positions < length) of `batch` sequences of one layer, described
 * like b200asr_paged_decode's inputs (cu_seqlens_k NULL: none), and up to two
 * contiguous ranges (16-byte aligned, multiples of 16 bytes; NULL: none), e.g. the
 * next layer's weights. Out-of-pool block ids are skipped. The lengths and tables are
 * read before the wait: with PDL on they follow the contract of b200asr_set_pdl.     */
typedef struct {
  const int32_t *cu_seqlens_k;
  const int32_t *block_tables;
  int32_t bt_stride, batch, block_size, num_kv_heads, head_dim;
  const void *k_cache, *v_cache;
  int64_t num_slots;
  const void *range[2];
  int64_t range_bytes[2];
} b200asr_l2_prefetch;

B200ASR_API int b200asr_linear_small_add(const void *x, int64_t x_row_stride, int32_t m, int32_t k,
                             const void *w, int32_t n, void *residual,
                             int64_t residual_row_stride, float *h_out, int64_t h_row_stride,
                             float *ss_out, const b200asr_l2_prefetch *prefetch,
                             int32_t *error_flag, b200asr_stream_t stream);
B200ASR_API int b200asr_linear_small_norm(const float *h, int64_t h_row_stride, const float *ss,
                              int32_t ss_tiles, const void *norm_weight, float eps, int32_t m,
                              int32_t k, const void *w, int32_t n, int32_t silu_inner, void *y,
                              int64_t y_row_stride, const b200asr_l2_prefetch *prefetch,
                              int32_t *error_flag, b200asr_stream_t stream);
B200ASR_API int b200asr_linear_small_norm_qk_rope(
    const float *h, int64_t h_row_stride, const float *ss, int32_t ss_tiles,
    const void *norm_weight, float eps, int32_t m, int32_t k, const void *w, int32_t num_heads,
    int32_t num_kv_heads, int32_t head_dim, const void *q_norm_weight, const void *k_norm_weight,
    float qk_eps, const int64_t *positions, const float *cos_sin_cache, int32_t max_position,
    void *q_out, int64_t q_out_row_stride, void *k_cache, void *v_cache,
    const int32_t *slot_mapping, int64_t num_slots, const b200asr_l2_prefetch *prefetch,
    int32_t *error_flag, b200asr_stream_t stream);
/* linear_small_qk_rope: the same qkv_proj + q/k norm + RoPE + KV store on an already
 * normalised bf16 x [m, k] (row stride in elements) -- the unfused decode step's qkv_proj
 * (models/qwen3.py:43-48 after the layer's input norm) for models whose hidden size is
 * too large for the RMSNorm prologue; any k that is a multiple of 64.                 */
B200ASR_API int b200asr_linear_small_qk_rope(
    const void *x, int64_t x_row_stride, int32_t m, int32_t k, const void *w, int32_t num_heads,
    int32_t num_kv_heads, int32_t head_dim, const void *q_norm_weight, const void *k_norm_weight,
    float qk_eps, const int64_t *positions, const float *cos_sin_cache, int32_t max_position,
    void *q_out, int64_t q_out_row_stride, void *k_cache, void *v_cache,
    const int32_t *slot_mapping, int64_t num_slots, int32_t *error_flag,
    b200asr_stream_t stream);
B200ASR_API int b200asr_rms_stats(const void *x, void *residual, int32_t rows, int32_t hidden,
                      float *h_out, float *ss_out, b200asr_stream_t stream);
B200ASR_API int b200asr_norm_apply(const float *h, const float *ss, const void *weight, float eps,
                       int32_t rows, int32_t hidden, void *out, b200asr_stream_t stream);

/* ------------------------------------------------------------- mel frontend ----
 * Replaces AudioFrontend.__call__ (audio/frontend.py:71-94), the stock Whisper log-mel
 * extractor run per clip on the host: centred STFT (reflect pad 200), periodic Hann
 * window, n_fft 400, hop 160, power of bins 0..200, last frame dropped (n / 160 frames
 * for n samples), mel = filters^T power, log10(max(mel, 1e-10)), per clip
 * max(x, clip max - 8), (x + 4) / 4, rounded to bf16.
 *   waveform     fp32 clips laid end to end; cu_samples int64 [batch + 1] (each clip
 *                longer than 200 samples, else B200ASR_DEVERR_LENGTH)
 *   frame_start  int32 [batch + 1] prefix sums of n_b / 160; total_frames its last entry
 *   tables       fp32 [1200]: Hann window[400], cos[400], sin[400] of 2*pi*j/400
 *   mel_filters  fp32 [201][128]; filter_range int32 [128][2] first nonzero bin, count
 *   out          bf16 [128][out_stride]; clip b fills columns out_col[b] .. + frames_b
 *   workspace    >= b200asr_log_mel_workspace_size(batch, total_frames) bytes, 256-byte
 *                aligned (per-clip maxima + fp32 log-mel scratch)                     */
B200ASR_API size_t b200asr_log_mel_workspace_size(int32_t batch, int32_t total_frames);
B200ASR_API int b200asr_log_mel(const float *waveform, const int64_t *cu_samples,
                    const int32_t *frame_start, int32_t batch, int32_t total_frames,
                    const float *tables, const float *mel_filters, const int32_t *filter_range,
                    void *workspace, size_t workspace_bytes, void *out, int64_t out_stride,
                    const int32_t *out_col, int32_t *error_flag, b200asr_stream_t stream);

/* --------------------------------------------------------------- encoder front ----
 * Conv2d(kernel 3, stride 2, padding 1) + bias + GELU (erf form), the audio tower's
 * downsampler convolutions: conv2d1 / conv2d2 / conv2d3 each followed by F.gelu in
 * AudioEncoder (models/audio_encoder.py:145-175), which the reference runs as cuDNN
 * convolutions plus separate bias and GELU kernels.
 * x: channels-last bf16 [n][h][w][c_in] (for c_in = 1 simply [n][h][w]). Output
 * ho = (h - 1) / 2 + 1, wo = (w - 1) / 2 + 1; y[i * y_stride_n + oy * y_stride_y +
 * ox * y_stride_x + c] bf16 (channels contiguous, any pixel order -- e.g. [n][ox][oy][c]
 * for the conv_out projection that follows). Rounding as the reference: bf16
 * convolution output, bias added and rounded, GELU rounded.
 * packed_weight: b200asr_conv_weight_bytes(c_out, c_in) bytes written by
 * b200asr_conv_pack_weight from the module's [c_out][c_in][3][3] bf16 weight (once, at
 * load time). c_in = 1 runs a direct stencil on CUDA cores; c_in > 1 (a multiple of 8)
 * an implicit GEMM on tcgen05 with c_out a multiple of 32. error_flag records a
 * timed-out wait (B200ASR_DEVERR_TIMEOUT 16).                                        */
B200ASR_API size_t b200asr_conv_weight_bytes(int32_t c_out, int32_t c_in);
B200ASR_API int b200asr_conv_pack_weight(const void *weight, int32_t c_out, int32_t c_in,
                                         void *packed, b200asr_stream_t stream);
B200ASR_API int b200asr_conv3x3s2_gelu(const void *x, int32_t n, int32_t h, int32_t w,
                                       int32_t c_in, const void *packed_weight,
                                       const void *bias, int32_t c_out, void *y,
                                       int64_t y_stride_n, int64_t y_stride_y,
                                       int64_t y_stride_x, int32_t *error_flag,
                                       b200asr_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200ASR_H_ */
