// On-GPU ragged batch packers.
//
// pack_decoder        <- ModelRunner._prepare           (engine/model_runner.py:183-233)
// pack_decode_bucket  <- GraphRunner.run host staging   (engine/graph_runner.py:149-191)
// pack_audio          <- pack_audio_batch metadata      (audio/batcher.py:101-141,
//                                                        audio/tokens.py:30-52)
// audio_chunk_pad     <- AudioEncoder._chunk_and_pad    (models/audio_encoder.py:130-143)
// audio_gather_pos    <- AudioEncoder.forward "conv.gather" (models/audio_encoder.py:169-173):
//                        positional add + valid-token selection of the conv output
//
// The host uploads one compact per-request descriptor (a few int32 per request plus
// the concatenated block tables and query tokens); everything per token is derived
// here. Prefix sums over requests are block scans in shared memory; each CTA of a
// multi-CTA launch recomputes them (a batch holds at most 1024 requests) so no
// inter-CTA synchronisation is needed.
#include "common.cuh"

namespace b200asr {

constexpr int kPackThreads = 1024;

// Inclusive block scan of one int per thread (blockDim.x == kPackThreads).
__device__ int block_inclusive_scan(int v, int *warp_buf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) warp_buf[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = warp_buf[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    warp_buf[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v += warp_buf[warp - 1];
  __syncthreads();
  return v;
}

__device__ int block_max(int v, int *warp_buf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) warp_buf[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = warp_buf[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = max(w, __shfl_xor_sync(0xffffffffu, w, o));
    warp_buf[lane] = w;
  }
  __syncthreads();
  int r = warp_buf[0];
  __syncthreads();
  return r;
}

// ------------------------------------------------------------------ decoder

__global__ void __launch_bounds__(kPackThreads)
    pack_decoder_kernel(const int32_t *__restrict__ req_start, const int32_t *__restrict__ req_end,
                        const int32_t *__restrict__ table_off, const int32_t *__restrict__ table_len,
                        const int32_t *__restrict__ tables, const int32_t *__restrict__ query_tokens,
                        int batch, int total_tokens, int width, int block_size,
                        int64_t *__restrict__ input_ids, int64_t *__restrict__ positions,
                        int32_t *__restrict__ slot_mapping, int32_t *__restrict__ cu_seqlens_q,
                        int32_t *__restrict__ cu_seqlens_k, int32_t *__restrict__ max_seqlen,
                        int32_t *__restrict__ block_tables, int64_t *__restrict__ last_token_index) {
  __shared__ int s_cuq[kPackThreads + 1];
  __shared__ int s_start[kPackThreads];
  __shared__ int s_toff[kPackThreads];
  __shared__ int s_tlen[kPackThreads];
  __shared__ int warp_buf[32];
  const int tid = threadIdx.x;
  int qlen = 0, klen = 0;
  if (tid < batch) {
    s_start[tid] = req_start[tid];
    s_toff[tid] = table_off[tid];
    s_tlen[tid] = table_len[tid];
    klen = req_end[tid];
    qlen = klen - s_start[tid];
  }
  const int incl_q = block_inclusive_scan(qlen, warp_buf);
  const int incl_k = block_inclusive_scan(klen, warp_buf);
  if (tid < batch) s_cuq[tid + 1] = incl_q;
  if (tid == 0) s_cuq[0] = 0;
  const int mq = block_max(qlen, warp_buf);
  const int mk = block_max(klen, warp_buf);
  __syncthreads();

  if (blockIdx.x == 0) {
    if (tid < batch) {
      cu_seqlens_q[tid + 1] = incl_q;
      cu_seqlens_k[tid + 1] = incl_k;
      last_token_index[tid] = static_cast<int64_t>(incl_q) - 1;
    }
    if (tid == 0) {
      cu_seqlens_q[0] = 0;
      cu_seqlens_k[0] = 0;
      max_seqlen[0] = mq;
      max_seqlen[1] = mk;
    }
    for (int idx = tid; idx < batch * width; idx += blockDim.x) {
      const int b = idx / width, j = idx - b * width;
      block_tables[idx] = j < s_tlen[b] ? tables[s_toff[b] + j] : -1;
    }
  }

  // Per-token work, grid-strided across CTAs.
  for (int t = blockIdx.x * blockDim.x + tid; t < total_tokens; t += gridDim.x * blockDim.x) {
    int lo = 0, hi = batch - 1;  // largest b with s_cuq[b] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_cuq[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    const int pos = s_start[b] + (t - s_cuq[b]);
    const int blk = pos / block_size;
    input_ids[t] = static_cast<int64_t>(query_tokens[t]);
    positions[t] = pos;
    slot_mapping[t] = blk < s_tlen[b] ? tables[s_toff[b] + blk] * block_size + (pos - blk * block_size)
                                      : -1;
  }
}

// ------------------------------------------------------------ decode bucket

__global__ void __launch_bounds__(kPackThreads)
    pack_decode_bucket_kernel(const int32_t *__restrict__ lens, const int32_t *__restrict__ last_ids,
                              const int32_t *__restrict__ table_off,
                              const int32_t *__restrict__ table_len,
                              const int32_t *__restrict__ tables, int batch, int bucket,
                              int max_blocks, int block_size, int64_t *__restrict__ input_ids,
                              int64_t *__restrict__ positions, int32_t *__restrict__ slot_mapping,
                              int32_t *__restrict__ cu_seqlens_k,
                              int32_t *__restrict__ block_tables) {
  __shared__ int warp_buf[32];
  __shared__ int s_toff[kPackThreads];
  __shared__ int s_tlen[kPackThreads];
  const int tid = threadIdx.x;
  int klen = 0;
  if (tid < batch) {
    klen = lens[tid];
    s_toff[tid] = table_off[tid];
    s_tlen[tid] = table_len[tid];
  } else if (tid < bucket) {
    klen = 1;  // padding rows read one key (block 0, slot 0)
    s_toff[tid] = 0;
    s_tlen[tid] = 0;
  }
  const int incl = block_inclusive_scan(klen, warp_buf);
  if (tid < bucket) {
    cu_seqlens_k[tid + 1] = incl;
    if (tid < batch) {
      const int pos = klen - 1;
      const int blk = pos / block_size;
      input_ids[tid] = last_ids[tid];
      positions[tid] = pos;
      slot_mapping[tid] =
          blk < s_tlen[tid] ? tables[s_toff[tid] + blk] * block_size + (pos - blk * block_size) : -1;
    } else {
      input_ids[tid] = 0;
      positions[tid] = 0;
      slot_mapping[tid] = -1;
    }
  }
  if (tid == 0) cu_seqlens_k[0] = 0;
  __syncthreads();
  for (int idx = tid; idx < bucket * max_blocks; idx += blockDim.x) {
    const int b = idx / max_blocks, j = idx - b * max_blocks;
    block_tables[idx] = (b < batch && j < s_tlen[b]) ? tables[s_toff[b] + j] : 0;
  }
}

// -------------------------------------------------------------------- audio

__device__ __forceinline__ int conv_len(int n) { return (n - 1) / 2 + 1; }
__device__ __forceinline__ int after_cnn(int n) { return conv_len(conv_len(conv_len(n))); }

__global__ void __launch_bounds__(kPackThreads)
    pack_audio_kernel(const int32_t *__restrict__ mel_frames, int batch, int chunk_frames,
                      int window_tokens, int max_chunks, int max_windows,
                      int64_t *__restrict__ chunk_lengths, int64_t *__restrict__ chunk_valid_lens,
                      int32_t *__restrict__ chunk_start, int32_t *__restrict__ audio_token_lens,
                      int32_t *__restrict__ cu_seqlens, int32_t *__restrict__ counts,
                      int32_t *__restrict__ error_flag) {
  __shared__ int warp_buf[32];
  const int tid = threadIdx.x;
  int frames = 0, nchunks = 0, tokens = 0, nwin = 0, wmax = 0;
  if (tid < batch) {
    frames = mel_frames[tid];
    const int full = frames / chunk_frames, tail = frames - full * chunk_frames;
    nchunks = full + (tail > 0 ? 1 : 0);
    tokens = full * after_cnn(chunk_frames) + (tail > 0 ? after_cnn(tail) : 0);
    nwin = (tokens + window_tokens - 1) / window_tokens;
    wmax = min(tokens, window_tokens);
  }
  const int frame_end = block_inclusive_scan(frames, warp_buf);
  const int chunk_end = block_inclusive_scan(nchunks, warp_buf);
  const int tok_end = block_inclusive_scan(tokens, warp_buf);
  const int win_end = block_inclusive_scan(nwin, warp_buf);
  const int mx = block_max(wmax, warp_buf);
  // Totals live in the last request's thread; broadcast through shared memory.
  __shared__ int s_tot[2];
  if (tid == batch - 1) {
    s_tot[0] = chunk_end;
    s_tot[1] = win_end;
  }
  __syncthreads();
  const int total_chunks = s_tot[0], total_windows = s_tot[1];
  const bool overflow = total_chunks > max_chunks || total_windows > max_windows;
  if (tid == 0) {
    counts[0] = total_chunks;
    counts[1] = total_windows;
    counts[2] = mx;
    if (max_windows >= 0) cu_seqlens[0] = 0;
    if (overflow) raise_flag(error_flag, B200ASR_DEVERR_LENGTH);
  }
  if (tid >= batch || overflow) return;
  audio_token_lens[tid] = tokens;
  const int c0 = chunk_end - nchunks, f0 = frame_end - frames;
  for (int i = 0; i < nchunks; ++i) {
    const int len = min(chunk_frames, frames - i * chunk_frames);
    chunk_lengths[c0 + i] = len;
    chunk_valid_lens[c0 + i] = after_cnn(len);
    chunk_start[c0 + i] = f0 + i * chunk_frames;
  }
  const int w0 = win_end - nwin, t0 = tok_end - tokens;
  for (int j = 0; j < nwin; ++j) cu_seqlens[w0 + j + 1] = t0 + min((j + 1) * window_tokens, tokens);
}

__global__ void audio_chunk_pad_kernel(const __nv_bfloat16 *__restrict__ mel, int bins,
                                       int total_frames, const int32_t *__restrict__ chunk_start,
                                       const int64_t *__restrict__ chunk_lengths, int num_chunks,
                                       int chunk_frames, __nv_bfloat16 *__restrict__ padded) {
  const int64_t n = static_cast<int64_t>(num_chunks) * bins * chunk_frames;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i % chunk_frames);
    const int64_t row = i / chunk_frames;
    const int m = static_cast<int>(row % bins);
    const int c = static_cast<int>(row / bins);
    const int len = static_cast<int>(chunk_lengths[c]);
    const int f = chunk_start[c] + t;
    padded[i] = (t < len && f < total_frames) ? mel[static_cast<int64_t>(m) * total_frames + f]
                                              : __float2bfloat16_rn(0.f);
  }
}

// Valid-token gather of the conv front with the positional add, one warp per output row
// (16-byte accesses): row i < tokens is embed[src] + pos[src % tokens_per_chunk] with
// src = token_index[i], added in fp32 and rounded once to bf16 (torch's bf16 + bf16);
// rows [tokens, rows_out) are zero (the bucketed padding the encoder layers run over).
// An index outside embed's rows raises B200ASR_DEVERR_LENGTH and its row is zeroed.
__global__ void audio_gather_pos_kernel(const __nv_bfloat16 *__restrict__ embed,
                                        int64_t embed_rows, const __nv_bfloat16 *__restrict__ pos,
                                        int tokens_per_chunk,
                                        const int64_t *__restrict__ token_index, int tokens,
                                        int rows_out, int d, __nv_bfloat16 *__restrict__ out,
                                        int32_t *error_flag) {
  const int row = static_cast<int>((blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows_out) return;
  uint4 *dst = reinterpret_cast<uint4 *>(out + static_cast<int64_t>(row) * d);
  const int n8 = d >> 3;
  int64_t src = -1;
  if (row < tokens) {
    src = token_index[row];
    if (src < 0 || src >= embed_rows) {
      if (lane == 0) raise_flag(error_flag, B200ASR_DEVERR_LENGTH);
      src = -1;
    }
  }
  if (src < 0) {
    for (int i = lane; i < n8; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4 *e = reinterpret_cast<const uint4 *>(embed + src * d);
  const uint4 *p = reinterpret_cast<const uint4 *>(pos + (src % tokens_per_chunk) * d);
  for (int i = lane; i < n8; i += 32) {
    const uint4 a = e[i], b = p[i];
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    uint32_t y[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      y[k] = pack2(__uint_as_float(av[k] << 16) + __uint_as_float(bv[k] << 16),
                   __uint_as_float(av[k] & 0xffff0000u) + __uint_as_float(bv[k] & 0xffff0000u));
    dst[i] = make_uint4(y[0], y[1], y[2], y[3]);
  }
}

// Advances a decode-bucket descriptor by one generated token on the device: for every
// real row (non-empty block table) the length grows by one and the last token becomes
// the one just sampled. Lets consecutive decode-graph replays run without a host round
// trip when their block tables already cover the next positions.
__global__ void advance_decode_bucket_kernel(int32_t *__restrict__ lens,
                                             int32_t *__restrict__ last_ids,
                                             const int32_t *__restrict__ table_len,
                                             const int64_t *__restrict__ sampled, int bucket) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < bucket && table_len[i] > 0) {
    lens[i] += 1;
    last_ids[i] = static_cast<int32_t>(sampled[i]);
  }
}

}  // namespace b200asr

using namespace b200asr;

extern "C" int b200asr_pack_decoder(const int32_t *req_start, const int32_t *req_end,
                                    const int32_t *table_off, const int32_t *table_len,
                                    const int32_t *tables, const int32_t *query_tokens,
                                    int32_t batch, int32_t total_tokens, int32_t width,
                                    int32_t block_size, int64_t *input_ids, int64_t *positions,
                                    int32_t *slot_mapping, int32_t *cu_seqlens_q,
                                    int32_t *cu_seqlens_k, int32_t *max_seqlen,
                                    int32_t *block_tables, int64_t *last_token_index,
                                    b200asr_stream_t stream) {
  B200_REQUIRE(batch >= 1 && batch <= kPackThreads, "pack_decoder: batch %d not in [1, %d]",
               batch, kPackThreads);
  B200_REQUIRE(total_tokens >= 0 && width >= 1 && block_size >= 1,
               "pack_decoder: bad sizes (tokens %d, width %d, block %d)", total_tokens, width,
               block_size);
  B200_REQUIRE(req_start && req_end && table_off && table_len && tables && input_ids &&
                   positions && slot_mapping && cu_seqlens_q && cu_seqlens_k && max_seqlen &&
                   block_tables && last_token_index && (query_tokens || total_tokens == 0),
               "pack_decoder: null pointer");
  const int grid = max(1, min(148, (total_tokens + kPackThreads - 1) / kPackThreads));
  pack_decoder_kernel<<<grid, kPackThreads, 0, stream>>>(
      req_start, req_end, table_off, table_len, tables, query_tokens, batch, total_tokens, width,
      block_size, input_ids, positions, slot_mapping, cu_seqlens_q, cu_seqlens_k, max_seqlen,
      block_tables, last_token_index);
  B200_CUDA_LAUNCH_CHECK("pack_decoder");
  return B200ASR_OK;
}

extern "C" int b200asr_pack_decode_bucket(const int32_t *lens, const int32_t *last_ids,
                                          const int32_t *table_off, const int32_t *table_len,
                                          const int32_t *tables, int32_t batch, int32_t bucket,
                                          int32_t max_blocks, int32_t block_size,
                                          int64_t *input_ids, int64_t *positions,
                                          int32_t *slot_mapping, int32_t *cu_seqlens_k,
                                          int32_t *block_tables, b200asr_stream_t stream) {
  B200_REQUIRE(batch >= 0 && bucket >= batch && bucket >= 1 && bucket <= kPackThreads,
               "pack_decode_bucket: batch %d / bucket %d invalid", batch, bucket);
  B200_REQUIRE(max_blocks >= 1 && block_size >= 1, "pack_decode_bucket: bad table geometry");
  B200_REQUIRE(input_ids && positions && slot_mapping && cu_seqlens_k && block_tables &&
                   (batch == 0 || (lens && last_ids && table_off && table_len && tables)),
               "pack_decode_bucket: null pointer");
  pack_decode_bucket_kernel<<<1, kPackThreads, 0, stream>>>(
      lens, last_ids, table_off, table_len, tables, batch, bucket, max_blocks, block_size,
      input_ids, positions, slot_mapping, cu_seqlens_k, block_tables);
  B200_CUDA_LAUNCH_CHECK("pack_decode_bucket");
  return B200ASR_OK;
}

extern "C" int b200asr_advance_decode_bucket(int32_t *lens, int32_t *last_ids,
                                             const int32_t *table_len, const int64_t *sampled,
                                             int32_t bucket, b200asr_stream_t stream) {
  B200_REQUIRE(bucket >= 0, "advance_decode_bucket: negative bucket");
  if (bucket == 0) return B200ASR_OK;
  B200_REQUIRE(lens && last_ids && table_len && sampled, "advance_decode_bucket: null pointer");
  B200_LAUNCH_CHECK_ERR(launch_kernel(advance_decode_bucket_kernel, dim3((bucket + 127) / 128),
                                      dim3(128), 0, stream, true, 1, lens, last_ids, table_len,
                                      sampled, static_cast<int>(bucket)),
                        "advance_decode_bucket");
  return B200ASR_OK;
}

extern "C" int b200asr_pack_audio(const int32_t *mel_frames, int32_t batch, int32_t chunk_frames,
                                  int32_t window_tokens, int32_t max_chunks, int32_t max_windows,
                                  int64_t *chunk_lengths, int64_t *chunk_valid_lens,
                                  int32_t *chunk_start, int32_t *audio_token_lens,
                                  int32_t *cu_seqlens, int32_t *counts, int32_t *error_flag,
                                  b200asr_stream_t stream) {
  B200_REQUIRE(batch >= 1 && batch <= kPackThreads, "pack_audio: batch %d not in [1, %d]", batch,
               kPackThreads);
  B200_REQUIRE(chunk_frames >= 1 && window_tokens >= 1 && max_chunks >= 0 && max_windows >= 0,
               "pack_audio: bad geometry");
  B200_REQUIRE(mel_frames && chunk_lengths && chunk_valid_lens && chunk_start &&
                   audio_token_lens && cu_seqlens && counts,
               "pack_audio: null pointer");
  pack_audio_kernel<<<1, kPackThreads, 0, stream>>>(
      mel_frames, batch, chunk_frames, window_tokens, max_chunks, max_windows, chunk_lengths,
      chunk_valid_lens, chunk_start, audio_token_lens, cu_seqlens, counts, error_flag);
  B200_CUDA_LAUNCH_CHECK("pack_audio");
  return B200ASR_OK;
}

extern "C" int b200asr_audio_chunk_pad(const void *mel, int32_t bins, int32_t total_frames,
                                       const int32_t *chunk_start, const int64_t *chunk_lengths,
                                       int32_t num_chunks, int32_t chunk_frames, void *padded,
                                       b200asr_stream_t stream) {
  B200_REQUIRE(bins >= 1 && total_frames >= 0 && num_chunks >= 0 && chunk_frames >= 1,
               "audio_chunk_pad: bad sizes");
  if (num_chunks == 0) return B200ASR_OK;
  B200_REQUIRE(mel && chunk_start && chunk_lengths && padded, "audio_chunk_pad: null pointer");
  const int64_t n = static_cast<int64_t>(num_chunks) * bins * chunk_frames;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16));
  audio_chunk_pad_kernel<<<grid, 256, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(mel), bins, total_frames, chunk_start, chunk_lengths,
      num_chunks, chunk_frames, static_cast<__nv_bfloat16 *>(padded));
  B200_CUDA_LAUNCH_CHECK("audio_chunk_pad");
  return B200ASR_OK;
}

extern "C" int b200asr_audio_gather_pos(const void *embed, int64_t embed_rows, const void *pos,
                                        int32_t tokens_per_chunk, const int64_t *token_index,
                                        int32_t tokens, int32_t rows_out, int32_t d, void *out,
                                        int32_t *error_flag, b200asr_stream_t stream) {
  B200_REQUIRE(embed_rows >= 0 && tokens_per_chunk >= 1 && tokens >= 0 && rows_out >= tokens &&
                   d >= 8 && d % 8 == 0,
               "audio_gather_pos: bad sizes (tokens %d, rows_out %d, d %d)", tokens, rows_out, d);
  if (rows_out == 0) return B200ASR_OK;
  B200_REQUIRE(out && (tokens == 0 || (embed && pos && token_index)),
               "audio_gather_pos: null pointer");
  B200_REQUIRE(aligned16(out) && (tokens == 0 || (aligned16(embed) && aligned16(pos))),
               "audio_gather_pos: rows must be 16-byte aligned");
  const int64_t threads = static_cast<int64_t>(rows_out) * 32;
  audio_gather_pos_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(embed), embed_rows,
      static_cast<const __nv_bfloat16 *>(pos), tokens_per_chunk, token_index, tokens, rows_out, d,
      static_cast<__nv_bfloat16 *>(out), error_flag);
  B200_CUDA_LAUNCH_CHECK("audio_gather_pos");
  return B200ASR_OK;
}
