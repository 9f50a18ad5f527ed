// Log-mel audio frontend on the GPU.
//
// Replaces the host-side AudioFrontend.__call__ (audio/frontend.py:71-94 of the
// reference), which runs the stock Whisper feature extractor (transformers
// WhisperFeatureExtractor, its torch path) one clip at a time:
//   centred STFT with reflect padding of n_fft/2, periodic Hann window, n_fft 400,
//   hop 160, power |X|^2 of bins 0..200, the last STFT frame dropped (so a clip of n
//   samples has n / 160 frames); mel = filters^T power (128 filters);
//   log10(max(mel, 1e-10)); per clip x = max(x, clip_max - 8); x = (x + 4) / 4.
// The features land, rounded to bf16, directly in the encoder's packed [128, frames]
// input at each clip's column offset, so waveforms are the only host-to-device copy.
//
// log_mel_kernel: a CTA takes 4 consecutive frames of the packed batch. The windowed
// frames sit in shared memory; thread f forms DFT bin f of all 4 frames from a 400-entry
// twiddle table (angle index f*k mod 400), so every twiddle load feeds 8 FMAs. Each mel
// filter is a triangle over a short run of bins; the host passes that run per filter and
// the product skips the zeros. The clip's running maximum is an atomicMax on an
// order-preserving integer image of the float.
// log_mel_finish_kernel: 32-frame tiles: clamp, scale, transpose, round to bf16.
#include "common.cuh"

namespace b200asr {

constexpr int kMelFft = 400;
constexpr int kMelHop = 160;
constexpr int kMelBins = kMelFft / 2 + 1;  // 201
constexpr int kMel = 128;
constexpr int kMelFpc = 4;  // frames per CTA
constexpr int kMelThreads = 256;
constexpr size_t kMelMaxAlign = 256;

// Monotonic map float -> uint32 (and back): a < b  <=>  key(a) < key(b).
__device__ __forceinline__ unsigned order_key(float x) {
  const unsigned u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_order_key(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct MelArgs {
  const float *wave;             // concatenated clips, fp32
  const int64_t *cu_samples;     // [batch + 1]
  const int32_t *frame_start;    // [batch + 1] prefix of n_b / 160
  int batch;
  int total_frames;
  const float *tables;           // window[400], cos[400], sin[400] of 2*pi*j/400
  const float *filters;          // [201][128]
  const int32_t *filter_range;   // [128][2]: first bin and count of nonzero bins
  float *logmel;                 // [total_frames][128] scratch
  unsigned *clip_max;            // [batch] order keys, zero before log_mel_kernel
  __nv_bfloat16 *out;            // [128][out_stride]
  int64_t out_stride;
  const int32_t *out_col;        // [batch] first output column of each clip
  int32_t *error_flag;
};

__device__ __forceinline__ int clip_of(const int32_t *frame_start, int batch, int g) {
  int lo = 0, hi = batch - 1;  // largest b with frame_start[b] <= g
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (frame_start[mid] <= g) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kMelThreads) log_mel_kernel(const MelArgs a) {
  __shared__ float s_tab[3 * kMelFft];
  __shared__ float s_x[kMelFpc][kMelFft];
  __shared__ float s_pow[kMelFpc][kMelBins + 3];
  __shared__ int s_clip[kMelFpc];
  const int tid = threadIdx.x;
  const int g0 = blockIdx.x * kMelFpc;
  for (int i = tid; i < 3 * kMelFft; i += kMelThreads) s_tab[i] = a.tables[i];
  if (tid < kMelFpc) {
    const int g = g0 + tid;
    s_clip[tid] = g < a.total_frames ? clip_of(a.frame_start, a.batch, g) : -1;
  }
  __syncthreads();
  for (int idx = tid; idx < kMelFpc * kMelFft; idx += kMelThreads) {
    const int j = idx / kMelFft, k = idx % kMelFft;
    const int b = s_clip[j];
    float v = 0.f;
    if (b >= 0) {
      const int t = g0 + j - a.frame_start[b];
      const int64_t base = a.cu_samples[b], n = a.cu_samples[b + 1] - base;
      int64_t i = static_cast<int64_t>(t) * kMelHop + k - kMelFft / 2;  // centred frame
      if (i < 0) i = -i;                                                // reflect
      if (i >= n) i = 2 * (n - 1) - i;
      if (i >= 0 && i < n) {
        v = a.wave[base + i] * s_tab[k];
      } else {
        raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);  // clip too short to reflect
      }
    }
    s_x[j][k] = v;
  }
  __syncthreads();
  if (tid < kMelBins) {
    const int f = tid;
    float re[kMelFpc], im[kMelFpc];
#pragma unroll
    for (int j = 0; j < kMelFpc; ++j) re[j] = im[j] = 0.f;
    int ang = 0;  // f * k mod 400
    for (int k = 0; k < kMelFft; ++k) {
      const float c = s_tab[kMelFft + ang], s = s_tab[2 * kMelFft + ang];
#pragma unroll
      for (int j = 0; j < kMelFpc; ++j) {
        const float x = s_x[j][k];
        re[j] = fmaf(x, c, re[j]);
        im[j] = fmaf(-x, s, im[j]);
      }
      ang += f;
      if (ang >= kMelFft) ang -= kMelFft;
    }
#pragma unroll
    for (int j = 0; j < kMelFpc; ++j) s_pow[j][f] = re[j] * re[j] + im[j] * im[j];
  }
  __syncthreads();
  const int m = tid & (kMel - 1);
  const int lo = a.filter_range[2 * m], cnt = a.filter_range[2 * m + 1];
  for (int j = tid / kMel; j < kMelFpc; j += kMelThreads / kMel) {
    const int b = s_clip[j];
    if (b < 0) continue;  // uniform per warp: a warp's 32 threads share j
    float acc = 0.f;
    for (int q = 0; q < cnt; ++q) acc = fmaf(a.filters[(lo + q) * kMel + m], s_pow[j][lo + q], acc);
    const float lg = log10f(fmaxf(acc, 1e-10f));
    a.logmel[static_cast<int64_t>(g0 + j) * kMel + m] = lg;
    const float wm = warp_max(lg);
    if ((tid & 31) == 0) atomicMax(a.clip_max + b, order_key(wm));
  }
}

__global__ void __launch_bounds__(kMelThreads) log_mel_finish_kernel(const MelArgs a) {
  __shared__ float tile[32][kMel + 1];
  __shared__ int64_t s_col[32];
  __shared__ float s_floor[32];
  const int tid = threadIdx.x;
  const int g0 = blockIdx.x * 32;
  if (tid < 32) {
    const int g = g0 + tid;
    if (g < a.total_frames) {
      const int b = clip_of(a.frame_start, a.batch, g);
      s_col[tid] = static_cast<int64_t>(a.out_col[b]) + (g - a.frame_start[b]);
      s_floor[tid] = from_order_key(a.clip_max[b]) - 8.0f;
    } else {
      s_col[tid] = -1;
      s_floor[tid] = 0.f;
    }
  }
  for (int idx = tid; idx < 32 * kMel; idx += kMelThreads) {
    const int r = idx / kMel, m = idx % kMel;
    tile[r][m] = g0 + r < a.total_frames ? a.logmel[static_cast<int64_t>(g0 + r) * kMel + m] : 0.f;
  }
  __syncthreads();
  for (int idx = tid; idx < 32 * kMel; idx += kMelThreads) {
    const int m = idx / 32, r = idx % 32;
    if (s_col[r] < 0) continue;
    const float v = (fmaxf(tile[r][m], s_floor[r]) + 4.0f) * 0.25f;
    a.out[m * a.out_stride + s_col[r]] = __float2bfloat16_rn(v);
  }
}

size_t mel_align(size_t x) { return (x + kMelMaxAlign - 1) / kMelMaxAlign * kMelMaxAlign; }

}  // namespace b200asr

using namespace b200asr;

extern "C" size_t b200asr_log_mel_workspace_size(int32_t batch, int32_t total_frames) {
  if (batch <= 0 || total_frames < 0) return 0;
  return mel_align(static_cast<size_t>(batch) * sizeof(unsigned)) +
         static_cast<size_t>(total_frames) * kMel * sizeof(float);
}

extern "C" int b200asr_log_mel(const float *waveform, const int64_t *cu_samples,
                               const int32_t *frame_start, int32_t batch, int32_t total_frames,
                               const float *tables, const float *mel_filters,
                               const int32_t *filter_range, void *workspace,
                               size_t workspace_bytes, void *out, int64_t out_stride,
                               const int32_t *out_col, int32_t *error_flag,
                               b200asr_stream_t stream) {
  B200_REQUIRE(batch >= 0 && total_frames >= 0, "log_mel: negative batch or frame count");
  if (batch == 0 || total_frames == 0) return B200ASR_OK;
  B200_REQUIRE(waveform && cu_samples && frame_start && tables && mel_filters && filter_range &&
                   workspace && out && out_col,
               "log_mel: null pointer");
  B200_REQUIRE(out_stride >= 1, "log_mel: bad output stride");
  const size_t need = b200asr_log_mel_workspace_size(batch, total_frames);
  if (workspace_bytes < need) {
    set_error("log_mel: workspace %zu bytes < %zu needed", workspace_bytes, need);
    return B200ASR_ERR_WORKSPACE;
  }
  B200_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & (kMelMaxAlign - 1)) == 0,
               "log_mel: workspace must be 256-byte aligned");
  MelArgs a{};
  a.wave = waveform;
  a.cu_samples = cu_samples;
  a.frame_start = frame_start;
  a.batch = batch;
  a.total_frames = total_frames;
  a.tables = tables;
  a.filters = mel_filters;
  a.filter_range = filter_range;
  a.clip_max = static_cast<unsigned *>(workspace);
  a.logmel = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) +
                                       mel_align(static_cast<size_t>(batch) * sizeof(unsigned)));
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.out_stride = out_stride;
  a.out_col = out_col;
  a.error_flag = error_flag;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(a.clip_max, 0, static_cast<size_t>(batch) * sizeof(unsigned), st);
  if (e != cudaSuccess) {
    set_error("log_mel: memset failed: %s", cudaGetErrorString(e));
    return B200ASR_ERR_CUDA;
  }
  log_mel_kernel<<<(total_frames + kMelFpc - 1) / kMelFpc, kMelThreads, 0, st>>>(a);
  B200_CUDA_LAUNCH_CHECK("log_mel");
  log_mel_finish_kernel<<<(total_frames + 31) / 32, kMelThreads, 0, st>>>(a);
  B200_CUDA_LAUNCH_CHECK("log_mel_finish");
  return B200ASR_OK;
}
