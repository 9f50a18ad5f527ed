// Memory-bound per-token kernels of the decoder layer.
//
// store_kvcache        <- _store_kvcache_kernel / store_kvcache (layers/attention.py:31-67)
// qk_norm_rope_store   <- Qwen3Attention.forward q/k norm + RoPE (models/qwen3.py:43-48),
//                         RMSNorm._norm (layers/layernorm.py:19-25),
//                         RotaryEmbedding.forward (layers/rotary_embedding.py:9-32),
//                         fused with the KV store of PagedAttention.forward (attention.py:90)
// rmsnorm / add        <- RMSNorm._norm / RMSNorm._add_norm (layers/layernorm.py:19-36)
// silu_mul             <- SiluAndMul.forward (layers/activation.py:11-14)
//
// Rounding follows the reference's eager semantics: fp32 math, a bf16 rounding after
// the normalisation, another after the weight multiply, one after the rotation.
#include "common.cuh"

namespace b200asr {

// ------------------------------------------------------------------ KV store
// One warp copies one (token, K|V) row of `hidden` bf16 with 16-byte accesses.
__global__ void store_kvcache_kernel(const __nv_bfloat16 *__restrict__ key, int64_t key_stride,
                                     const __nv_bfloat16 *__restrict__ value,
                                     int64_t value_stride, __nv_bfloat16 *__restrict__ k_cache,
                                     __nv_bfloat16 *__restrict__ v_cache,
                                     const int32_t *__restrict__ slot_mapping, int num_tokens,
                                     int hidden, int64_t num_slots, int32_t *error_flag) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= 2 * num_tokens) return;
  const int t = warp >> 1;
  const bool is_v = warp & 1;
  const int64_t slot = slot_mapping[t];
  if (slot == -1) return;
  if (slot < 0 || slot >= num_slots) {
    if (lane == 0) raise_flag(error_flag, B200ASR_DEVERR_SLOT);
    return;
  }
  const uint4 *src = reinterpret_cast<const uint4 *>(is_v ? value + t * value_stride
                                                          : key + t * key_stride);
  uint4 *dst = reinterpret_cast<uint4 *>((is_v ? v_cache : k_cache) + slot * hidden);
  const int n16 = hidden >> 3;
  for (int i = lane; i < n16; i += 32) dst[i] = __ldg(src + i);
}

// ------------------------------------------------------ QK norm + RoPE + store
// A warp takes TPW consecutive (token, head-vector) tasks and issues all their loads
// before computing: TPW = 4 for prefill-sized batches, where it keeps more loads in flight
// per warp, and 1 for decode-sized ones, where spreading the few tasks over more warps is
// what keeps the latency down. Task j of a token: 0..H-1
// query heads, H..H+Hkv-1 key heads, H+Hkv..H+2Hkv-1 value heads (plain copy into the
// cache). Lane l holds EPL = head_dim/32 consecutive elements starting at l*EPL; the RoPE
// partner of element d (< D/2) is d + D/2, which lives in lane l ^ 16.

template <int EPL>
__device__ __forceinline__ void load_epl(const __nv_bfloat16 *src, float *x) {
  if constexpr (EPL == 4) {
    const uint2 u = *reinterpret_cast<const uint2 *>(src);
    x[0] = __uint_as_float(u.x << 16);
    x[1] = __uint_as_float(u.x & 0xffff0000u);
    x[2] = __uint_as_float(u.y << 16);
    x[3] = __uint_as_float(u.y & 0xffff0000u);
  } else {
    const uint32_t u = *reinterpret_cast<const uint32_t *>(src);
    x[0] = __uint_as_float(u << 16);
    x[1] = __uint_as_float(u & 0xffff0000u);
  }
}

template <int EPL>
__device__ __forceinline__ void store_epl(__nv_bfloat16 *dst, const float *o) {
  if constexpr (EPL == 4)
    *reinterpret_cast<uint2 *>(dst) = make_uint2(pack2(o[0], o[1]), pack2(o[2], o[3]));
  else
    *reinterpret_cast<uint32_t *>(dst) = pack2(o[0], o[1]);
}

template <int EPL, int TPW>
__global__ void qk_norm_rope_store_kernel(
    const __nv_bfloat16 *__restrict__ qkv, int64_t qkv_stride, const int64_t *__restrict__ positions,
    int num_tokens, int num_heads, int num_kv_heads, const __nv_bfloat16 *__restrict__ qw,
    const __nv_bfloat16 *__restrict__ kw, float eps, const float *__restrict__ cos_sin,
    int max_position, __nv_bfloat16 *__restrict__ q_out, int64_t q_out_stride,
    __nv_bfloat16 *__restrict__ k_out, __nv_bfloat16 *__restrict__ k_cache,
    __nv_bfloat16 *__restrict__ v_cache, const int32_t *__restrict__ slot_mapping,
    int64_t num_slots, int32_t *error_flag) {
  constexpr int D = EPL * 32;
  pdl_trigger();
  const int tasks_per_token = num_heads + 2 * num_kv_heads;
  const int64_t total = static_cast<int64_t>(num_tokens) * tasks_per_token;
  const int64_t first = ((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * TPW;
  const int lane = threadIdx.x & 31;
  if (first >= total) return;
  float wq[EPL], wk[EPL];  // static weights: before the wait
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    wq[e] = bf2f(qw[lane * EPL + e]);
    wk[e] = bf2f(kw[lane * EPL + e]);
  }
  pdl_wait();
  const int kv_hidden = num_kv_heads * D;

  int tok[TPW], head[TPW];
  float x[TPW][EPL];
  int64_t pos[TPW], slot[TPW];
#pragma unroll
  for (int i = 0; i < TPW; ++i) {  // every load of the warp's tasks first
    const int64_t task = first + i < total ? first + i : first;
    tok[i] = static_cast<int>(task / tasks_per_token);
    head[i] = static_cast<int>(task - static_cast<int64_t>(tok[i]) * tasks_per_token);
    load_epl<EPL>(qkv + tok[i] * qkv_stride + static_cast<int64_t>(head[i]) * D + lane * EPL, x[i]);
    pos[i] = positions[tok[i]];
    slot[i] = slot_mapping ? slot_mapping[tok[i]] : -1;
  }
#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    if (first + i >= total) break;
    const int t = tok[i], j = head[i];
    if (j >= num_heads + num_kv_heads) {  // value head: copy into the cache
      if (slot[i] == -1) continue;
      if (slot[i] < 0 || slot[i] >= num_slots) {
        if (lane == 0) raise_flag(error_flag, B200ASR_DEVERR_SLOT);
        continue;
      }
      const int h = j - num_heads - num_kv_heads;
      store_epl<EPL>(v_cache + slot[i] * kv_hidden + h * D + lane * EPL, x[i]);
      continue;
    }
    const bool is_q = j < num_heads;
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) ss += x[i][e] * x[i][e];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(D) + eps);
    float y[EPL];  // x.to(bf16), then .mul_(weight) rounded: paired conversions
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
      const float2 n = round2_bf16(x[i][e] * r, x[i][e + 1] * r);
      const float2 m = round2_bf16(n.x * (is_q ? wq[e] : wk[e]), n.y * (is_q ? wq[e + 1] : wk[e + 1]));
      y[e] = m.x;
      y[e + 1] = m.y;
    }
    int64_t p = pos[i];
    if (p < 0 || p >= max_position) {
      if (lane == 0) raise_flag(error_flag, B200ASR_DEVERR_POSITION);
      p = 0;
    }
    const float *cs = cos_sin + p * D;
    const bool first_half = lane < 16;
    float o[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, y[e], 16);
      const int dd = (lane & 15) * EPL + e;  // index within the half
      const float c = cs[dd], sn = cs[D / 2 + dd];
      // first*cos - second*sin | second*cos + first*sin, each product rounded (no FMA)
      o[e] = first_half ? __fsub_rn(__fmul_rn(y[e], c), __fmul_rn(partner, sn))
                        : __fadd_rn(__fmul_rn(y[e], c), __fmul_rn(partner, sn));
    }
    if (is_q) {
      store_epl<EPL>(q_out + t * q_out_stride + static_cast<int64_t>(j) * D + lane * EPL, o);
      continue;
    }
    const int h = j - num_heads;
    if (k_out != nullptr) store_epl<EPL>(k_out + static_cast<int64_t>(t) * kv_hidden + h * D + lane * EPL, o);
    if (slot[i] == -1) continue;
    if (slot[i] < 0 || slot[i] >= num_slots) {
      if (lane == 0) raise_flag(error_flag, B200ASR_DEVERR_SLOT);
      continue;
    }
    store_epl<EPL>(k_cache + slot[i] * kv_hidden + h * D + lane * EPL, o);
  }
}

// ------------------------------------------------------------------- RMSNorm
// One CTA per row; each thread owns 8 consecutive elements (hidden % 8 == 0).
__global__ void rmsnorm_kernel(const __nv_bfloat16 *__restrict__ x, __nv_bfloat16 *residual,
                               const __nv_bfloat16 *__restrict__ weight, float eps, int hidden,
                               __nv_bfloat16 *__restrict__ out) {
  __shared__ float red[32];
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int i8 = threadIdx.x;
  const bool active = i8 * 8 < hidden;
  float w[8];
  if (active) unpack8(*reinterpret_cast<const uint4 *>(weight + i8 * 8), w);  // static
  pdl_wait();
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (active) {
    unpack8(*reinterpret_cast<const uint4 *>(x + row * hidden + i8 * 8), v);
    if (residual != nullptr) {
      float r[8];
      uint4 *rp = reinterpret_cast<uint4 *>(residual + row * hidden + i8 * 8);
      unpack8(*rp, r);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += r[e];
      *rp = make_uint4(pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
  ss = warp_sum(ss);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (blockDim.x + 31) / 32 ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / static_cast<float>(hidden) + eps);
  if (!active) return;
  uint32_t y[4];  // bf16(bf16(v * r) * w), paired conversions; the second is the output
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 n = round2_bf16(v[2 * e] * r, v[2 * e + 1] * r);
    y[e] = pack2(n.x * w[2 * e], n.y * w[2 * e + 1]);
  }
  *reinterpret_cast<uint4 *>(out + row * hidden + i8 * 8) = make_uint4(y[0], y[1], y[2], y[3]);
}

// ------------------------------------------------------------------- SiLU*mul
__global__ void silu_mul_kernel(const __nv_bfloat16 *__restrict__ x, int64_t rows, int inner,
                                __nv_bfloat16 *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t n8 = rows * (inner / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / (inner / 8);
    const int c = static_cast<int>(i - row * (inner / 8)) * 8;
    float g[8], u[8];
    unpack8(*reinterpret_cast<const uint4 *>(x + row * 2 * inner + c), g);
    unpack8(*reinterpret_cast<const uint4 *>(x + row * 2 * inner + inner + c), u);
    uint32_t y[4];  // F.silu -> bf16, times u -> bf16 (paired conversions)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 sb = round2_bf16(g[2 * e] / (1.0f + expf(-g[2 * e])),
                                    g[2 * e + 1] / (1.0f + expf(-g[2 * e + 1])));
      y[e] = pack2(sb.x * u[2 * e], sb.y * u[2 * e + 1]);
    }
    *reinterpret_cast<uint4 *>(out + row * inner + c) = make_uint4(y[0], y[1], y[2], y[3]);
  }
}

}  // namespace b200asr

using namespace b200asr;

extern "C" int b200asr_store_kvcache(const void *key, int64_t key_row_stride, const void *value,
                                     int64_t value_row_stride, void *k_cache, void *v_cache,
                                     const int32_t *slot_mapping, int32_t num_tokens,
                                     int32_t num_kv_heads, int32_t head_dim, int64_t num_slots,
                                     int32_t *error_flag, b200asr_stream_t stream) {
  const int hidden = num_kv_heads * head_dim;
  B200_REQUIRE(num_tokens >= 0 && num_kv_heads >= 1 && head_dim >= 1 && num_slots >= 1,
               "store_kvcache: bad sizes");
  if (num_tokens == 0) return B200ASR_OK;
  B200_REQUIRE(key && value && k_cache && v_cache && slot_mapping, "store_kvcache: null pointer");
  B200_REQUIRE(hidden % 8 == 0 && key_row_stride % 8 == 0 && value_row_stride % 8 == 0 &&
                   aligned16(key) && aligned16(value) && aligned16(k_cache) && aligned16(v_cache),
               "store_kvcache: rows must be 16-byte aligned (hidden %d, strides %lld/%lld)",
               hidden, (long long)key_row_stride, (long long)value_row_stride);
  const int64_t threads = 2LL * num_tokens * 32;
  const int block = 256;
  B200_LAUNCH_CHECK_ERR(
      launch_kernel(store_kvcache_kernel, dim3(static_cast<unsigned>((threads + block - 1) / block)),
                    dim3(block), 0, stream, true, 1, static_cast<const __nv_bfloat16 *>(key),
                    key_row_stride, static_cast<const __nv_bfloat16 *>(value), value_row_stride,
                    static_cast<__nv_bfloat16 *>(k_cache), static_cast<__nv_bfloat16 *>(v_cache),
                    slot_mapping, num_tokens, hidden, num_slots, error_flag),
      "store_kvcache");
  return B200ASR_OK;
}

extern "C" int b200asr_qk_norm_rope_store(
    const void *qkv, int64_t qkv_row_stride, const int64_t *positions, int32_t num_tokens,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, const void *q_norm_weight,
    const void *k_norm_weight, float eps, const float *cos_sin_cache, int32_t max_position,
    void *q_out, int64_t q_out_row_stride, void *k_out, void *k_cache, void *v_cache,
    const int32_t *slot_mapping, int64_t num_slots, int32_t *error_flag,
    b200asr_stream_t stream) {
  B200_REQUIRE(num_tokens >= 0 && num_heads >= 1 && num_kv_heads >= 1 && max_position >= 1,
               "qk_norm_rope_store: bad sizes");
  B200_REQUIRE(head_dim == 64 || head_dim == 128, "qk_norm_rope_store: head_dim %d unsupported",
               head_dim);
  if (num_tokens == 0) return B200ASR_OK;
  B200_REQUIRE(qkv && positions && q_norm_weight && k_norm_weight && cos_sin_cache && q_out,
               "qk_norm_rope_store: null pointer");
  B200_REQUIRE(slot_mapping == nullptr || (k_cache && v_cache && num_slots >= 1),
               "qk_norm_rope_store: slot_mapping given without caches");
  B200_REQUIRE(qkv_row_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(qkv) & 7) == 0,
               "qk_norm_rope_store: qkv rows must be 8-byte aligned");
  B200_REQUIRE(q_out_row_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(q_out) & 7) == 0 &&
                   (reinterpret_cast<uintptr_t>(k_out) & 7) == 0 &&
                   (reinterpret_cast<uintptr_t>(k_cache) & 7) == 0 &&
                   (reinterpret_cast<uintptr_t>(v_cache) & 7) == 0,
               "qk_norm_rope_store: outputs must be 8-byte aligned (q_out rows too)");
  const int64_t tasks = static_cast<int64_t>(num_tokens) * (num_heads + 2 * num_kv_heads);
  const bool wide = num_tokens > 256;  // prefill-sized: 4 tasks per warp
  const int64_t warps = wide ? (tasks + 3) / 4 : tasks;
  const int block = 256;
  const unsigned grid = static_cast<unsigned>((warps * 32 + block - 1) / block);
  auto kfn = head_dim == 128 ? (wide ? qk_norm_rope_store_kernel<4, 4> : qk_norm_rope_store_kernel<4, 1>)
                             : (wide ? qk_norm_rope_store_kernel<2, 4> : qk_norm_rope_store_kernel<2, 1>);
  B200_LAUNCH_CHECK_ERR(
      launch_kernel(kfn, dim3(grid), dim3(block), 0, stream, true, 1,
                    static_cast<const __nv_bfloat16 *>(qkv), qkv_row_stride, positions, num_tokens,
                    num_heads, num_kv_heads, static_cast<const __nv_bfloat16 *>(q_norm_weight),
                    static_cast<const __nv_bfloat16 *>(k_norm_weight), eps, cos_sin_cache,
                    max_position, static_cast<__nv_bfloat16 *>(q_out), q_out_row_stride,
                    static_cast<__nv_bfloat16 *>(k_out), static_cast<__nv_bfloat16 *>(k_cache),
                    static_cast<__nv_bfloat16 *>(v_cache), slot_mapping, num_slots, error_flag),
      "qk_norm_rope_store");
  return B200ASR_OK;
}

extern "C" int b200asr_rmsnorm(const void *x, void *residual, const void *weight, float eps,
                               int32_t rows, int32_t hidden, void *out, b200asr_stream_t stream) {
  B200_REQUIRE(rows >= 0 && hidden >= 8 && hidden % 8 == 0 && hidden <= 8 * 1024,
               "rmsnorm: hidden %d must be a multiple of 8 in [8, 8192]", hidden);
  if (rows == 0) return B200ASR_OK;
  B200_REQUIRE(x && weight && out, "rmsnorm: null pointer");
  B200_REQUIRE(aligned16(x) && aligned16(weight) && aligned16(out) &&
                   (residual == nullptr || aligned16(residual)),
               "rmsnorm: tensors must be 16-byte aligned");
  const int threads = ((hidden / 8) + 31) / 32 * 32;
  B200_LAUNCH_CHECK_ERR(
      launch_kernel(rmsnorm_kernel, dim3(rows), dim3(threads), 0, stream, true, 1,
                    static_cast<const __nv_bfloat16 *>(x), static_cast<__nv_bfloat16 *>(residual),
                    static_cast<const __nv_bfloat16 *>(weight), eps, hidden,
                    static_cast<__nv_bfloat16 *>(out)),
      "rmsnorm");
  return B200ASR_OK;
}

extern "C" int b200asr_silu_mul(const void *x, int32_t rows, int32_t inner, void *out,
                                b200asr_stream_t stream) {
  B200_REQUIRE(rows >= 0 && inner >= 8 && inner % 8 == 0, "silu_mul: inner %d must be a multiple of 8",
               inner);
  if (rows == 0) return B200ASR_OK;
  B200_REQUIRE(x && out && aligned16(x) && aligned16(out), "silu_mul: null or unaligned pointer");
  const int64_t n8 = static_cast<int64_t>(rows) * (inner / 8);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n8 + 255) / 256, 148 * 32));
  B200_LAUNCH_CHECK_ERR(
      launch_kernel(silu_mul_kernel, dim3(grid), dim3(256), 0, stream, true, 1,
                    static_cast<const __nv_bfloat16 *>(x), static_cast<int64_t>(rows), inner,
                    static_cast<__nv_bfloat16 *>(out)),
      "silu_mul");
  return B200ASR_OK;
}
