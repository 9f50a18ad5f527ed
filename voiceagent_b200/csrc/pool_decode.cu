// One-token paged decode attention over a page pool in the TTS talker's layout
// [pages, kv_heads, page_size, head_dim], with the current token's K/V written into the
// pool by the same launch.
//
// Replaces paged_attention_decode and its _paged_decode_attention_kernel
// (agent/qwen_tts_paged_attention.py:130-287 kernel, 383-516 launcher, 519-532 the
// current-token write of its torch path). Same contract: strided query [B, H, 1, D],
// int64 page table and lengths, optional key-valid mask (columns beyond its width are
// valid), optional new key/value [B, H_kv, 1, D] stored at position seq_len - 1 and
// attended in the same pass, attention over positions < min(seq_len, max_seq_len), a row
// without a valid key yields zeros. bf16, fp16 and fp32 elements.
//
// Design. Group size G = H / H_kv is small (2 for the talker) and the work is a stream
// over the row's K/V pages: about one FMA per byte, HBM-bound, so the kernel runs on the
// CUDA cores with 16-byte loads rather than on the tensor cores. One CTA (4 warps) owns
// one (row, KV head, chunk of positions) and serves all G query heads of that KV head, so
// every K/V byte is read once. A token's row of D elements is spread over lpt lanes
// (16 bytes each: 16 lanes for bf16 D = 128); a warp covers 32 / lpt tokens per step and
// each lane group keeps its own online softmax; groups and warps merge at the end, and
// the chunks of a row merge in the CTA that finishes last (a counter per (row, KV head)
// in the workspace), so one launch does everything. Chunks are sized from the batch so
// the grid gives every SM several CTAs.
#include <cuda_fp16.h>

#include "common.cuh"

namespace b200asr {
namespace {

constexpr int kPoolThreads = 128;
constexpr int kPoolWarps = kPoolThreads / 32;
constexpr int kPoolMinChunk = 64;

struct PoolArgs {
  const void *q;
  int64_t q_sb, q_sh;  // element strides of query rows / heads
  void *kp, *vp;
  int64_t sp, sh, ss;  // pool strides: page, head, position
  int32_t num_pages, page_size, page_shift;  // page_shift = log2(page_size) or -1
  const int64_t *table;
  int64_t table_stride;
  int32_t table_width;
  const int64_t *seq_lens;
  const uint8_t *valid;
  int64_t valid_stride;
  int32_t valid_len;
  const void *nk, *nv;
  int64_t n_sb, n_sh;
  void *out;
  int64_t o_sb, o_sh;
  int32_t num_kv_heads, head_dim, nvr, lpt_log2;
  int32_t max_seq_len, chunk, max_splits;
  int32_t pages_cap;  // page-offset slots staged per CTA (chunk / page_size + 2)
  float scale_log2;
  int *counters;
  float *ws;
  int32_t *error_flag;
};

template <typename T>
struct Vec16;
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int E = 8;
  static __device__ __forceinline__ void to_float(const uint4 &v, float *f) { unpack8(v, f); }
  static __device__ __forceinline__ void put(__nv_bfloat16 *p, float x) { *p = __float2bfloat16_rn(x); }
};
template <>
struct Vec16<__half> {
  static constexpr int E = 8;
  static __device__ __forceinline__ void to_float(const uint4 &v, float *f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
      const float2 x = __half22float2(h);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
  static __device__ __forceinline__ void put(__half *p, float x) { *p = __float2half_rn(x); }
};
template <>
struct Vec16<float> {
  static constexpr int E = 4;
  static __device__ __forceinline__ void to_float(const uint4 &v, float *f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  static __device__ __forceinline__ void put(float *p, float x) { *p = x; }
};

// 16-byte streaming load through the non-coherent path without L1 allocation. Pool
// bytes written by this launch (the current token) are never read back by it: the
// lanes that attend that position read the caller's new_key / new_value instead.
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// Element offset of position pos of row b in a pool (without the head term), or -1
// (with B200ASR_DEVERR_BLOCK raised) when the logical page lies outside the table or the
// physical page outside the pool.
__device__ __forceinline__ int64_t pool_offset(const PoolArgs &a, int b, int64_t pos) {
  const int64_t pi = a.page_shift >= 0 ? (pos >> a.page_shift) : pos / a.page_size;
  if (pi >= a.table_width) {
    raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
    return -1;
  }
  const int64_t page = __ldg(a.table + b * a.table_stride + pi);
  if (page < 0 || page >= a.num_pages) {
    raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
    return -1;
  }
  return page * a.sp + (pos - pi * a.page_size) * a.ss;
}

template <typename T, int G, int NPL>
__global__ void __launch_bounds__(kPoolThreads) pool_decode_kernel(const PoolArgs a) {
  using V = Vec16<T>;
  constexpr int E = V::E;
  // tokens in flight per lane group and step (fewer where the accumulators are large)
  constexpr int U = G * NPL <= 2 ? 4 : (G * NPL <= 8 ? 2 : 1);
  // [kPoolWarps][G][head_dim + 2] merge rows | int64 [pages_cap] page offsets | u8 [chunk]
  extern __shared__ float s_red[];
  __shared__ int s_last;

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lg = a.lpt_log2, lpt = 1 << lg, tpw = 32 >> lg;
  const int sub = lane & (lpt - 1), slot = lane >> lg;
  const int D = a.head_dim, rowf = D + 2;

  const int64_t seq = a.seq_lens[b];
  const int L = seq <= 0 ? 0 : static_cast<int>(min(seq, static_cast<int64_t>(a.max_seq_len)));
  if (split == 0 && kvh == 0 && tid == 0 && (seq <= 0 || seq > a.max_seq_len))
    raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);
  const int nsplit = L > 0 ? (L + a.chunk - 1) / a.chunk : 1;
  if (split >= nsplit) return;

  const T *nk = static_cast<const T *>(a.nk);
  const T *nv = static_cast<const T *>(a.nv);
  const bool has_new = nk != nullptr;
  const int64_t pos_new = seq - 1;
  const int64_t new_off = static_cast<int64_t>(b) * a.n_sb + static_cast<int64_t>(kvh) * a.n_sh;
  T *kp = static_cast<T *>(a.kp);
  T *vp = static_cast<T *>(a.vp);
  const int64_t head_off = static_cast<int64_t>(kvh) * a.sh;

  // The current token's K and V go into the pool once per (row, KV head): by the CTA
  // whose chunk holds that position (or chunk 0 when max_seq_len cuts it off).
  if (has_new && seq > 0) {
    const int writer = pos_new < L ? static_cast<int>(pos_new / a.chunk) : 0;
    if (split == writer && tid < 2 * a.nvr) {
      const int64_t off = pool_offset(a, b, pos_new);
      if (off >= 0) {
        const bool is_v = tid >= a.nvr;
        const int v = is_v ? tid - a.nvr : tid;
        const T *src = (is_v ? nv : nk) + new_off + v * E;
        T *dst = (is_v ? vp : kp) + off + head_off + v * E;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
      }
    }
  }

  // This lane's slice of the G query heads, pre-scaled for exp2.
  const T *q = static_cast<const T *>(a.q);
  float qf[G][NPL][E];
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int v = sub + j * lpt;
      if (v < a.nvr) {
        float t[E];
        V::to_float(*reinterpret_cast<const uint4 *>(
                        q + b * a.q_sb + static_cast<int64_t>(kvh * G + g) * a.q_sh + v * E),
                    t);
#pragma unroll
        for (int e = 0; e < E; ++e) qf[g][j][e] = t[e] * a.scale_log2;
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) qf[g][j][e] = 0.f;
      }
    }
  }

  float m[G], l[G], acc[G][NPL][E];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < NPL; ++j)
#pragma unroll
      for (int e = 0; e < E; ++e) acc[g][j][e] = 0.f;
  }

  const int t0 = split * a.chunk;
  const int t1 = min(L, t0 + a.chunk);

  // Stage this chunk's page offsets (element offset of the page plus the KV head, or -1
  // for a page outside the table or the pool) and per-position attend bytes in shared
  // memory, so the per-token addresses below need no global round trip and a step's
  // loads can all be in flight at once.
  int64_t *s_off = reinterpret_cast<int64_t *>(s_red + kPoolWarps * G * rowf);
  uint8_t *s_ok = reinterpret_cast<uint8_t *>(s_off + a.pages_cap);
  const int p0 = a.page_shift >= 0 ? (t0 >> a.page_shift) : t0 / a.page_size;
  if (t1 > t0) {
    const int p_last = a.page_shift >= 0 ? ((t1 - 1) >> a.page_shift) : (t1 - 1) / a.page_size;
    for (int i = tid; i <= p_last - p0; i += kPoolThreads) {
      const int pi = p0 + i;
      int64_t off = -1;
      if (pi < a.table_width) {
        const int64_t page = __ldg(a.table + b * a.table_stride + pi);
        if (page >= 0 && page < a.num_pages) off = page * a.sp + head_off;
      }
      s_off[i] = off;
    }
    for (int i = tid; i < t1 - t0; i += kPoolThreads) {
      const int t = t0 + i;
      s_ok[i] = (a.valid != nullptr && t < a.valid_len)
                    ? static_cast<uint8_t>(__ldg(a.valid + b * a.valid_stride + t) != 0)
                    : static_cast<uint8_t>(1);
    }
  }
  __syncthreads();

  const int step = kPoolWarps * tpw;
  for (int base = t0 + warp * tpw; base < t1; base += U * step) {  // warp-uniform bound
    // addresses of this step's U tokens (shared-memory lookups only) ...
    const T *kptr[U], *vptr[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = base + u * step + slot;
      ok[u] = t < t1 && s_ok[t - t0] != 0;
      kptr[u] = nk;
      vptr[u] = nv;
      if (ok[u] && !(has_new && t == pos_new)) {
        const int pi = a.page_shift >= 0 ? (t >> a.page_shift) : t / a.page_size;
        const int64_t off = s_off[pi - p0];
        if (off < 0) {
          raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
          ok[u] = false;
        } else {
          const int64_t row = off + static_cast<int64_t>(t - pi * a.page_size) * a.ss;
          kptr[u] = kp + row;
          vptr[u] = vp + row;
        }
      } else if (ok[u]) {
        kptr[u] = nk + new_off;
        vptr[u] = nv + new_off;
      }
    }
    // ... then all of their loads back to back
    uint4 kr[U][NPL], vr[U][NPL];
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int j = 0; j < NPL; ++j) {
        const int v = sub + j * lpt;
        if (ok[u] && v < a.nvr) {
          kr[u][j] = ld_stream16(kptr[u] + v * E);
          vr[u][j] = ld_stream16(vptr[u] + v * E);
        } else {
          kr[u][j] = make_uint4(0, 0, 0, 0);
          vr[u][j] = make_uint4(0, 0, 0, 0);
        }
      }
    }

    float s[U][G];
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int g = 0; g < G; ++g) s[u][g] = 0.f;
#pragma unroll
      for (int j = 0; j < NPL; ++j) {
        float kf[E];
        V::to_float(kr[u][j], kf);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int e = 0; e < E; ++e) s[u][g] = fmaf(qf[g][j][e], kf[e], s[u][g]);
      }
    }
    for (int o = 1; o < lpt; o <<= 1) {
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int g = 0; g < G; ++g) s[u][g] += __shfl_xor_sync(0xffffffffu, s[u][g], o);
    }

#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mc = -INFINITY;
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (ok[u]) mc = fmaxf(mc, s[u][g]);
      const float mn = fmaxf(m[g], mc);
      if (mn == -INFINITY) continue;  // nothing valid in this lane group yet
      const float corr = exp2f(m[g] - mn);  // 0 while m is still -inf
      float p[U], psum = 0.f;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        p[u] = ok[u] ? exp2f(s[u][g] - mn) : 0.f;
        psum += p[u];
      }
      l[g] = l[g] * corr + psum;
#pragma unroll
      for (int j = 0; j < NPL; ++j) {
#pragma unroll
        for (int e = 0; e < E; ++e) acc[g][j][e] *= corr;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float vf[E];
          V::to_float(vr[u][j], vf);
#pragma unroll
          for (int e = 0; e < E; ++e) acc[g][j][e] = fmaf(p[u], vf[e], acc[g][j][e]);
        }
      }
      m[g] = mn;
    }
  }

  // Merge the lane groups of each warp (lanes that differ in the bits above lg).
  for (int o = lpt; o < 32; o <<= 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[g], o);
      const float lo = __shfl_xor_sync(0xffffffffu, l[g], o);
      const float mn = fmaxf(m[g], mo);
      const float c1 = m[g] == -INFINITY ? 0.f : exp2f(m[g] - mn);
      const float c2 = mo == -INFINITY ? 0.f : exp2f(mo - mn);
      l[g] = l[g] * c1 + lo * c2;
#pragma unroll
      for (int j = 0; j < NPL; ++j)
#pragma unroll
        for (int e = 0; e < E; ++e)
          acc[g][j][e] = acc[g][j][e] * c1 + __shfl_xor_sync(0xffffffffu, acc[g][j][e], o) * c2;
      m[g] = mn;
    }
  }
  if (slot == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float *r = s_red + (warp * G + g) * rowf;
      if (sub == 0) {
        r[0] = m[g];
        r[1] = l[g];
      }
#pragma unroll
      for (int j = 0; j < NPL; ++j) {
        const int v = sub + j * lpt;
        if (v < a.nvr)
#pragma unroll
          for (int e = 0; e < E; ++e) r[2 + v * E + e] = acc[g][j][e];
      }
    }
  }
  __syncthreads();

  // Merge the warps; a single-chunk row is finished here.
  T *out = static_cast<T *>(a.out);
  const int64_t pair = static_cast<int64_t>(b) * a.num_kv_heads + kvh;
  float *part = a.ws + (pair * a.max_splits + split) * G * rowf;
  for (int idx = tid; idx < G * D; idx += kPoolThreads) {
    const int g = idx / D, d = idx - g * D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kPoolWarps; ++w) mx = fmaxf(mx, s_red[(w * G + g) * rowf]);
    float ls = 0.f, as = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kPoolWarps; ++w) {
        const float *r = s_red + (w * G + g) * rowf;
        if (r[0] == -INFINITY) continue;
        const float c = exp2f(r[0] - mx);
        ls = fmaf(r[1], c, ls);
        as = fmaf(r[2 + d], c, as);
      }
    }
    if (nsplit == 1) {
      V::put(out + b * a.o_sb + static_cast<int64_t>(kvh * G + g) * a.o_sh + d,
             ls > 0.f ? as / ls : 0.f);
    } else {
      float *p = part + g * rowf;
      if (d == 0) {
        p[0] = mx;
        p[1] = ls;
      }
      p[2 + d] = as;
    }
  }
  if (nsplit == 1) return;

  // Publish this chunk; the CTA that completes the count merges every chunk of the row.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int done;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                 : "=r"(done)
                 : "l"(a.counters + pair)
                 : "memory");
    s_last = done == nsplit - 1;
    if (s_last) a.counters[pair] = 0;  // ready for the next launch
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float *parts = a.ws + pair * a.max_splits * G * rowf;
  for (int idx = tid; idx < G * D; idx += kPoolThreads) {
    const int g = idx / D, d = idx - g * D;
    float mx = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) mx = fmaxf(mx, __ldcg(parts + (sp * G + g) * rowf));
    float ls = 0.f, as = 0.f;
    if (mx != -INFINITY) {
      for (int sp = 0; sp < nsplit; ++sp) {
        const float *p = parts + (sp * G + g) * rowf;
        const float pm = __ldcg(p);
        if (pm == -INFINITY) continue;
        const float c = exp2f(pm - mx);
        ls = fmaf(__ldcg(p + 1), c, ls);
        as = fmaf(__ldcg(p + 2 + d), c, as);
      }
    }
    V::put(out + b * a.o_sb + static_cast<int64_t>(kvh * G + g) * a.o_sh + d,
           ls > 0.f ? as / ls : 0.f);
  }
}


size_t header_bytes(int64_t pairs) { return static_cast<size_t>((pairs * 4 + 255) / 256 * 256); }

constexpr size_t kPoolSmemLimit = 48 * 1024;

// Shared memory a CTA stages for `chunk` positions: page offsets and attend bytes.
size_t pool_stage_bytes(int64_t chunk, int page_size) {
  return static_cast<size_t>((chunk / page_size + 2) * 8 + (chunk + 15) / 16 * 16);
}

template <typename T, int G, int NPL>
int launch_pool(const PoolArgs &a, int batch, size_t smem, cudaStream_t stream) {
  auto kernel = pool_decode_kernel<T, G, NPL>;
  dim3 grid(a.max_splits, a.num_kv_heads, batch);
  B200_LAUNCH_CHECK_ERR(launch_kernel(kernel, grid, dim3(kPoolThreads), smem, stream, false, 1, a),
                        "pool_paged_decode");
  return B200ASR_OK;
}

template <typename T, int NPL>
int dispatch_group(const PoolArgs &a, int g, int batch, size_t smem, cudaStream_t stream) {
  switch (g) {
    case 1: return launch_pool<T, 1, NPL>(a, batch, smem, stream);
    case 2: return launch_pool<T, 2, NPL>(a, batch, smem, stream);
    case 4: return launch_pool<T, 4, NPL>(a, batch, smem, stream);
    default: return launch_pool<T, 8, NPL>(a, batch, smem, stream);
  }
}

template <typename T>
int dispatch_width(const PoolArgs &a, int g, int npl, int batch, size_t smem, cudaStream_t stream) {
  return npl == 1 ? dispatch_group<T, 1>(a, g, batch, smem, stream)
                  : dispatch_group<T, 2>(a, g, batch, smem, stream);
}

}  // namespace
}  // namespace b200asr

using namespace b200asr;

extern "C" size_t b200asr_pool_paged_decode_workspace_size(int32_t batch, int32_t num_heads,
                                                           int32_t head_dim, int32_t max_seq_len) {
  if (batch <= 0 || num_heads <= 0 || head_dim <= 0 || max_seq_len <= 0) return 256;
  const int64_t pairs = static_cast<int64_t>(batch) * num_heads;
  const int64_t splits = (static_cast<int64_t>(max_seq_len) + kPoolMinChunk - 1) / kPoolMinChunk;
  return header_bytes(pairs) + static_cast<size_t>(pairs * splits * (head_dim + 2) * 4);
}

extern "C" int b200asr_pool_paged_decode(
    int32_t dtype, int32_t batch, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
    const void *query, int64_t q_stride_b, int64_t q_stride_h, void *key_pool, void *value_pool,
    int32_t num_pages, int32_t page_size, int64_t kv_stride_p, int64_t kv_stride_h,
    int64_t kv_stride_s, const int64_t *page_table, int64_t table_stride, int32_t table_width,
    const int64_t *seq_lens, const uint8_t *key_valid_mask, int64_t valid_stride,
    int32_t valid_len, const void *new_key, const void *new_value, int64_t new_stride_b,
    int64_t new_stride_h, void *out, int64_t out_stride_b, int64_t out_stride_h,
    int32_t max_seq_len, int32_t tokens_per_cta, float scale, void *workspace,
    size_t workspace_bytes, int32_t *error_flag, b200asr_stream_t stream) {
  B200_REQUIRE(dtype == B200ASR_DTYPE_BF16 || dtype == B200ASR_DTYPE_F16 ||
                   dtype == B200ASR_DTYPE_F32,
               "pool_paged_decode: unknown dtype %d", dtype);
  B200_REQUIRE(batch >= 0 && batch <= 65535, "pool_paged_decode: batch %d out of range", batch);
  if (batch == 0) return B200ASR_OK;
  B200_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_kv_heads <= 65535 &&
                   num_heads % num_kv_heads == 0,
               "pool_paged_decode: query heads must be divisible by KV heads (%d / %d)", num_heads,
               num_kv_heads);
  const int g = num_heads / num_kv_heads;
  if (g != 1 && g != 2 && g != 4 && g != 8) {
    set_error("pool_paged_decode: group size %d unsupported (1, 2, 4 or 8)", g);
    return B200ASR_ERR_UNSUPPORTED;
  }
  const int esz = dtype == B200ASR_DTYPE_F32 ? 4 : 2;
  const int E = 16 / esz;
  if (head_dim <= 0 || (head_dim * esz) % 16 != 0 || head_dim * esz > 1024) {
    set_error("pool_paged_decode: head_dim %d x %d bytes must be a multiple of 16 bytes, at most 1024",
              head_dim, esz);
    return B200ASR_ERR_UNSUPPORTED;
  }
  const size_t red_bytes = static_cast<size_t>(kPoolWarps) * g * (head_dim + 2) * sizeof(float);
  if (red_bytes + pool_stage_bytes(kPoolMinChunk, page_size) > kPoolSmemLimit) {
    set_error("pool_paged_decode: group %d x head_dim %d too large", g, head_dim);
    return B200ASR_ERR_UNSUPPORTED;
  }
  B200_REQUIRE(query && key_pool && value_pool && page_table && seq_lens && out && workspace,
               "pool_paged_decode: null pointer");
  B200_REQUIRE((new_key == nullptr) == (new_value == nullptr),
               "pool_paged_decode: new_key and new_value must be provided together");
  B200_REQUIRE(aligned16(query) && aligned16(key_pool) && aligned16(value_pool) &&
                   aligned16(workspace) && (new_key == nullptr || (aligned16(new_key) && aligned16(new_value))),
               "pool_paged_decode: query, pools and new K/V must be 16-byte aligned");
  B200_REQUIRE(q_stride_b % E == 0 && q_stride_h % E == 0 && kv_stride_p % E == 0 &&
                   kv_stride_h % E == 0 && kv_stride_s % E == 0 && new_stride_b % E == 0 &&
                   new_stride_h % E == 0,
               "pool_paged_decode: strides must be multiples of 16 bytes (unit head_dim stride)");
  B200_REQUIRE((reinterpret_cast<uintptr_t>(out) % esz) == 0, "pool_paged_decode: misaligned out");
  B200_REQUIRE(num_pages > 0 && page_size > 0 && table_width > 0 &&
                   (batch == 1 || table_stride >= table_width),
               "pool_paged_decode: bad pool / page table sizes");
  B200_REQUIRE(key_valid_mask == nullptr || (valid_len >= 0 && (batch == 1 || valid_stride >= valid_len)),
               "pool_paged_decode: bad key_valid_mask sizes");
  B200_REQUIRE(max_seq_len > 0, "pool_paged_decode: max_seq_len must be positive");
  B200_REQUIRE(tokens_per_cta == 0 || tokens_per_cta >= kPoolMinChunk,
               "pool_paged_decode: tokens_per_cta must be 0 (auto) or >= %d", kPoolMinChunk);
  const size_t need = b200asr_pool_paged_decode_workspace_size(batch, num_heads, head_dim, max_seq_len);
  if (workspace_bytes < need) {
    set_error("pool_paged_decode: workspace %zu bytes < %zu needed", workspace_bytes, need);
    return B200ASR_ERR_WORKSPACE;
  }
  // The talker's case -- bf16, head_dim 128, 16-position pages, heads contiguous in query
  // and out -- runs on the stream-K decode kernel (every CTA the same share of the batch's
  // pages, one TMA box per K / V page); tokens_per_cta != 0 asks for this kernel instead.
  if (dtype == B200ASR_DTYPE_BF16 && tokens_per_cta == 0) {
    PoolStreamK p{};
    p.batch = batch;
    p.num_heads = num_heads;
    p.num_kv_heads = num_kv_heads;
    p.head_dim = head_dim;
    p.query = query;
    p.q_stride_b = q_stride_b;
    p.q_stride_h = q_stride_h;
    p.key_pool = key_pool;
    p.value_pool = value_pool;
    p.num_pages = num_pages;
    p.page_size = page_size;
    p.kv_stride_p = kv_stride_p;
    p.kv_stride_h = kv_stride_h;
    p.kv_stride_s = kv_stride_s;
    p.page_table = page_table;
    p.table_stride = table_stride;
    p.table_width = table_width;
    p.seq_lens = seq_lens;
    p.valid = key_valid_mask;
    p.valid_stride = valid_stride;
    p.valid_len = valid_len;
    p.new_key = new_key;
    p.new_value = new_value;
    p.new_stride_b = new_stride_b;
    p.new_stride_h = new_stride_h;
    p.out = out;
    p.out_stride_b = out_stride_b;
    p.out_stride_h = out_stride_h;
    p.max_seq_len = max_seq_len;
    p.scale = scale;
    p.workspace = workspace;
    p.workspace_bytes = workspace_bytes;
    p.workspace_head = header_bytes(static_cast<int64_t>(batch) * num_heads);
    p.error_flag = error_flag;
    p.stream = stream;
    bool taken = false;
    const int rc = pool_decode_stream_k(p, &taken);
    if (taken || rc != B200ASR_OK) return rc;
  }

  PoolArgs a{};
  a.q = query;
  a.q_sb = q_stride_b;
  a.q_sh = q_stride_h;
  a.kp = key_pool;
  a.vp = value_pool;
  a.sp = kv_stride_p;
  a.sh = kv_stride_h;
  a.ss = kv_stride_s;
  a.num_pages = num_pages;
  a.page_size = page_size;
  a.page_shift = (page_size & (page_size - 1)) == 0 ? __builtin_ctz(static_cast<unsigned>(page_size)) : -1;
  a.table = page_table;
  a.table_stride = table_stride;
  a.table_width = table_width;
  a.seq_lens = seq_lens;
  a.valid = key_valid_mask;
  a.valid_stride = valid_stride;
  a.valid_len = key_valid_mask ? valid_len : 0;
  a.nk = new_key;
  a.nv = new_value;
  a.n_sb = new_stride_b;
  a.n_sh = new_stride_h;
  a.out = out;
  a.o_sb = out_stride_b;
  a.o_sh = out_stride_h;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.max_seq_len = max_seq_len;
  a.nvr = head_dim * esz / 16;
  const int npl = a.nvr > 32 ? 2 : 1;
  const int per_lane = (a.nvr + npl - 1) / npl;
  int lg = 0;
  while ((1 << lg) < per_lane) ++lg;
  a.lpt_log2 = lg;
  const int step = kPoolWarps * (32 >> lg);
  int64_t chunk = tokens_per_cta;
  if (chunk == 0) {
    // ~7 CTAs per SM at the longest row: 256 positions per CTA for the talker shape
    // (B = 32 x 8 KV heads at 1024 positions), the fastest measured there; at least
    // kPoolMinChunk.
    const int64_t target = static_cast<int64_t>(num_sms()) * 7;
    const int64_t work = static_cast<int64_t>(batch) * num_kv_heads * max_seq_len;
    chunk = (work + target - 1) / target;
    if (chunk < kPoolMinChunk) chunk = kPoolMinChunk;
    chunk = (chunk + step - 1) / step * step;
  }
  if (chunk > max_seq_len) chunk = max_seq_len;
  // the staged page offsets and attend bytes must fit next to the merge rows
  while (chunk > kPoolMinChunk && red_bytes + pool_stage_bytes(chunk, page_size) > kPoolSmemLimit)
    chunk = chunk / 2 > kPoolMinChunk ? chunk / 2 : kPoolMinChunk;
  a.chunk = static_cast<int32_t>(chunk);
  a.pages_cap = static_cast<int32_t>(chunk / page_size + 2);
  const size_t smem = red_bytes + pool_stage_bytes(chunk, page_size);
  a.max_splits = static_cast<int32_t>((max_seq_len + chunk - 1) / chunk);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.counters = static_cast<int *>(workspace);
  a.ws = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) +
                                   header_bytes(static_cast<int64_t>(batch) * num_heads));
  a.error_flag = error_flag;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == B200ASR_DTYPE_BF16) return dispatch_width<__nv_bfloat16>(a, g, npl, batch, smem, s);
  if (dtype == B200ASR_DTYPE_F16) return dispatch_width<__half>(a, g, npl, batch, smem, s);
  return dispatch_width<float>(a, g, npl, batch, smem, s);
}
