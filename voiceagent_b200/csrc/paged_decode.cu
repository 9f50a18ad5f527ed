// Split-K paged decode attention (one query token per sequence).
//
// Replaces the decode use of flash_attn_varlen_func over the paged cache inside the
// CUDA-graph decode (layers/attention.py:96-107 with max_seqlen_q = 1, fed by
// engine/graph_runner.py:81-94): out[b, h] = softmax(q[b, h] K_b^T * scale) V_b with
// K_b, V_b the first len_b rows of sequence b gathered through its block table, and
// query head h reading KV head h / (H / H_kv).
//
// Design (HBM-bound; one KV row is read once for all query heads of its group):
//  * Work item = (sequence, 64-token chunk inside one 256-token block). The K (or V)
//    rows of a chunk are ONE contiguous range of the cache (a slot holds all KV heads),
//    so a stage of 16 tokens is a single 32 KiB 1-D bulk copy per operand.
//  * Persistent grid, one CTA per SM. Warp 16 is the producer: it walks the same item
//    sequence as the consumers and keeps a 3-stage ring of K/V tiles in flight
//    (mbarrier full/empty pairs).
//  * 16 consumer warps: warp w % 8 owns KV head w % 8 (and its G query heads) and
//    token half w / 8 of every stage. Lane l holds head dims 4l..4l+3. The G x 8
//    partial dot products of a stage are summed with a butterfly reduce-scatter
//    (each lane ends with one full score), then an fp32 online softmax in base 2.
//  * At the end of an item the two token halves merge through shared memory. A
//    sequence with one item writes its bf16 output directly; longer ones write an
//    unnormalised fp32 partial (+ running max and sum) to the caller's workspace and
//    decode_combine merges them.
#include "common.cuh"

namespace b200asr {

constexpr int kDecD = 128;
constexpr int kDecChunk = 64;
constexpr int kDecStage = 16;
constexpr int kDecStages = 3;
constexpr int kDecHalf = kDecStage / 2;
constexpr int kDecMaxBatch = 1024;
constexpr float kLog2e = 1.4426950408889634f;

template <int HKV, int G>
struct Dec {
  static constexpr int H = HKV * G;
  static constexpr int ROW = HKV * kDecD;            // elements per slot (K or V)
  static constexpr int ROW_BYTES = ROW * 2;
  static constexpr int CONSUMERS = 2 * HKV;           // warps
  static constexpr int THREADS = (CONSUMERS + 1) * 32;
  static constexpr int STAGE_BYTES = kDecStage * ROW_BYTES;
  static constexpr int NV = kDecHalf * G;             // partial scores per warp per stage
  static constexpr int LOG2NV = NV == 8 ? 3 : NV == 16 ? 4 : NV == 32 ? 5 : -1;
  static constexpr int SHIFT = 5 - LOG2NV;            // lane bits that duplicate a score
  static constexpr int LOG2G = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : -1;
  static constexpr int MERGE_FLOATS = HKV * 32 * (4 * G) + HKV * 2 * G;
  static constexpr size_t SMEM = 2ull * kDecStages * STAGE_BYTES + MERGE_FLOATS * 4 +
                                 (kDecMaxBatch + 1) * 4 + 2 * kDecStages * 8 + 16;
  static_assert(LOG2NV > 0 && LOG2G >= 0, "unsupported group size");
};

struct DecodeArgs {
  const __nv_bfloat16 *q;
  int64_t q_stride;
  const __nv_bfloat16 *k_cache;
  const __nv_bfloat16 *v_cache;
  int num_blocks;
  int block_size;
  const int32_t *cu_seqlens_k;
  const int32_t *block_tables;
  int bt_stride;
  int batch;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16 *out;
  int64_t out_stride;
  float *ws_o;   // [items_cap][H][128]
  float *ws_ml;  // [items_cap][H][2]
  int items_cap;
  int32_t *error_flag;
};

__device__ __forceinline__ void consumer_barrier(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// Index of the sequence owning item `it` (largest b with item_start[b] <= it).
__device__ __forceinline__ int item_seq(const int *item_start, int batch, int it) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (item_start[mid] <= it) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <int HKV, int G>
__global__ void __launch_bounds__(Dec<HKV, G>::THREADS, 1)
    paged_decode_kernel(const DecodeArgs a) {
  using C = Dec<HKV, G>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *ks = smem;
  uint8_t *vs = smem + kDecStages * C::STAGE_BYTES;
  float *merge = reinterpret_cast<float *>(smem + 2 * kDecStages * C::STAGE_BYTES);
  int *item_start = reinterpret_cast<int *>(merge + C::MERGE_FLOATS);
  uint64_t *full = reinterpret_cast<uint64_t *>(item_start + kDecMaxBatch + 1 + 1);
  // (+1 int of padding keeps the barriers 8-byte aligned for any batch)
  full = reinterpret_cast<uint64_t *>((reinterpret_cast<uintptr_t>(full) + 7) & ~uintptr_t(7));
  uint64_t *empty = full + kDecStages;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // Item prefix over sequences (warp 0, 32 sequences per pass).
  if (warp == 0) {
    int carry = 0;
    for (int b0 = 0; b0 < a.batch; b0 += 32) {
      const int b = b0 + lane;
      int n = 0;
      if (b < a.batch) n = (a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b] + kDecChunk - 1) / kDecChunk;
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (b < a.batch) item_start[b] = carry + incl - n;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) item_start[a.batch] = carry;
  }
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::CONSUMERS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  int total = item_start[a.batch];
  if (total > a.items_cap) {
    if (tid == 0) raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);
    total = a.items_cap;
  }

  if (warp == C::CONSUMERS) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it_stage = 0;
      for (int it = blockIdx.x; it < total; it += gridDim.x) {
        const int b = item_seq(item_start, a.batch, it);
        const int c = it - item_start[b];
        const int len = a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b];
        const int start = c * kDecChunk;
        const int n = min(kDecChunk, len - start);
        int block = a.block_tables[static_cast<int64_t>(b) * a.bt_stride + start / a.block_size];
        if (block < 0 || block >= a.num_blocks) {
          raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
          block = 0;
        }
        const int64_t slot0 = static_cast<int64_t>(block) * a.block_size + (start % a.block_size);
        for (int s0 = 0; s0 < n; s0 += kDecStage, ++it_stage) {
          const int st = it_stage % kDecStages;
          const uint32_t ph = (it_stage / kDecStages) & 1;
          if (!mbar_wait(&empty[st], ph ^ 1, a.error_flag, &abort_flag)) return;
          const int ntok = min(kDecStage, n - s0);
          const uint32_t bytes = ntok * C::ROW_BYTES;
          mbar_arrive_expect_tx(&full[st], 2 * bytes);
          const int64_t off = (slot0 + s0) * C::ROW;
          bulk_g2s(ks + st * C::STAGE_BYTES, a.k_cache + off, bytes, &full[st]);
          bulk_g2s(vs + st * C::STAGE_BYTES, a.v_cache + off, bytes, &full[st]);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int w = warp % HKV;      // KV head
  const int half = warp / HKV;   // token half of each stage
  const int my_j = lane >> C::SHIFT;
  const int my_t = my_j >> C::LOG2G;
  const int my_g = my_j & (G - 1);
  uint32_t it_stage = 0;

  for (int it = blockIdx.x; it < total; it += gridDim.x) {
    const int b = item_seq(item_start, a.batch, it);
    const int c = it - item_start[b];
    const int len = a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b];
    const int n = min(kDecChunk, len - c * kDecChunk);
    const bool single = len <= kDecChunk;

    float qv[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint2 u = *reinterpret_cast<const uint2 *>(
          a.q + b * a.q_stride + (w * G + g) * kDecD + lane * 4);
      qv[g][0] = __uint_as_float(u.x << 16) * a.scale_log2;
      qv[g][1] = __uint_as_float(u.x & 0xffff0000u) * a.scale_log2;
      qv[g][2] = __uint_as_float(u.y << 16) * a.scale_log2;
      qv[g][3] = __uint_as_float(u.y & 0xffff0000u) * a.scale_log2;
    }
    float acc[G][4], m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[g][k] = 0.f;
    }

    for (int s0 = 0; s0 < n; s0 += kDecStage, ++it_stage) {
      const int st = it_stage % kDecStages;
      const uint32_t ph = (it_stage / kDecStages) & 1;
      if (!mbar_wait(&full[st], ph, a.error_flag, &abort_flag)) return;
      const int ntok = min(kDecStage, n - s0);
      const uint8_t *kt = ks + st * C::STAGE_BYTES + (w * kDecD + lane * 4) * 2;
      const uint8_t *vt = vs + st * C::STAGE_BYTES + (w * kDecD + lane * 4) * 2;

      // Partial dot products of this lane's 4 dims for 8 tokens x G heads.
      float part[C::NV];
#pragma unroll
      for (int t = 0; t < kDecHalf; ++t) {
        const int tt = half * kDecHalf + t;
        float kf[4] = {0.f, 0.f, 0.f, 0.f};
        if (tt < ntok) {
          const uint2 u = *reinterpret_cast<const uint2 *>(kt + tt * C::ROW_BYTES);
          kf[0] = __uint_as_float(u.x << 16);
          kf[1] = __uint_as_float(u.x & 0xffff0000u);
          kf[2] = __uint_as_float(u.y << 16);
          kf[3] = __uint_as_float(u.y & 0xffff0000u);
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
          part[t * G + g] = qv[g][0] * kf[0] + qv[g][1] * kf[1] + qv[g][2] * kf[2] + qv[g][3] * kf[3];
      }
      // Butterfly reduce-scatter: lane ends with the full score of index lane >> SHIFT.
#pragma unroll
      for (int step = 0; step < C::LOG2NV; ++step) {
        const int hn = C::NV >> (step + 1);
        const int mask = 16 >> step;
        const bool upper = (lane & mask) != 0;
#pragma unroll
        for (int i = 0; i < hn; ++i) {
          const float send = upper ? part[i] : part[i + hn];
          const float keep = upper ? part[i + hn] : part[i];
          part[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
        }
      }
#pragma unroll
      for (int mask = 16 >> C::LOG2NV; mask >= 1; mask >>= 1)
        part[0] += __shfl_xor_sync(0xffffffffu, part[0], mask);

      const bool valid = half * kDecHalf + my_t < ntok;
      const float s = valid ? part[0] : -INFINITY;
      // Per-head max over this half's tokens: reduce across the lane bits that hold t.
      float mx = s;
#pragma unroll
      for (int bit = C::SHIFT + C::LOG2G; bit < 5; ++bit)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1 << bit));
      float alpha[G], mnew[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float ms = __shfl_sync(0xffffffffu, mx, g << C::SHIFT);
        mnew[g] = fmaxf(m[g], ms);
        alpha[g] = mnew[g] == -INFINITY ? 1.f : exp2f(m[g] - mnew[g]);
      }
      float mine_m = mnew[0];
#pragma unroll
      for (int g = 1; g < G; ++g)
        if (my_g == g) mine_m = mnew[g];
      const float p = (valid && mine_m != -INFINITY) ? exp2f(s - mine_m) : 0.f;
      float ps = p;
#pragma unroll
      for (int bit = C::SHIFT + C::LOG2G; bit < 5; ++bit)
        ps += __shfl_xor_sync(0xffffffffu, ps, 1 << bit);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float ls = __shfl_sync(0xffffffffu, ps, g << C::SHIFT);
        l[g] = l[g] * alpha[g] + ls;
        m[g] = mnew[g];
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[g][k] *= alpha[g];
      }
      // P V for this half's tokens.
#pragma unroll
      for (int t = 0; t < kDecHalf; ++t) {
        const int tt = half * kDecHalf + t;
        if (tt < ntok) {
          const uint2 u = *reinterpret_cast<const uint2 *>(vt + tt * C::ROW_BYTES);
          const float v0 = __uint_as_float(u.x << 16), v1 = __uint_as_float(u.x & 0xffff0000u);
          const float v2 = __uint_as_float(u.y << 16), v3 = __uint_as_float(u.y & 0xffff0000u);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float pg = __shfl_sync(0xffffffffu, p, ((t * G + g) << C::SHIFT));
            acc[g][0] += pg * v0;
            acc[g][1] += pg * v1;
            acc[g][2] += pg * v2;
            acc[g][3] += pg * v3;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // Merge the two token halves of this item.
    float *mine = merge + (w * 32 + lane) * (4 * G);
    float *ml = merge + HKV * 32 * (4 * G) + w * 2 * G;
    if (half == 1) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int k = 0; k < 4; ++k) mine[g * 4 + k] = acc[g][k];
        if (lane == 0) {
          ml[2 * g] = m[g];
          ml[2 * g + 1] = l[g];
        }
      }
    }
    consumer_barrier(C::CONSUMERS * 32);
    if (half == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float m1 = ml[2 * g], l1 = ml[2 * g + 1];
        const float mm = fmaxf(m[g], m1);
        const float a0 = m[g] == -INFINITY ? 0.f : exp2f(m[g] - mm);
        const float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mm);
        const float lt = l[g] * a0 + l1 * a1;
        float o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = acc[g][k] * a0 + mine[g * 4 + k] * a1;
        const int h = w * G + g;
        if (single) {
          const float inv = 1.f / lt;
          uint2 u;
          u.x = pack2(o[0] * inv, o[1] * inv);
          u.y = pack2(o[2] * inv, o[3] * inv);
          *reinterpret_cast<uint2 *>(a.out + b * a.out_stride + h * kDecD + lane * 4) = u;
        } else {
          float4 *dst = reinterpret_cast<float4 *>(a.ws_o + (static_cast<int64_t>(it) * C::H + h) * kDecD) + lane;
          *dst = make_float4(o[0], o[1], o[2], o[3]);
          if (lane == 0) {
            a.ws_ml[(static_cast<int64_t>(it) * C::H + h) * 2] = mm;
            a.ws_ml[(static_cast<int64_t>(it) * C::H + h) * 2 + 1] = lt;
          }
        }
      }
    }
    consumer_barrier(C::CONSUMERS * 32);
  }
}

// Merge the per-item partials of every sequence longer than one item.
// One CTA per sequence, H x 32 threads; thread (h, lane) owns dims 4*lane..+3.
template <int H>
__global__ void decode_combine_kernel(const DecodeArgs a) {
  const int b = blockIdx.x;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Items before this sequence: warp-parallel sum over the preceding lengths.
  int first = 0;
  for (int i0 = 0; i0 < b; i0 += 32) {
    const int i = i0 + lane;
    int n_i = 0;
    if (i < b) n_i = (a.cu_seqlens_k[i + 1] - a.cu_seqlens_k[i] + kDecChunk - 1) / kDecChunk;
    first += n_i;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) first += __shfl_xor_sync(0xffffffffu, first, o);
  const int len = a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b];
  const int n = (len + kDecChunk - 1) / kDecChunk;
  __nv_bfloat16 *dst = a.out + b * a.out_stride + h * kDecD + lane * 4;
  if (n == 1) return;
  if (n <= 0 || first + n > a.items_cap) {
    *reinterpret_cast<uint2 *>(dst) = make_uint2(0u, 0u);
    return;
  }
  float mm = -INFINITY;
#pragma unroll 8
  for (int i = 0; i < n; ++i) mm = fmaxf(mm, a.ws_ml[(static_cast<int64_t>(first + i) * H + h) * 2]);
  float lt = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
  for (int i = 0; i < n; ++i) {
    const int64_t base = static_cast<int64_t>(first + i) * H + h;
    const float mi = a.ws_ml[base * 2];
    const float w = mi == -INFINITY ? 0.f : exp2f(mi - mm);
    lt += a.ws_ml[base * 2 + 1] * w;
    const float4 v = reinterpret_cast<const float4 *>(a.ws_o + base * kDecD)[lane];
    o[0] += v.x * w;
    o[1] += v.y * w;
    o[2] += v.z * w;
    o[3] += v.w * w;
  }
  const float inv = 1.f / lt;
  *reinterpret_cast<uint2 *>(dst) = make_uint2(pack2(o[0] * inv, o[1] * inv), pack2(o[2] * inv, o[3] * inv));
}

int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

template <int HKV, int G>
int launch_decode(const DecodeArgs &a, cudaStream_t stream) {
  using C = Dec<HKV, G>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(paged_decode_kernel<HKV, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(C::SMEM));
    if (e != cudaSuccess) {
      set_error("paged_decode: cannot reserve %zu bytes of shared memory: %s", C::SMEM,
                cudaGetErrorString(e));
      return B200ASR_ERR_CUDA;
    }
    configured = true;
  }
  const int grid = std::max(1, std::min(a.items_cap, num_sms()));
  paged_decode_kernel<HKV, G><<<grid, C::THREADS, C::SMEM, stream>>>(a);
  B200_CUDA_LAUNCH_CHECK("paged_decode");
  decode_combine_kernel<C::H><<<a.batch, C::H * 32, 0, stream>>>(a);
  B200_CUDA_LAUNCH_CHECK("paged_decode_combine");
  return B200ASR_OK;
}

size_t decode_items_cap(int batch, int max_seqlen_k) {
  return static_cast<size_t>(batch) * ((std::max(max_seqlen_k, 1) + kDecChunk - 1) / kDecChunk);
}

}  // namespace b200asr

using namespace b200asr;

extern "C" size_t b200asr_paged_decode_workspace_size(int32_t batch, int32_t max_seqlen_k,
                                                      int32_t num_heads, int32_t head_dim) {
  if (batch <= 0 || num_heads <= 0 || head_dim <= 0) return 0;
  const size_t items = decode_items_cap(batch, max_seqlen_k);
  return items * num_heads * (static_cast<size_t>(head_dim) + 2) * sizeof(float) + 256;
}

extern "C" int b200asr_paged_decode(const void *q, int64_t q_row_stride, const void *k_cache,
                                    const void *v_cache, int32_t num_blocks, int32_t block_size,
                                    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                    const int32_t *cu_seqlens_k, const int32_t *block_tables,
                                    int32_t bt_stride, int32_t batch, int32_t max_seqlen_k,
                                    float scale, void *out, int64_t out_row_stride,
                                    void *workspace, size_t workspace_bytes, int32_t *error_flag,
                                    b200asr_stream_t stream) {
  B200_REQUIRE(head_dim == kDecD, "paged_decode: head_dim %d unsupported (needs 128)", head_dim);
  B200_REQUIRE(batch >= 0 && batch <= kDecMaxBatch, "paged_decode: batch %d not in [0, %d]",
               batch, kDecMaxBatch);
  if (batch == 0) return B200ASR_OK;
  B200_REQUIRE(block_size >= kDecChunk && block_size % kDecChunk == 0,
               "paged_decode: block_size %d must be a multiple of %d", block_size, kDecChunk);
  B200_REQUIRE(num_blocks >= 1 && bt_stride >= 1 && max_seqlen_k >= 1,
               "paged_decode: bad table geometry");
  B200_REQUIRE(q && k_cache && v_cache && cu_seqlens_k && block_tables && out && workspace,
               "paged_decode: null pointer");
  B200_REQUIRE(q_row_stride % 4 == 0 && out_row_stride % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(q) & 7) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 7) == 0 && aligned16(k_cache) &&
                   aligned16(v_cache) && aligned16(workspace),
               "paged_decode: misaligned tensor");
  const size_t need = b200asr_paged_decode_workspace_size(batch, max_seqlen_k, num_heads, head_dim);
  if (workspace_bytes < need) {
    set_error("paged_decode: workspace %zu bytes < %zu needed", workspace_bytes, need);
    return B200ASR_ERR_WORKSPACE;
  }
  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16 *>(q);
  a.q_stride = q_row_stride;
  a.k_cache = static_cast<const __nv_bfloat16 *>(k_cache);
  a.v_cache = static_cast<const __nv_bfloat16 *>(v_cache);
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.cu_seqlens_k = cu_seqlens_k;
  a.block_tables = block_tables;
  a.bt_stride = bt_stride;
  a.batch = batch;
  a.scale_log2 = scale * kLog2e;
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.out_stride = out_row_stride;
  a.items_cap = static_cast<int>(decode_items_cap(batch, max_seqlen_k));
  a.ws_o = static_cast<float *>(workspace);
  a.ws_ml = a.ws_o + static_cast<size_t>(a.items_cap) * num_heads * head_dim;
  a.error_flag = error_flag;
  if (num_kv_heads == 8 && num_heads == 16) return launch_decode<8, 2>(a, stream);
  if (num_kv_heads == 8 && num_heads == 8) return launch_decode<8, 1>(a, stream);
  if (num_kv_heads == 4 && num_heads == 16) return launch_decode<4, 4>(a, stream);
  if (num_kv_heads == 4 && num_heads == 8) return launch_decode<4, 2>(a, stream);
  if (num_kv_heads == 2 && num_heads == 4) return launch_decode<2, 2>(a, stream);
  set_error("paged_decode: %d query / %d KV heads unsupported", num_heads, num_kv_heads);
  return B200ASR_ERR_UNSUPPORTED;
}

// -----------------------------------------------------------------------------
// Allocation-free paged decode.
//
// Some callers of this library cannot hand it device scratch memory: an FFI host that
// owns no CUDA allocator, a serving process whose memory pool was fully reserved for the
// KV cache at start-up, or code that runs while a CUDA graph is being captured, where a
// cudaMalloc is not allowed. For them the split-K partials of the decode pass live in a
// fixed array compiled into this library instead of a caller workspace.
//
// The array is a file-scope __device__ symbol of B200ASR_NOALLOC_SCRATCH_BYTES; every GPU
// that loads the library holds that much memory until the process exits. Host code cannot
// use the symbol's name as a device address, so on the first call on each device (with
// that device current) cudaGetSymbolAddress resolves it once and the pointer is cached.
// That first call may trigger module loading, so it must come before any stream capture.
// All calls share the one array and nothing in it needs clearing (every partial is written
// before it is read), so two calls whose kernels overlap on the GPU -- different streams,
// or graphs replayed concurrently -- race on it and must be serialised by the caller.
#include <mutex>

namespace b200asr {

static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[B200ASR_NOALLOC_SCRATCH_BYTES];

static void *noalloc_scratch(int *status) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void *resolved[kMaxDevices] = {};
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("paged_decode_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    *status = B200ASR_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (resolved[dev] == nullptr) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("paged_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      *status = B200ASR_ERR_CUDA;
      return nullptr;
    }
    resolved[dev] = p;
  }
  return resolved[dev];
}

}  // namespace b200asr

extern "C" int b200asr_paged_decode_noalloc(const void *q, int64_t q_row_stride,
                                            const void *k_cache, const void *v_cache,
                                            int32_t num_blocks, int32_t block_size,
                                            int32_t num_heads, int32_t num_kv_heads,
                                            int32_t head_dim, const int32_t *cu_seqlens_k,
                                            const int32_t *block_tables, int32_t bt_stride,
                                            int32_t batch, int32_t max_seqlen_k, float scale,
                                            void *out, int64_t out_row_stride,
                                            int32_t *error_flag, b200asr_stream_t stream) {
  const size_t need =
      b200asr_paged_decode_workspace_size(batch, max_seqlen_k, num_heads, head_dim);
  if (need > static_cast<size_t>(B200ASR_NOALLOC_SCRATCH_BYTES)) {
    set_error("paged_decode_noalloc: batch %d x max_seqlen_k %d x %d heads needs %zu bytes of "
              "scratch, more than the built-in %zu; use b200asr_paged_decode with a workspace",
              batch, max_seqlen_k, num_heads, need,
              static_cast<size_t>(B200ASR_NOALLOC_SCRATCH_BYTES));
    return B200ASR_ERR_WORKSPACE;
  }
  if (batch == 0) return B200ASR_OK;
  int status = B200ASR_OK;
  void *scratch = noalloc_scratch(&status);
  if (scratch == nullptr) return status;
  return b200asr_paged_decode(q, q_row_stride, k_cache, v_cache, num_blocks, block_size,
                              num_heads, num_kv_heads, head_dim, cu_seqlens_k, block_tables,
                              bt_stride, batch, max_seqlen_k, scale, out, out_row_stride, scratch,
                              B200ASR_NOALLOC_SCRATCH_BYTES, error_flag, stream);
}
