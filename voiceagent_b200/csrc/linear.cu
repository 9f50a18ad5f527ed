// Decode-size linear layers on tcgen05: Y[M, :] = X[M, K] W^T for M <= 64 rows.
//
// The decoder's projections in a decode step (layers qkv_proj / o_proj / gate_up_proj /
// down_proj and lm_head of models/qwen3.py, called with the graph bucket's 1..64 rows)
// are pure weight streaming: 4-12 MB of bf16 weights against a few KB of activations.
// A library GEMM tiles the problem for large M and leaves most SMs idle or splits K with
// an extra reduction pass; here the weights are the 128-row tcgen05 A operand and the
// batch is the MMA's N (32 or 64 columns), so every CTA streams its own weight tile once.
//
//  * CTA = (128 weight rows, 1/ks of K). The ks CTAs sharing a tile form a thread-block
//    cluster; each accumulates its K slice in TMEM. CTA r reduces batch columns
//    [r * MP / ks, (r + 1) * MP / ks): every CTA pushes the columns its peers own from
//    registers straight into their shared memory (st.async, completion counted in bytes
//    on the receiver's mbarrier), so a receiver waits only for its own bytes, sums the ks
//    partials in rank order and writes bf16 -- on chip, no workspace, no second kernel,
//    and no cluster-wide barrier after the MMAs.
//  * A 4-deep TMA ring (128-byte swizzle) per CTA: each weight tile arrives as two 64-row
//    boxes, the activation tile as one box whose rows past M are zero-filled.
//  * Fused SiLU*mul (layers/activation.py:11-14) for gate_up_proj: a tile's two boxes are
//    64 gate rows and the matching 64 up rows of the unmodified [gate; up] weight, so the
//    epilogue writes silu(gate) * up directly, with the rounding of the unfused path
//    (bf16 projections, bf16 silu, bf16 product).
//
//  * Decode-step fusions around the decoder layer's RMSNorms (layers/layernorm.py:19-36)
//    and q/k norm + RoPE + KV store (models/qwen3.py:43-48, attention.py:90):
//      - residual-add epilogue (o_proj, down_proj): h = bf16(y) + residual in fp32,
//        residual <- bf16(h), h kept in fp32 and, per 128-column tile, the row's partial
//        sum of squares of h (a warp reduction in a fixed order: deterministic);
//      - RMSNorm prologue (qkv_proj, gate_up_proj): the CTA's K slice of the normalised
//        activation bf16(bf16(h * rsqrt(sum / K + eps)) * w) is computed from that fp32 h
//        and the tile partials (summed in tile order) and written straight into shared
//        memory in the 128-byte-swizzled layout the MMA reads, instead of a TMA load;
//      - q/k-norm + RoPE + store epilogue (qkv_proj): a 128-row tile is one head, so the
//        per-head RMSNorm, the rotation (partner dims in lane ^ 16) and the paged-cache
//        store of K and V happen on the reduced tile, with the rounding of the unfused
//        kernels (bf16 projection, bf16 after the norm, after the weight, after RoPE).
//    A decode layer is then qkv (norm + rope + store) -> attention -> o_proj (+residual)
//    -> gate_up (norm, SiLU*mul) -> down (+residual): five launches instead of eight.
//
// No TMA multicast is used. Every CTA takes part in the one (split) cluster barrier and
// pushes all its bytes whatever happens (a timed-out wait only skips work and raises the
// flag), so no CTA waits for one that left.
#include "common.cuh"

namespace b200asr {

constexpr int kLnBK = 64;       // K elements per stage (one 128-byte swizzle row)
constexpr int kLnRows = 128;    // weight rows per CTA (MMA M)
constexpr int kLnStages = 4;
constexpr int kLnThreads = 128;
constexpr int kLnMaxSplit = 16;

// Ring depth: 4 stages, except for 64 rows fed by TMA, where 3 stages (~106 KB) let two
// CTAs share an SM (4 stages, ~130 KB, fit only one). The RMSNorm prologue keeps 4: it
// needs a CTA's whole K slice in the ring.
template <int MP, bool NORM_IN = false>
struct Ln {
  static constexpr int STAGES = (MP == 64 && !NORM_IN) ? 3 : kLnStages;
  static constexpr int W_BYTES = kLnRows * kLnBK * 2;  // 16 KiB
  static constexpr int X_BYTES = MP * kLnBK * 2;       // 4 or 8 KiB
  static constexpr int STAGE = W_BYTES + X_BYTES;
  static constexpr int RED_BYTES = MP * kLnRows * 4;   // [MP][128] fp32 partial
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(STAGES) * STAGE + RED_BYTES + 256;
  static_assert(STAGES * STAGE >= MP * kLnRows * 4, "the ring holds the column-major partial");
  static constexpr uint32_t TMEM_COLS = MP;            // 32 or 64 (power of two >= 32)
  static_assert(MP == 32 || MP == 64, "MMA N");
};

struct LinearArgs {
  int m;           // valid activation rows
  int steps;       // K stages per CTA
  int k_split;     // CTAs per cluster along K
  int silu_inner;  // 0: plain; I: rows [0, I) gate, [I, 2I) up, output I columns
  __nv_bfloat16 *y;
  int64_t y_stride;
  int32_t *error_flag;
};

enum : int { kEpiPlain = 0, kEpiSilu = 1, kEpiAdd = 2, kEpiQkRope = 3 };

struct LinearFuse {
  // RMSNorm prologue: x[r, k] = bf16(bf16(h[r, k] * rsqrt(sum_t ss[t][r] / K + eps)) * w[k])
  const float *h;          // fp32 [m, >= K], row stride h_stride
  int64_t h_stride;
  const float *ss;         // [m][ss_tiles] partial sums of squares (row-major, 16-B rows)
  int ss_tiles;
  const __nv_bfloat16 *norm_w;
  float norm_eps;
  int norm_k;              // K of the normalised row (the full hidden size)
  // residual-add epilogue
  __nv_bfloat16 *residual;
  int64_t res_stride;
  float *h_out;            // fp32 [m, N], row stride h_out_stride
  int64_t h_out_stride;
  float *ss_out;           // [m][N / 128]
  // q/k-norm + RoPE + store epilogue (head_dim 128 = one tile)
  int num_heads, num_kv_heads;
  const __nv_bfloat16 *q_w, *k_w;
  float qk_eps;
  const int64_t *positions;
  const float *cos_sin;    // fp32 [max_position, 128]: cos | sin
  int max_position;
  __nv_bfloat16 *q_out;
  int64_t q_out_stride;
  __nv_bfloat16 *k_cache, *v_cache;
  const int32_t *slot_mapping;
  int64_t num_slots;
  // optional L2 prefetch, issued before the wait (b200asr_l2_prefetch): a layer's cached
  // K/V rows of the listed sequences, and up to two contiguous byte ranges
  const int32_t *pf_cu_seqlens_k;  // null: no K/V prefetch
  const int32_t *pf_block_tables;
  int pf_bt_stride, pf_batch, pf_block_size, pf_row_bytes;
  int64_t pf_num_blocks;
  const uint8_t *pf_k_cache, *pf_v_cache;
  const uint8_t *pf_range[2];
  int64_t pf_range_bytes[2];
};

constexpr uint32_t kPfChunk = 16 * 1024;

__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// One warp: request sequence b's cached K and V rows (all KV heads, positions < len)
// into L2, 16 KiB per prefetch, each block's rows being one contiguous range.
__device__ __forceinline__ void prefetch_sequence_kv(const LinearFuse &f, int b, int lane) {
  const int len = f.pf_cu_seqlens_k[b + 1] - f.pf_cu_seqlens_k[b];
  const int bs = f.pf_block_size;
  const int nblk = min((len + bs - 1) / bs, f.pf_bt_stride);
  const int64_t row_bytes = f.pf_row_bytes;
  for (int j = 0; j < nblk; ++j) {
    const int blk = f.pf_block_tables[static_cast<int64_t>(b) * f.pf_bt_stride + j];
    if (blk < 0 || blk >= f.pf_num_blocks) continue;  // a hint only: skip, never fault
    const int64_t bytes = static_cast<int64_t>(min(bs, len - j * bs)) * row_bytes;
    const int64_t off = static_cast<int64_t>(blk) * bs * row_bytes;
    for (int64_t c = static_cast<int64_t>(lane) * kPfChunk; c < bytes; c += 32 * kPfChunk) {
      const uint32_t sz = static_cast<uint32_t>(min(static_cast<int64_t>(kPfChunk), bytes - c));
      prefetch_l2_bulk(f.pf_k_cache + off + c, sz);
      prefetch_l2_bulk(f.pf_v_cache + off + c, sz);
    }
  }
}

// One warp of each CTA: this CTA's share of a contiguous range (16-byte multiples).
__device__ __forceinline__ void prefetch_range_share(const uint8_t *base, int64_t bytes, int lane) {
  const int64_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) / 16 * 16;
  const int64_t start = static_cast<int64_t>(blockIdx.x) * per;
  const int64_t end = min(bytes, start + per);
  for (int64_t c = start + static_cast<int64_t>(lane) * kPfChunk; c < end; c += 32 * kPfChunk)
    prefetch_l2_bulk(base + c, static_cast<uint32_t>(min(static_cast<int64_t>(kPfChunk), end - c)));
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_saddr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
  return remote;
}
// 16-byte store into another CTA's shared memory whose completion is counted (in bytes)
// on that CTA's mbarrier.
__device__ __forceinline__ void st_async_v4(uint32_t remote_saddr, float4 v, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::
          "r"(remote_saddr),
      "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(remote_bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t c0,
                                            int32_t c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// silu(g) * u for two columns, with the unfused path's roundings: g, u are bf16
// projections, F.silu returns bf16, the product is rounded to bf16 (the packed result).
// Conversions in pairs: one paired conversion per two values.
__device__ __forceinline__ uint32_t silu_mul2(float g0, float g1, float u0, float u1) {
  const float2 gb = round2_bf16(g0, g1), ub = round2_bf16(u0, u1);
  const float2 sb = round2_bf16(gb.x / (1.0f + expf(-gb.x)), gb.y / (1.0f + expf(-gb.y)));
  return pack2(sb.x * ub.x, sb.y * ub.y);
}

constexpr int kNormMaxTiles = 32;  // RMSNorm prologue: hidden <= 32 x 128
constexpr int kEpiPre = 2;         // epilogue rows per warp whose operands are prefetched
static_assert(kEpiPre == 2, "the epilogue selects pre[0] / pre[1] by name");

// This thread's norm weights for the RMSNorm prologue (static: read before the wait on
// the previous kernel). Thread t owns chunks (t & 3) and (t & 3) + 4 of every stage.
__device__ __forceinline__ void norm_in_weights(uint4 (&wv)[kLnStages][2], const LinearArgs &a,
                                                const LinearFuse &f, int k0) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int s = 0; s < kLnStages; ++s)
#pragma unroll
    for (int jj = 0; jj < 2; ++jj)
      wv[s][jj] = s < a.steps ? *reinterpret_cast<const uint4 *>(
                                    f.norm_w + k0 + s * kLnBK + ((tid & 3) + 4 * jj) * 8)
                              : make_uint4(0, 0, 0, 0);
}

// The CTA's K slice of the RMS-normalised activation, written into the x halves of the
// first a.steps stages in the layout a 128-byte-swizzled TMA box {64, MP} would leave:
// row r at r * 128 bytes, its 16-byte chunk j at chunk j ^ (r & 7). Rows >= m are zero.
// Thread t owns row t / 4 (and + 32 for MP = 64). The row's tile sums (row-major, 16-byte
// vectors) and its h values are requested together: one L2 round trip per row.
template <int MP>
__device__ __forceinline__ void norm_in_fill(uint8_t *stages, const LinearArgs &a,
                                             const LinearFuse &f, int k0,
                                             const uint4 (&wv)[kLnStages][2]) {
  using C = Ln<MP, true>;  // the RMSNorm prologue
  const int tid = threadIdx.x;
#pragma unroll
  for (int rr = 0; rr < MP / 32; ++rr) {
    const int r = (tid >> 2) + rr * 32;
    uint8_t *xrow = stages + C::W_BYTES + r * 128;
    if (r >= a.m) {
#pragma unroll
      for (int s = 0; s < kLnStages; ++s)
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int j = (tid & 3) + 4 * jj;
          if (s < a.steps)
            *reinterpret_cast<uint4 *>(xrow + s * C::STAGE + ((j ^ (r & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
        }
      continue;
    }
    const float4 *srow = reinterpret_cast<const float4 *>(f.ss + r * f.ss_tiles);
    const float *hrow = f.h + r * f.h_stride;
    float4 sv[kNormMaxTiles / 4];
    float4 hv[kLnStages][2][2];
#pragma unroll
    for (int i = 0; i < kNormMaxTiles / 4; ++i)
      if (4 * i < f.ss_tiles) sv[i] = srow[i];
#pragma unroll
    for (int s = 0; s < kLnStages; ++s)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int kc = k0 + s * kLnBK + ((tid & 3) + 4 * jj) * 8;
        if (s < a.steps) {
          hv[s][jj][0] = *reinterpret_cast<const float4 *>(hrow + kc);
          hv[s][jj][1] = *reinterpret_cast<const float4 *>(hrow + kc + 4);
        }
      }
    float ss = 0.f;  // tile order, as norm_apply sums
#pragma unroll
    for (int i = 0; i < kNormMaxTiles / 4; ++i)
      if (4 * i < f.ss_tiles) {
        ss += sv[i].x;
        ss += sv[i].y;
        ss += sv[i].z;
        ss += sv[i].w;
      }
    const float rs = rsqrtf(ss / static_cast<float>(f.norm_k) + f.norm_eps);
#pragma unroll
    for (int s = 0; s < kLnStages; ++s)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        if (s >= a.steps) continue;
        const int j = (tid & 3) + 4 * jj;
        float w[8];
        unpack8(wv[s][jj], w);
        const float h[8] = {hv[s][jj][0].x, hv[s][jj][0].y, hv[s][jj][0].z, hv[s][jj][0].w,
                            hv[s][jj][1].x, hv[s][jj][1].y, hv[s][jj][1].z, hv[s][jj][1].w};
        // bf16(bf16(h * rs) * w), converted in pairs; the second rounding is the output
        uint32_t y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 n = round2_bf16(h[2 * e] * rs, h[2 * e + 1] * rs);
          y[e] = pack2(n.x * w[2 * e], n.y * w[2 * e + 1]);
        }
        *reinterpret_cast<uint4 *>(xrow + s * C::STAGE + ((j ^ (r & 7)) << 4)) =
            make_uint4(y[0], y[1], y[2], y[3]);
      }
  }
}

// Operands of one epilogue row that do not depend on this kernel's result.
struct EpiRow {
  int64_t slot;   // q/k-rope: cache slot (-1: none)
  float cs[8];    // q/k-rope: cos of dims 4*(lane&15)+e, then sin
  uint2 res;      // residual add: this lane's 4 residual values
};

template <int EPI>
__device__ __forceinline__ void epi_fetch(EpiRow &o, const LinearFuse &f, const LinearArgs &a,
                                          int c, int tile, int lane) {
  if (EPI == kEpiAdd) {
    o.res = *reinterpret_cast<const uint2 *>(f.residual + c * f.res_stride + tile * kLnRows + lane * 4);
  } else if (EPI == kEpiQkRope) {
    o.slot = f.slot_mapping ? f.slot_mapping[c] : -1;
    if (tile < f.num_heads + f.num_kv_heads) {
      int64_t p = f.positions[c];
      if (p < 0 || p >= f.max_position) {
        if (lane == 0) raise_flag(a.error_flag, B200ASR_DEVERR_POSITION);
        p = 0;
      }
      const float4 cv = *reinterpret_cast<const float4 *>(f.cos_sin + p * kLnRows + (lane & 15) * 4);
      const float4 sv = *reinterpret_cast<const float4 *>(f.cos_sin + p * kLnRows + kLnRows / 2 +
                                                          (lane & 15) * 4);
      o.cs[0] = cv.x; o.cs[1] = cv.y; o.cs[2] = cv.z; o.cs[3] = cv.w;
      o.cs[4] = sv.x; o.cs[5] = sv.y; o.cs[6] = sv.z; o.cs[7] = sv.w;
    }
  }
}

// q/k RMSNorm + RoPE + paged store of one head vector: lane holds dims 4*lane .. +3 of
// row c of head `head` (0..H-1 query, H..H+Hkv-1 key, then value heads); nw = this lane's
// 4 q- or k-norm weights.
__device__ __forceinline__ void qk_rope_store4(const LinearFuse &f, const LinearArgs &a, int c,
                                               int head, int lane, const float *acc,
                                               const EpiRow &pre, const float *nw) {
  constexpr int D = kLnRows;
  // the bf16 projection output (paired conversions)
  const uint32_t xp[2] = {pack2(acc[0], acc[1]), pack2(acc[2], acc[3])};
  const float2 x01 = unpack2(xp[0]), x23 = unpack2(xp[1]);
  const float x[4] = {x01.x, x01.y, x23.x, x23.y};
  const int kv_hidden = f.num_kv_heads * D;
  const int64_t slot = pre.slot;
  const bool slot_bad = slot != -1 && (slot < 0 || slot >= f.num_slots);
  if (head >= f.num_heads + f.num_kv_heads) {  // value head: copy into the cache
    if (slot == -1) return;
    if (slot_bad) {
      if (lane == 0) raise_flag(a.error_flag, B200ASR_DEVERR_SLOT);
      return;
    }
    const int hv = head - f.num_heads - f.num_kv_heads;
    *reinterpret_cast<uint2 *>(f.v_cache + slot * kv_hidden + hv * D + lane * 4) =
        make_uint2(xp[0], xp[1]);
    return;
  }
  const bool is_q = head < f.num_heads;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss += x[e] * x[e];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(D) + f.qk_eps);
  float y[4];  // bf16(bf16(x * r) * w), paired conversions
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float2 n = round2_bf16(x[2 * e] * r, x[2 * e + 1] * r);
    const float2 m = round2_bf16(n.x * nw[2 * e], n.y * nw[2 * e + 1]);
    y[2 * e] = m.x;
    y[2 * e + 1] = m.y;
  }
  const bool first_half = lane < 16;
  float o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[e], 16);
    const float cv = pre.cs[e], sv = pre.cs[4 + e];
    o[e] = first_half ? __fsub_rn(__fmul_rn(y[e], cv), __fmul_rn(partner, sv))
                      : __fadd_rn(__fmul_rn(y[e], cv), __fmul_rn(partner, sv));
  }
  const uint2 packed = make_uint2(pack2(o[0], o[1]), pack2(o[2], o[3]));
  if (is_q) {
    *reinterpret_cast<uint2 *>(f.q_out + c * f.q_out_stride + head * D + lane * 4) = packed;
    return;
  }
  if (slot == -1) return;
  if (slot_bad) {
    if (lane == 0) raise_flag(a.error_flag, B200ASR_DEVERR_SLOT);
    return;
  }
  *reinterpret_cast<uint2 *>(f.k_cache + slot * kv_hidden + (head - f.num_heads) * D +
                             lane * 4) = packed;
}

template <int MP, bool NORM_IN, int EPI>
__global__ void __launch_bounds__(kLnThreads)
    linear_small_kernel(const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_x, const LinearArgs a,
                        const __grid_constant__ LinearFuse f) {
  using C = Ln<MP, NORM_IN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *stages = smem;
  float *red = reinterpret_cast<float *>(smem + C::STAGES * C::STAGE);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE + C::RED_BYTES);
  uint64_t *empty = full + C::STAGES;
  uint64_t *done = empty + C::STAGES;
  uint64_t *recv_bar = done + 1;  // completes when every peer's columns have arrived
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(recv_bar + 1);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_trigger();
  const int ks = a.k_split;
  const int cols = MP / ks;  // batch columns this CTA reduces (ks divides MP: powers of two)
  const int cols_log2 = __ffs(cols) - 1;
  const int kz = static_cast<int>(cluster_rank());
  const int tile = blockIdx.x / ks;
  const int k0 = kz * a.steps * kLnBK;
  int r0, r1;  // first weight row of the two 64-row boxes
  if (EPI == kEpiSilu) {
    r0 = tile * 64;
    r1 = a.silu_inner + tile * 64;
  } else {
    r0 = tile * kLnRows;
    r1 = r0 + 64;
  }

  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(recv_bar, 1);
    fence_barrier_init();
    // bytes the ks - 1 peers push: their 128 rows x this CTA's columns, fp32
    mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((ks - 1) * kLnRows * cols * 4));
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Peers push partials into this CTA's shared memory later: its receive barrier must be
  // initialised first. Arrive now, wait just before the first push (split cluster barrier,
  // so the weight loads and the prologue are not held up by it).
  if (ks > 1) cluster_arrive();

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    if (!NORM_IN) prefetch_tmap(&tm_x);
    // The weights are static: the first ring's worth is requested before waiting for
    // the kernel that produces x (programmatic dependent launch). With the RMSNorm
    // prologue the whole K slice fits the ring (the host guarantees steps <= stages).
    const int first = a.steps < C::STAGES ? a.steps : C::STAGES;
    for (int s = 0; s < first; ++s) {
      uint8_t *w = stages + s * C::STAGE;
      const int kc = k0 + s * kLnBK;
      mbar_arrive_expect_tx(&full[s], NORM_IN ? C::W_BYTES : C::STAGE);
      tma_load_2d(w, &tm_w, kc, r0, &full[s]);
      tma_load_2d(w + C::W_BYTES / 2, &tm_w, kc, r1, &full[s]);
    }
  }
  // static epilogue operand: this lane's q- or k-norm weights (the tile is one head)
  float qk_nw[4] = {0.f, 0.f, 0.f, 0.f};
  if (EPI == kEpiQkRope && tile < f.num_heads + f.num_kv_heads) {
    const __nv_bfloat16 *nw = (tile < f.num_heads ? f.q_w : f.k_w) + lane * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) qk_nw[e] = bf2f(nw[e]);
  }
  // L2 prefetch hints (data of later kernels; read-only, fixed before this step began)
  if (f.pf_cu_seqlens_k != nullptr && warp == 2)
    for (int b = blockIdx.x; b < f.pf_batch; b += gridDim.x) prefetch_sequence_kv(f, b, lane);
  if (warp == 3)
    for (int i = 0; i < 2; ++i)
      if (f.pf_range[i] != nullptr) prefetch_range_share(f.pf_range[i], f.pf_range_bytes[i], lane);
  if (NORM_IN) {
    uint4 wv[kLnStages][2];  // NORM_IN: C::STAGES == kLnStages
    norm_in_weights(wv, a, f, k0);
    pdl_wait();  // h and the tile sums come from the previous kernel
    __syncwarp();
    norm_in_fill<MP>(stages, a, f, k0, wv);
    fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
    __syncthreads();
  } else if (warp == 0 && lane == 0) {
    const int first = a.steps < C::STAGES ? a.steps : C::STAGES;
    pdl_wait();
    for (int s = 0; s < first; ++s)
      tma_load_2d(stages + s * C::STAGE + C::W_BYTES, &tm_x, k0 + s * kLnBK, 0, &full[s]);
    for (int s = first; s < a.steps; ++s) {
      const int st = s % C::STAGES;
      if (!mbar_wait(&empty[st], ((s / C::STAGES) - 1) & 1, a.error_flag, &abort_flag)) break;
      uint8_t *w = stages + st * C::STAGE;
      const int kc = k0 + s * kLnBK;
      mbar_arrive_expect_tx(&full[st], C::STAGE);
      tma_load_2d(w, &tm_w, kc, r0, &full[st]);
      tma_load_2d(w + C::W_BYTES / 2, &tm_w, kc, r1, &full[st]);
      tma_load_2d(w + C::W_BYTES, &tm_x, kc, 0, &full[st]);
    }
  }
  if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_bf16_f32(kLnRows, MP, false, false);
    bool ok = true;
    for (int s = 0; s < a.steps && ok; ++s) {
      const int st = s % C::STAGES;
      ok = mbar_wait(&full[st], (s / C::STAGES) & 1, a.error_flag, &abort_flag);
      if (!ok) break;
      tc_fence_after();
      const uint32_t wb = smem_addr(stages + st * C::STAGE), xb = wb + C::W_BYTES;
#pragma unroll
      for (int kk = 0; kk < kLnBK / 16; ++kk)
        umma_f16_ss(tmem, smem_desc_sw128(wb + kk * 32, 16, 1024),
                    smem_desc_sw128(xb + kk * 32, 16, 1024), idesc, (s > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&empty[st]);
    }
    if (ok) umma_commit(done);
  }

  // Every thread: its TMEM lane = weight row (w*32 + lane) of the tile -> partial[.][row].
  __syncwarp();  // the producer / MMA lanes rejoin their warps (tcgen05.ld is warp-aligned)
  // While the MMAs run: the epilogue operands of this warp's first rows (inputs written by
  // earlier kernels; the wait returns at once, x or h was already waited for).
  EpiRow pre[kEpiPre];
  if (EPI == kEpiAdd || EPI == kEpiQkRope) {
    pdl_wait();
#pragma unroll
    for (int i = 0; i < kEpiPre; ++i) {
      const int cl = warp + 4 * i, c = kz * cols + cl;
      if (cl < cols && c < a.m) epi_fetch<EPI>(pre[i], f, a, c, tile, lane);
    }
  }
  // Split-K reduction by push: CTA r of the cluster reduces batch columns
  // [r * cols, (r + 1) * cols). The partial (thread = weight row, one TMEM lane, all MP
  // columns) is first laid out column-major in this CTA's stage ring, free once the MMAs
  // are done; then 16-byte pieces (4 rows of one column) go to the CTA owning the
  // column: st.async into a peer's receive buffer (bytes counted on its barrier), a plain
  // store into this CTA's own. Receive buffer: red[src][cl][128 rows] fp32.
  const int row = warp * 32 + lane;
  const bool have = __all_sync(0xffffffffu, mbar_wait(done, 0, a.error_flag, &abort_flag));
  const uint32_t red_base = smem_addr(red), bar_base = smem_addr(recv_bar);
  float *colmaj = reinterpret_cast<float *>(stages);  // [MP][128]
  {
    tc_fence_after();
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll
    for (int cc = 0; cc < MP / 32; ++cc) {
      float v[32];
      if (have) {
        tmem_ld32(lane_base + cc * 32, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = 0.f;  // keeps the byte counts; the flag is raised
      }
#pragma unroll
      for (int c = 0; c < 32; ++c) colmaj[(cc * 32 + c) * kLnRows + row] = v[c];
    }
  }
  __syncthreads();
  if (ks > 1) cluster_wait();  // every peer's receive barrier is initialised
#pragma unroll
  for (int i = 0; i < MP * (kLnRows / 4) / kLnThreads; ++i) {
    const int id = i * kLnThreads + tid;  // (column, 4-row group): warps write 512 B runs
    const int col = id / (kLnRows / 4), q = id % (kLnRows / 4);
    const int r = col >> cols_log2, cl = col & (cols - 1);  // cols: a power of two
    const float4 v = *reinterpret_cast<const float4 *>(&colmaj[col * kLnRows + q * 4]);
    const uint32_t off = static_cast<uint32_t>(((kz * cols + cl) * kLnRows + q * 4) * 4);
    if (r == kz) {
      *reinterpret_cast<float4 *>(&red[(kz * cols + cl) * kLnRows + q * 4]) = v;
    } else {
      st_async_v4(mapa_shared(red_base + off, static_cast<uint32_t>(r)), v,
                  mapa_shared(bar_base, static_cast<uint32_t>(r)));
    }
  }
  tc_fence_before();
  __syncthreads();  // this CTA's own columns are in its buffer
  const bool got = mbar_wait(recv_bar, 0, a.error_flag, &abort_flag);  // the peers' columns

  pdl_wait();  // (returns at once: the producer's wait has passed) orders the writes below
  // Warp w takes local columns w, w + 4, ...; each lane 4 consecutive tile rows.
  for (int cl = warp, i = 0; cl < cols; cl += 4, ++i) {
    const int c = kz * cols + cl;
    if (c >= a.m) break;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);  // sources in rank order
    for (int j = 0; j < ks; ++j) {
      const float4 p = *reinterpret_cast<const float4 *>(&red[(j * cols + cl) * kLnRows + lane * 4]);
      acc.x += p.x;
      acc.y += p.y;
      acc.z += p.z;
      acc.w += p.w;
    }
    if (!have || !got) continue;
    if (EPI == kEpiSilu) {  // lanes 0-15: gate rows 0-63; lanes 16-31: the matching up rows
      const float ux = __shfl_down_sync(0xffffffffu, acc.x, 16);
      const float uy = __shfl_down_sync(0xffffffffu, acc.y, 16);
      const float uz = __shfl_down_sync(0xffffffffu, acc.z, 16);
      const float uw = __shfl_down_sync(0xffffffffu, acc.w, 16);
      if (lane < 16) {
        __nv_bfloat16 *dst = a.y + c * a.y_stride + tile * 64 + lane * 4;
        *reinterpret_cast<uint2 *>(dst) =
            make_uint2(silu_mul2(acc.x, acc.y, ux, uy), silu_mul2(acc.z, acc.w, uz, uw));
      }
    } else if (EPI == kEpiAdd) {
      const int col = tile * kLnRows + lane * 4;
      __nv_bfloat16 *rp = f.residual + c * f.res_stride + col;
      EpiRow cur;
      if (i == 0) cur = pre[0];
      else if (i == 1) cur = pre[1];
      else epi_fetch<EPI>(cur, f, a, c, tile, lane);
      const uint2 rv = cur.res;
      const float y[4] = {acc.x, acc.y, acc.z, acc.w};
      const float rr[4] = {__uint_as_float(rv.x << 16), __uint_as_float(rv.x & 0xffff0000u),
                           __uint_as_float(rv.y << 16), __uint_as_float(rv.y & 0xffff0000u)};
      const float2 y01 = round2_bf16(y[0], y[1]), y23 = round2_bf16(y[2], y[3]);
      const float yb[4] = {y01.x, y01.y, y23.x, y23.y};  // the bf16 projection output
      float h[4], ss = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        h[e] = yb[e] + rr[e];  // + residual, in fp32
        ss += h[e] * h[e];
      }
      *reinterpret_cast<uint2 *>(rp) = make_uint2(pack2(h[0], h[1]), pack2(h[2], h[3]));
      *reinterpret_cast<float4 *>(f.h_out + c * f.h_out_stride + col) =
          make_float4(h[0], h[1], h[2], h[3]);
      ss = warp_sum(ss);
      if (lane == 0) f.ss_out[c * (gridDim.x / ks) + tile] = ss;
    } else if (EPI == kEpiQkRope) {
      const float v4[4] = {acc.x, acc.y, acc.z, acc.w};
      EpiRow cur;
      if (i == 0) cur = pre[0];
      else if (i == 1) cur = pre[1];
      else epi_fetch<EPI>(cur, f, a, c, tile, lane);
      qk_rope_store4(f, a, c, tile, lane, v4, cur, qk_nw);
    } else {
      __nv_bfloat16 *dst = a.y + c * a.y_stride + tile * kLnRows + lane * 4;
      *reinterpret_cast<uint2 *>(dst) = make_uint2(pack2(acc.x, acc.y), pack2(acc.z, acc.w));
    }
  }
  // No closing cluster barrier: nothing reads another CTA's memory, and a CTA leaves only
  // after every byte addressed to it has arrived.
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// -----------------------------------------------------------------------------
// Persistent streaming projection for plain outputs with more 128-row tiles than two
// waves of CTAs (the lm_head: 151936 vocabulary rows = 1187 tiles). linear_small gives
// each tile a CTA, so such a launch runs in ~4 waves and every CTA pays its own set-up,
// first TMA round trip and epilogue. Here at most two CTAs per SM walk the tiles
// (t = blockIdx.x, + gridDim.x, ...) through one continuous TMA ring: warp 4 streams the
// weight and activation stages of tile after tile, warp 5 issues the MMAs into one of two
// TMEM accumulators, and warps 0-3 write a tile out of the other while the next tile
// accumulates. The MMA sequence of a tile is linear_small's with one K split (same
// stages, same order), so the outputs are identical.
// -----------------------------------------------------------------------------
constexpr int kLsThreads = 192;  // warps 0-3 epilogue, 4 producer, 5 TMEM + MMA
constexpr int kLsStages = 4;

template <int MP>
struct Ls {
  static constexpr int W_BYTES = kLnRows * kLnBK * 2;
  static constexpr int X_BYTES = MP * kLnBK * 2;
  static constexpr int STAGE = W_BYTES + X_BYTES;
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(kLsStages) * STAGE + 256;
  static constexpr uint32_t TMEM_COLS = 2 * MP;  // two accumulators
};

template <int MP>
__global__ void __launch_bounds__(kLsThreads, 2)
    linear_stream_kernel(const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_x, int m, int k_steps, int tiles,
                         __nv_bfloat16 *__restrict__ y, int64_t y_stride, int32_t *error_flag) {
  using C = Ls<MP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *stages = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(stages + kLsStages * C::STAGE);
  uint64_t *empty = full + kLsStages;
  uint64_t *acc_full = empty + kLsStages;   // [2] the tile's MMAs are done
  uint64_t *acc_empty = acc_full + 2;       // [2] the epilogue has read the accumulator
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  __shared__ int abort_flag;
  __shared__ int slot_last[kLsStages];      // ring position last issued into each slot

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_trigger();
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < kLsStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      slot_last[s] = -1;
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_x);
      // The weights are static: the first ring's worth (of the first tile) is requested
      // before waiting for the kernel that produces x; those stages' x follow the wait.
      const int first = k_steps < kLsStages ? k_steps : kLsStages;
      const int t0 = blockIdx.x;
      for (int s = 0; s < first; ++s) {
        uint8_t *w = stages + s * C::STAGE;
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        tma_load_2d(w, &tm_w, s * kLnBK, t0 * kLnRows, &full[s]);
        tma_load_2d(w + C::W_BYTES / 2, &tm_w, s * kLnBK, t0 * kLnRows + 64, &full[s]);
        slot_last[s] = s;
      }
      pdl_wait();
      for (int s = 0; s < first; ++s)
        tma_load_2d(stages + s * C::STAGE + C::W_BYTES, &tm_x, s * kLnBK, 0, &full[s]);
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        for (int s = 0; s < k_steps; ++s, ++it) {
          if (t == static_cast<int>(blockIdx.x) && s < first) continue;  // issued above
          const int st = static_cast<int>(it % kLsStages);
          ok = mbar_wait(&empty[st], ((it / kLsStages) - 1) & 1, error_flag, &abort_flag);
          if (!ok) break;
          uint8_t *w = stages + st * C::STAGE;
          mbar_arrive_expect_tx(&full[st], C::STAGE);
          tma_load_2d(w, &tm_w, s * kLnBK, t * kLnRows, &full[st]);
          tma_load_2d(w + C::W_BYTES / 2, &tm_w, s * kLnBK, t * kLnRows + 64, &full[st]);
          tma_load_2d(w + C::W_BYTES, &tm_x, s * kLnBK, 0, &full[st]);
          slot_last[st] = static_cast<int>(it);
        }
      }
      if (abort_flag)  // let the copies already issued land before the CTA exits
        for (int s = 0; s < kLsStages; ++s)
          if (slot_last[s] >= 0) mbar_drain(&full[s], (slot_last[s] / kLsStages) & 1);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kLnRows, MP, false, false);
      uint32_t it = 0;
      int j = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++j) {
        const int acc = j & 1;
        ok = mbar_wait(&acc_empty[acc], ((j >> 1) & 1) ^ 1, error_flag, &abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * MP;
        for (int s = 0; s < k_steps; ++s, ++it) {
          const int st = static_cast<int>(it % kLsStages);
          ok = mbar_wait(&full[st], (it / kLsStages) & 1, error_flag, &abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t wb = smem_addr(stages + st * C::STAGE), xb = wb + C::W_BYTES;
#pragma unroll
          for (int kk = 0; kk < kLnBK / 16; ++kk)
            umma_f16_ss(d, smem_desc_sw128(wb + kk * 32, 16, 1024),
                        smem_desc_sw128(xb + kk * 32, 16, 1024), idesc, (s > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&acc_full[acc]);
      }
    }
  } else {
    // ----------------------------------------------------------------- epilogue
    // Thread = TMEM lane = weight row (warp * 32 + lane) of the tile; column c of the
    // accumulator is activation row c. Each column's 32 lanes store 64 contiguous bytes.
    pdl_wait();  // outputs are written after the kernel before this one
    const int row = warp * 32 + lane;
    int j = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int acc = j & 1;
      if (!mbar_wait(&acc_full[acc], (j >> 1) & 1, error_flag, &abort_flag)) break;
      tc_fence_after();
      float v[MP];
      const uint32_t base = tmem + acc * MP + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll
      for (int cc = 0; cc < MP / 32; ++cc) tmem_ld32(base + cc * 32, v + cc * 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      __nv_bfloat16 *dst = y + static_cast<int64_t>(t) * kLnRows + row;
#pragma unroll
      for (int c = 0; c < MP; ++c)
        if (c < m) dst[c * y_stride] = __float2bfloat16_rn(v[c]);
    }
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int MP>
int launch_linear_stream(const void *x, int64_t x_stride, int m, int k, const void *w, int n,
                         void *y, int64_t y_stride, int32_t *error_flag, cudaStream_t stream) {
  using C = Ls<MP>;
  auto kfn = linear_stream_kernel<MP>;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(C::SMEM));
    if (e != cudaSuccess) {
      set_error("linear_small (stream): kernel configuration failed: %s", cudaGetErrorString(e));
      return B200ASR_ERR_CUDA;
    }
    configured = true;
  }
  CUtensorMap tw, tx;
  const uint64_t wdims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
  const uint64_t wstr[1] = {static_cast<uint64_t>(k) * 2};
  const uint32_t wbox[2] = {kLnBK, 64};
  if (!make_tmap_bf16(&tw, w, 2, wdims, wstr, wbox)) return B200ASR_ERR_CUDA;
  const uint64_t xdims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
  const uint64_t xstr[1] = {static_cast<uint64_t>(x_stride) * 2};
  const uint32_t xbox[2] = {kLnBK, MP};
  if (!make_tmap_bf16(&tx, x, 2, xdims, xstr, xbox)) return B200ASR_ERR_CUDA;
  const int tiles = n / kLnRows;
  const int grid = std::min(tiles, 2 * num_sms());
  B200_LAUNCH_CHECK_ERR(launch_kernel(kfn, dim3(grid), dim3(kLsThreads), C::SMEM, stream, true,
                                      1, tw, tx, m, k / kLnBK, tiles,
                                      static_cast<__nv_bfloat16 *>(y), y_stride, error_flag),
                        "linear_small (stream)");
  return B200ASR_OK;
}

// Rows of x (+ residual, updated in place) as the residual-add epilogue would leave them:
// h (fp32) and per-128-column partial sums of squares, for a following RMSNorm prologue
// or norm_apply. One warp per (row, 128 columns).
__global__ void rms_stats_kernel(const __nv_bfloat16 *__restrict__ x, __nv_bfloat16 *residual,
                                 int rows, int hidden, float *__restrict__ h_out,
                                 float *__restrict__ ss_out) {
  pdl_trigger();
  pdl_wait();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int tiles = hidden / kLnRows;
  if (gw >= rows * tiles) return;
  const int r = gw / tiles, t = gw - (gw / tiles) * tiles;
  const int col = t * kLnRows + lane * 4;
  const uint2 xv = *reinterpret_cast<const uint2 *>(x + static_cast<int64_t>(r) * hidden + col);
  float h[4] = {__uint_as_float(xv.x << 16), __uint_as_float(xv.x & 0xffff0000u),
                __uint_as_float(xv.y << 16), __uint_as_float(xv.y & 0xffff0000u)};
  if (residual != nullptr) {
    uint2 *rp = reinterpret_cast<uint2 *>(residual + static_cast<int64_t>(r) * hidden + col);
    const uint2 rv = *rp;
    h[0] += __uint_as_float(rv.x << 16);
    h[1] += __uint_as_float(rv.x & 0xffff0000u);
    h[2] += __uint_as_float(rv.y << 16);
    h[3] += __uint_as_float(rv.y & 0xffff0000u);
    *rp = make_uint2(pack2(h[0], h[1]), pack2(h[2], h[3]));
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss += h[e] * h[e];
  *reinterpret_cast<float4 *>(h_out + static_cast<int64_t>(r) * hidden + col) =
      make_float4(h[0], h[1], h[2], h[3]);
  ss = warp_sum(ss);
  if (lane == 0) ss_out[r * tiles + t] = ss;
}

// out = bf16(bf16(h * rsqrt(sum_t ss[t][r] / hidden + eps)) * w): the RMSNorm of rows
// held as h + tile sums (the model's final norm in a decode step).
__global__ void norm_apply_kernel(const float *__restrict__ h, const float *__restrict__ ss,
                                  const __nv_bfloat16 *__restrict__ weight, float eps, int rows,
                                  int hidden, __nv_bfloat16 *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int tiles = hidden / kLnRows;
  if (gw >= rows * tiles) return;
  const int r = gw / tiles, t = gw - (gw / tiles) * tiles;
  float sum = 0.f;
  for (int i = 0; i < tiles; ++i) sum += ss[r * tiles + i];
  const float rs = rsqrtf(sum / static_cast<float>(hidden) + eps);
  const int col = t * kLnRows + lane * 4;
  const float4 hv = *reinterpret_cast<const float4 *>(h + static_cast<int64_t>(r) * hidden + col);
  const uint2 wv = *reinterpret_cast<const uint2 *>(weight + col);
  const float w[4] = {__uint_as_float(wv.x << 16), __uint_as_float(wv.x & 0xffff0000u),
                      __uint_as_float(wv.y << 16), __uint_as_float(wv.y & 0xffff0000u)};
  const float hh[4] = {hv.x, hv.y, hv.z, hv.w};
  uint32_t y[2];  // bf16(bf16(h * rs) * w), paired conversions
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float2 n = round2_bf16(hh[2 * e] * rs, hh[2 * e + 1] * rs);
    y[e] = pack2(n.x * w[2 * e], n.y * w[2 * e + 1]);
  }
  *reinterpret_cast<uint2 *>(out + static_cast<int64_t>(r) * hidden + col) = make_uint2(y[0], y[1]);
}

// Smallest split (power of two dividing the K stages, <= 16) that puts >= 120 CTAs on
// the GPU; the largest allowed one when no split gets there.
int linear_split(int tiles, int k_steps) {
  int best = 1;
  for (int ks = 1; ks <= kLnMaxSplit; ks *= 2) {
    if (k_steps % ks) break;
    best = ks;
    if (tiles * ks >= 120) break;
  }
  return best;
}

template <int MP, bool NORM_IN, int EPI>
int launch_linear(const void *x, int64_t x_stride, int m, int k, const void *w, int n,
                  const LinearArgs &proto, const LinearFuse &fuse, int tiles,
                  cudaStream_t stream) {
  using C = Ln<MP, NORM_IN>;
  auto kfn = linear_small_kernel<MP, NORM_IN, EPI>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(C::SMEM));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) {
      set_error("linear_small: kernel configuration failed: %s", cudaGetErrorString(e));
      return B200ASR_ERR_CUDA;
    }
    configured = true;
  }
  CUtensorMap tw, tx;
  const uint64_t wdims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
  const uint64_t wstr[1] = {static_cast<uint64_t>(k) * 2};
  const uint32_t wbox[2] = {kLnBK, 64};
  if (!make_tmap_bf16(&tw, w, 2, wdims, wstr, wbox)) return B200ASR_ERR_CUDA;
  if (NORM_IN) {
    tx = tw;  // unused: the prologue builds x in shared memory
  } else {
    const uint64_t xdims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t xstr[1] = {static_cast<uint64_t>(x_stride) * 2};
    const uint32_t xbox[2] = {kLnBK, MP};
    if (!make_tmap_bf16(&tx, x, 2, xdims, xstr, xbox)) return B200ASR_ERR_CUDA;
  }
  LinearArgs a = proto;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kLnThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Halve a split whose cluster cannot be resident (16 CTAs is a non-portable size). The
  // RMSNorm prologue needs the whole K slice in the ring, so it cannot go below that.
  const int min_split = NORM_IN ? (k / kLnBK + kLnStages - 1) / kLnStages : 1;
  while (a.k_split > 1) {
    attr[0].val.clusterDim.x = a.k_split;
    cfg.gridDim = dim3(tiles * a.k_split, 1, 1);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kfn, &cfg) == cudaSuccess && clusters > 0)
      break;
    cudaGetLastError();
    if (a.k_split / 2 < min_split) {
      set_error("linear_small: a cluster of %d CTAs cannot be resident", a.k_split);
      return B200ASR_ERR_UNSUPPORTED;
    }
    a.k_split /= 2;
  }
  a.steps = k / kLnBK / a.k_split;
  cfg.gridDim = dim3(tiles * a.k_split, 1, 1);
  attr[0].val.clusterDim.x = a.k_split;
  if (pdl_enabled()) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, tw, tx, a, fuse);
  if (e != cudaSuccess) {
    set_error("linear_small: launch failed (%d x %d CTAs, cluster %d): %s", tiles, a.k_split,
              a.k_split, cudaGetErrorString(e));
    return B200ASR_ERR_CUDA;
  }
  return B200ASR_OK;
}

// K split for the RMSNorm prologue: at least enough CTAs that each K slice fits the
// ring; a power of two dividing the K stages, at most 16. 0 when none exists.
int norm_in_split(int tiles, int k_steps) {
  int ks = linear_split(tiles, k_steps);
  while (ks <= kLnMaxSplit && (k_steps % ks != 0 || k_steps / ks > kLnStages)) ks *= 2;
  return ks <= kLnMaxSplit && k_steps % ks == 0 ? ks : 0;
}

template <bool NORM_IN, int EPI>
int dispatch_linear(const void *x, int64_t x_stride, int m, int k, const void *w, int n,
                    const LinearArgs &a, const LinearFuse &f, int tiles, cudaStream_t st) {
  return m <= 32 ? launch_linear<32, NORM_IN, EPI>(x, x_stride, m, k, w, n, a, f, tiles, st)
                 : launch_linear<64, NORM_IN, EPI>(x, x_stride, m, k, w, n, a, f, tiles, st);
}

}  // namespace b200asr

using namespace b200asr;

namespace {

bool valid_weight_rows(int n, int silu_inner, int *tiles) {
  if (silu_inner) {
    if (silu_inner <= 0 || silu_inner % 64 != 0 || n != 2 * silu_inner) return false;
    *tiles = silu_inner / 64;
  } else {
    if (n <= 0 || n % kLnRows != 0) return false;
    *tiles = n / kLnRows;
  }
  return true;
}

LinearArgs make_args(int m, int k_split, int silu_inner, void *y, int64_t y_stride,
                     int32_t *error_flag) {
  LinearArgs a{};
  a.m = m;
  a.steps = 0;
  a.k_split = k_split;
  a.silu_inner = silu_inner;
  a.y = static_cast<__nv_bfloat16 *>(y);
  a.y_stride = y_stride;
  a.error_flag = error_flag;
  return a;
}

// Shared checks of the RMSNorm prologue's inputs; fills the prologue part of f.
int norm_in_args(const float *h, int64_t h_stride, const float *ss, int32_t ss_tiles,
                 const void *norm_weight, float eps, int32_t m, int32_t k, LinearFuse *f) {
  B200_REQUIRE(h && ss && norm_weight, "linear_small (RMSNorm prologue): null pointer");
  B200_REQUIRE(aligned16(h) && h_stride >= k && h_stride % 4 == 0 && aligned16(norm_weight),
               "linear_small (RMSNorm prologue): misaligned h or weight");
  B200_REQUIRE(ss_tiles >= 4 && ss_tiles <= kNormMaxTiles && ss_tiles % 4 == 0 && aligned16(ss),
               "linear_small: ss_tiles %d must be a multiple of 4 in [4, %d] (hidden %% 512 == 0)",
               ss_tiles, kNormMaxTiles);
  f->h = h;
  f->h_stride = h_stride;
  f->ss = ss;
  f->ss_tiles = ss_tiles;
  f->norm_w = static_cast<const __nv_bfloat16 *>(norm_weight);
  f->norm_eps = eps;
  f->norm_k = k;
  (void)m;
  return B200ASR_OK;
}

// Validates a b200asr_l2_prefetch and fills the prefetch part of f (NULL: none).
int prefetch_args(const b200asr_l2_prefetch *p, LinearFuse *f) {
  if (p == nullptr) return B200ASR_OK;
  if (p->cu_seqlens_k != nullptr) {
    B200_REQUIRE(p->block_tables && p->bt_stride > 0 && p->batch >= 0 && p->block_size > 0 &&
                     p->num_kv_heads > 0 && p->head_dim > 0 && p->k_cache && p->v_cache &&
                     p->num_slots > 0 && p->num_slots % p->block_size == 0 &&
                     aligned16(p->k_cache) && aligned16(p->v_cache) &&
                     (p->num_kv_heads * p->head_dim * 2) % 16 == 0,
                 "l2_prefetch: bad K/V geometry");
    f->pf_cu_seqlens_k = p->cu_seqlens_k;
    f->pf_block_tables = p->block_tables;
    f->pf_bt_stride = p->bt_stride;
    f->pf_batch = p->batch;
    f->pf_block_size = p->block_size;
    f->pf_row_bytes = p->num_kv_heads * p->head_dim * 2;
    f->pf_num_blocks = p->num_slots / p->block_size;
    f->pf_k_cache = static_cast<const uint8_t *>(p->k_cache);
    f->pf_v_cache = static_cast<const uint8_t *>(p->v_cache);
  }
  for (int i = 0; i < 2; ++i) {
    if (p->range[i] == nullptr) continue;
    B200_REQUIRE(aligned16(p->range[i]) && p->range_bytes[i] > 0 && p->range_bytes[i] % 16 == 0,
                 "l2_prefetch: range %d must be 16-byte aligned and a multiple of 16 bytes", i);
    f->pf_range[i] = static_cast<const uint8_t *>(p->range[i]);
    f->pf_range_bytes[i] = p->range_bytes[i];
  }
  return B200ASR_OK;
}

}  // namespace

extern "C" int b200asr_linear_small(const void *x, int64_t x_row_stride, int32_t m, int32_t k,
                                    const void *w, int32_t n, int32_t silu_inner, void *y,
                                    int64_t y_row_stride, int32_t *error_flag,
                                    b200asr_stream_t stream) {
  B200_REQUIRE(m >= 0 && m <= 64, "linear_small: %d rows (at most 64)", m);
  if (m == 0) return B200ASR_OK;
  B200_REQUIRE(k > 0 && k % kLnBK == 0, "linear_small: K %d must be a multiple of %d", k, kLnBK);
  B200_REQUIRE(x && w && y, "linear_small: null pointer");
  B200_REQUIRE(aligned16(x) && aligned16(w) && aligned16(y) && x_row_stride >= k &&
                   x_row_stride % 8 == 0 && y_row_stride % 4 == 0,
               "linear_small: misaligned tensor");
  int tiles = 0;
  B200_REQUIRE(valid_weight_rows(n, silu_inner, &tiles),
               "linear_small: N %d / SiLU inner %d unsupported (N %% 128 == 0, or N = 2 I with "
               "I %% 64 == 0)", n, silu_inner);
  B200_REQUIRE(y_row_stride >= (silu_inner ? silu_inner : n),
               "linear_small: output row stride too small");
  const LinearArgs a = make_args(m, linear_split(tiles, k / kLnBK), silu_inner, y, y_row_stride,
                                 error_flag);
  const LinearFuse f = {};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // More tiles than two waves of CTAs, no K split: the persistent streaming kernel.
  if (!silu_inner && a.k_split == 1 && tiles > 2 * num_sms())
    return m <= 32 ? launch_linear_stream<32>(x, x_row_stride, m, k, w, n, y, y_row_stride,
                                              error_flag, st)
                   : launch_linear_stream<64>(x, x_row_stride, m, k, w, n, y, y_row_stride,
                                              error_flag, st);
  return silu_inner ? dispatch_linear<false, kEpiSilu>(x, x_row_stride, m, k, w, n, a, f, tiles, st)
                    : dispatch_linear<false, kEpiPlain>(x, x_row_stride, m, k, w, n, a, f, tiles, st);
}

extern "C" int b200asr_linear_small_add(const void *x, int64_t x_row_stride, int32_t m, int32_t k,
                                        const void *w, int32_t n, void *residual,
                                        int64_t residual_row_stride, float *h_out,
                                        int64_t h_row_stride, float *ss_out,
                                        const b200asr_l2_prefetch *prefetch,
                                        int32_t *error_flag, b200asr_stream_t stream) {
  B200_REQUIRE(m >= 0 && m <= 64, "linear_small_add: %d rows (at most 64)", m);
  if (m == 0) return B200ASR_OK;
  B200_REQUIRE(k > 0 && k % kLnBK == 0, "linear_small_add: K %d must be a multiple of %d", k, kLnBK);
  B200_REQUIRE(n > 0 && n % kLnRows == 0 && n / kLnRows <= 64,
               "linear_small_add: N %d must be a multiple of %d (at most 64 tiles)", n, kLnRows);
  B200_REQUIRE(x && w && residual && h_out && ss_out, "linear_small_add: null pointer");
  B200_REQUIRE(aligned16(x) && aligned16(w) && aligned16(residual) && aligned16(h_out) &&
                   x_row_stride >= k && x_row_stride % 8 == 0 && residual_row_stride >= n &&
                   residual_row_stride % 8 == 0 && h_row_stride >= n && h_row_stride % 4 == 0,
               "linear_small_add: misaligned tensor");
  const int tiles = n / kLnRows;
  const LinearArgs a = make_args(m, linear_split(tiles, k / kLnBK), 0, nullptr, 0, error_flag);
  LinearFuse f = {};
  f.residual = static_cast<__nv_bfloat16 *>(residual);
  f.res_stride = residual_row_stride;
  f.h_out = h_out;
  f.h_out_stride = h_row_stride;
  f.ss_out = ss_out;
  const int prc = prefetch_args(prefetch, &f);
  if (prc != B200ASR_OK) return prc;
  return dispatch_linear<false, kEpiAdd>(x, x_row_stride, m, k, w, n, a, f, tiles,
                                         static_cast<cudaStream_t>(stream));
}

extern "C" int b200asr_linear_small_norm(const float *h, int64_t h_row_stride, const float *ss,
                                         int32_t ss_tiles, const void *norm_weight, float eps,
                                         int32_t m, int32_t k, const void *w, int32_t n,
                                         int32_t silu_inner, void *y, int64_t y_row_stride,
                                         const b200asr_l2_prefetch *prefetch,
                                         int32_t *error_flag, b200asr_stream_t stream) {
  B200_REQUIRE(m >= 0 && m <= 64, "linear_small_norm: %d rows (at most 64)", m);
  if (m == 0) return B200ASR_OK;
  B200_REQUIRE(k > 0 && k % kLnBK == 0, "linear_small_norm: K %d must be a multiple of %d", k, kLnBK);
  B200_REQUIRE(w && y && aligned16(w) && aligned16(y) && y_row_stride % 4 == 0,
               "linear_small_norm: null or misaligned tensor");
  LinearFuse f = {};
  const int rc = norm_in_args(h, h_row_stride, ss, ss_tiles, norm_weight, eps, m, k, &f);
  if (rc != B200ASR_OK) return rc;
  const int prc = prefetch_args(prefetch, &f);
  if (prc != B200ASR_OK) return prc;
  int tiles = 0;
  B200_REQUIRE(valid_weight_rows(n, silu_inner, &tiles),
               "linear_small_norm: N %d / SiLU inner %d unsupported", n, silu_inner);
  B200_REQUIRE(y_row_stride >= (silu_inner ? silu_inner : n),
               "linear_small_norm: output row stride too small");
  const int ks = norm_in_split(tiles, k / kLnBK);
  B200_REQUIRE(ks > 0, "linear_small_norm: K %d too large for the RMSNorm prologue", k);
  const LinearArgs a = make_args(m, ks, silu_inner, y, y_row_stride, error_flag);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return silu_inner ? dispatch_linear<true, kEpiSilu>(nullptr, 0, m, k, w, n, a, f, tiles, st)
                    : dispatch_linear<true, kEpiPlain>(nullptr, 0, m, k, w, n, a, f, tiles, st);
}

extern "C" int b200asr_linear_small_norm_qk_rope(
    const float *h, int64_t h_row_stride, const float *ss, int32_t ss_tiles,
    const void *norm_weight, float eps, int32_t m, int32_t k, const void *w, int32_t num_heads,
    int32_t num_kv_heads, int32_t head_dim, const void *q_norm_weight, const void *k_norm_weight,
    float qk_eps, const int64_t *positions, const float *cos_sin_cache, int32_t max_position,
    void *q_out, int64_t q_out_row_stride, void *k_cache, void *v_cache,
    const int32_t *slot_mapping, int64_t num_slots, const b200asr_l2_prefetch *prefetch,
    int32_t *error_flag, b200asr_stream_t stream) {
  B200_REQUIRE(m >= 0 && m <= 64, "linear_small_norm_qk_rope: %d rows (at most 64)", m);
  if (m == 0) return B200ASR_OK;
  B200_REQUIRE(head_dim == kLnRows, "linear_small_norm_qk_rope: head_dim %d (needs %d)", head_dim,
               kLnRows);
  B200_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
               "linear_small_norm_qk_rope: bad head counts %d / %d", num_heads, num_kv_heads);
  B200_REQUIRE(k > 0 && k % kLnBK == 0, "linear_small_norm_qk_rope: K %d must be a multiple of %d",
               k, kLnBK);
  B200_REQUIRE(w && aligned16(w) && q_norm_weight && k_norm_weight && positions && cos_sin_cache &&
                   q_out && aligned16(q_out) && q_out_row_stride >= num_heads * head_dim &&
                   q_out_row_stride % 4 == 0 && k_cache && v_cache && aligned16(k_cache) &&
                   aligned16(v_cache) && max_position > 0,
               "linear_small_norm_qk_rope: null or misaligned tensor");
  LinearFuse f = {};
  const int rc = norm_in_args(h, h_row_stride, ss, ss_tiles, norm_weight, eps, m, k, &f);
  if (rc != B200ASR_OK) return rc;
  const int n = (num_heads + 2 * num_kv_heads) * head_dim;
  const int tiles = n / kLnRows;
  const int ks = norm_in_split(tiles, k / kLnBK);
  B200_REQUIRE(ks > 0, "linear_small_norm_qk_rope: K %d too large for the RMSNorm prologue", k);
  f.num_heads = num_heads;
  f.num_kv_heads = num_kv_heads;
  f.q_w = static_cast<const __nv_bfloat16 *>(q_norm_weight);
  f.k_w = static_cast<const __nv_bfloat16 *>(k_norm_weight);
  f.qk_eps = qk_eps;
  f.positions = positions;
  f.cos_sin = cos_sin_cache;
  f.max_position = max_position;
  f.q_out = static_cast<__nv_bfloat16 *>(q_out);
  f.q_out_stride = q_out_row_stride;
  f.k_cache = static_cast<__nv_bfloat16 *>(k_cache);
  f.v_cache = static_cast<__nv_bfloat16 *>(v_cache);
  f.slot_mapping = slot_mapping;
  f.num_slots = num_slots;
  const int prc = prefetch_args(prefetch, &f);
  if (prc != B200ASR_OK) return prc;
  const LinearArgs a = make_args(m, ks, 0, nullptr, 0, error_flag);
  return dispatch_linear<true, kEpiQkRope>(nullptr, 0, m, k, w, n, a, f, tiles,
                                           static_cast<cudaStream_t>(stream));
}

extern "C" int b200asr_linear_small_qk_rope(
    const void *x, int64_t x_row_stride, int32_t m, int32_t k, const void *w, int32_t num_heads,
    int32_t num_kv_heads, int32_t head_dim, const void *q_norm_weight, const void *k_norm_weight,
    float qk_eps, const int64_t *positions, const float *cos_sin_cache, int32_t max_position,
    void *q_out, int64_t q_out_row_stride, void *k_cache, void *v_cache,
    const int32_t *slot_mapping, int64_t num_slots, int32_t *error_flag,
    b200asr_stream_t stream) {
  B200_REQUIRE(m >= 0 && m <= 64, "linear_small_qk_rope: %d rows (at most 64)", m);
  if (m == 0) return B200ASR_OK;
  B200_REQUIRE(head_dim == kLnRows, "linear_small_qk_rope: head_dim %d (needs %d)", head_dim,
               kLnRows);
  B200_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
               "linear_small_qk_rope: bad head counts %d / %d", num_heads, num_kv_heads);
  B200_REQUIRE(k > 0 && k % kLnBK == 0, "linear_small_qk_rope: K %d must be a multiple of %d", k,
               kLnBK);
  B200_REQUIRE(x && aligned16(x) && x_row_stride >= k && x_row_stride % 8 == 0 && w &&
                   aligned16(w) && q_norm_weight && k_norm_weight && positions && cos_sin_cache &&
                   q_out && aligned16(q_out) && q_out_row_stride >= num_heads * head_dim &&
                   q_out_row_stride % 4 == 0 && k_cache && v_cache && aligned16(k_cache) &&
                   aligned16(v_cache) && max_position > 0,
               "linear_small_qk_rope: null or misaligned tensor");
  LinearFuse f = {};
  const int n = (num_heads + 2 * num_kv_heads) * head_dim;
  const int tiles = n / kLnRows;
  f.num_heads = num_heads;
  f.num_kv_heads = num_kv_heads;
  f.q_w = static_cast<const __nv_bfloat16 *>(q_norm_weight);
  f.k_w = static_cast<const __nv_bfloat16 *>(k_norm_weight);
  f.qk_eps = qk_eps;
  f.positions = positions;
  f.cos_sin = cos_sin_cache;
  f.max_position = max_position;
  f.q_out = static_cast<__nv_bfloat16 *>(q_out);
  f.q_out_stride = q_out_row_stride;
  f.k_cache = static_cast<__nv_bfloat16 *>(k_cache);
  f.v_cache = static_cast<__nv_bfloat16 *>(v_cache);
  f.slot_mapping = slot_mapping;
  f.num_slots = num_slots;
  const LinearArgs a = make_args(m, linear_split(tiles, k / kLnBK), 0, nullptr, 0, error_flag);
  return dispatch_linear<false, kEpiQkRope>(x, x_row_stride, m, k, w, n, a, f, tiles,
                                            static_cast<cudaStream_t>(stream));
}

extern "C" int b200asr_rms_stats(const void *x, void *residual, int32_t rows, int32_t hidden,
                                 float *h_out, float *ss_out, b200asr_stream_t stream) {
  B200_REQUIRE(rows >= 0 && rows <= 64, "rms_stats: %d rows (at most 64)", rows);
  if (rows == 0) return B200ASR_OK;
  B200_REQUIRE(hidden > 0 && hidden % kLnRows == 0 && hidden / kLnRows <= 64,
               "rms_stats: hidden %d must be a multiple of %d", hidden, kLnRows);
  B200_REQUIRE(x && h_out && ss_out && aligned16(x) && aligned16(h_out) &&
                   (residual == nullptr || aligned16(residual)),
               "rms_stats: null or misaligned tensor");
  const int warps = rows * (hidden / kLnRows);
  B200_LAUNCH_CHECK_ERR(
      launch_kernel(rms_stats_kernel, dim3((warps + 7) / 8), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), true, 1,
                    static_cast<const __nv_bfloat16 *>(x), static_cast<__nv_bfloat16 *>(residual),
                    static_cast<int>(rows), static_cast<int>(hidden), h_out, ss_out),
      "rms_stats");
  return B200ASR_OK;
}

extern "C" int b200asr_norm_apply(const float *h, const float *ss, const void *weight, float eps,
                                  int32_t rows, int32_t hidden, void *out,
                                  b200asr_stream_t stream) {
  B200_REQUIRE(rows >= 0 && rows <= 64, "norm_apply: %d rows (at most 64)", rows);
  if (rows == 0) return B200ASR_OK;
  B200_REQUIRE(hidden > 0 && hidden % kLnRows == 0 && hidden / kLnRows <= 64,
               "norm_apply: hidden %d must be a multiple of %d", hidden, kLnRows);
  B200_REQUIRE(h && ss && weight && out && aligned16(h) && aligned16(out),
               "norm_apply: null or misaligned tensor");
  const int warps = rows * (hidden / kLnRows);
  B200_LAUNCH_CHECK_ERR(
      launch_kernel(norm_apply_kernel, dim3((warps + 7) / 8), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), true, 1, h, ss,
                    static_cast<const __nv_bfloat16 *>(weight), eps, static_cast<int>(rows),
                    static_cast<int>(hidden), static_cast<__nv_bfloat16 *>(out)),
      "norm_apply");
  return B200ASR_OK;
}
