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
//    cluster; each accumulates its K slice in TMEM, stages the 128 x MP fp32 partial in
//    shared memory, and after a cluster barrier every CTA sums a share of the batch rows
//    across the cluster through distributed shared memory (on-chip, no workspace, no
//    second kernel) and writes bf16.
//  * A 4-deep TMA ring (128-byte swizzle) per CTA: each weight tile arrives as two 64-row
//    boxes, the activation tile as one box whose rows past M are zero-filled.
//  * Fused SiLU*mul (layers/activation.py:11-14) for gate_up_proj: a tile's two boxes are
//    64 gate rows and the matching 64 up rows of the unmodified [gate; up] weight, so the
//    epilogue writes silu(gate) * up directly, with the rounding of the unfused path
//    (bf16 projections, bf16 silu, bf16 product).
//
// No TMA multicast is used. Every CTA arrives at both cluster barriers whatever happens
// (a timed-out mbarrier wait only skips work), so no CTA waits for one that left.
#include "common.cuh"

namespace b200asr {

constexpr int kLnBK = 64;       // K elements per stage (one 128-byte swizzle row)
constexpr int kLnRows = 128;    // weight rows per CTA (MMA M)
constexpr int kLnStages = 4;
constexpr int kLnThreads = 128;
constexpr int kLnMaxSplit = 16;

template <int MP>
struct Ln {
  static constexpr int W_BYTES = kLnRows * kLnBK * 2;  // 16 KiB
  static constexpr int X_BYTES = MP * kLnBK * 2;       // 4 or 8 KiB
  static constexpr int STAGE = W_BYTES + X_BYTES;
  static constexpr int RED_BYTES = MP * kLnRows * 4;   // [MP][128] fp32 partial
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(kLnStages) * STAGE + RED_BYTES + 256;
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

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t local_saddr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_saddr), "r"(rank));
  float4 v;  // ordered after the cluster barrier by the barrier's acquire
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote));
  return v;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t c0,
                                            int32_t c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// silu(g) * u with the unfused path's roundings: g, u are bf16 projections, F.silu
// returns bf16, the product is rounded once more by the caller's pack.
__device__ __forceinline__ float silu_mul1(float g, float u) {
  const float gb = bf2f(f2bf(g)), ub = bf2f(f2bf(u));
  return bf2f(f2bf(gb / (1.0f + expf(-gb)))) * ub;
}

template <int MP>
__global__ void __launch_bounds__(kLnThreads)
    linear_small_kernel(const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_x, const LinearArgs a) {
  using C = Ln<MP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *stages = smem;
  float *red = reinterpret_cast<float *>(smem + kLnStages * C::STAGE);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kLnStages * C::STAGE + C::RED_BYTES);
  uint64_t *empty = full + kLnStages;
  uint64_t *done = empty + kLnStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_trigger();
  const int ks = a.k_split;
  const int kz = static_cast<int>(cluster_rank());
  const int tile = blockIdx.x / ks;
  const int k0 = kz * a.steps * kLnBK;
  int r0, r1;  // first weight row of the two 64-row boxes
  if (a.silu_inner) {
    r0 = tile * 64;
    r1 = a.silu_inner + tile * 64;
  } else {
    r0 = tile * kLnRows;
    r1 = r0 + 64;
  }

  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < kLnStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
    // The weights are static: the first ring's worth is requested before waiting for
    // the kernel that produces x (programmatic dependent launch).
    const int first = a.steps < kLnStages ? a.steps : kLnStages;
    for (int s = 0; s < first; ++s) {
      uint8_t *w = stages + s * C::STAGE;
      const int kc = k0 + s * kLnBK;
      mbar_arrive_expect_tx(&full[s], C::STAGE);
      tma_load_2d(w, &tm_w, kc, r0, &full[s]);
      tma_load_2d(w + C::W_BYTES / 2, &tm_w, kc, r1, &full[s]);
    }
    pdl_wait();
    for (int s = 0; s < first; ++s)
      tma_load_2d(stages + s * C::STAGE + C::W_BYTES, &tm_x, k0 + s * kLnBK, 0, &full[s]);
    for (int s = first; s < a.steps; ++s) {
      const int st = s % kLnStages;
      if (!mbar_wait(&empty[st], ((s / kLnStages) - 1) & 1, a.error_flag, &abort_flag)) break;
      uint8_t *w = stages + st * C::STAGE;
      const int kc = k0 + s * kLnBK;
      mbar_arrive_expect_tx(&full[st], C::STAGE);
      tma_load_2d(w, &tm_w, kc, r0, &full[st]);
      tma_load_2d(w + C::W_BYTES / 2, &tm_w, kc, r1, &full[st]);
      tma_load_2d(w + C::W_BYTES, &tm_x, kc, 0, &full[st]);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_bf16_f32(kLnRows, MP, false, false);
    bool ok = true;
    for (int s = 0; s < a.steps && ok; ++s) {
      const int st = s % kLnStages;
      ok = mbar_wait(&full[st], (s / kLnStages) & 1, a.error_flag, &abort_flag);
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
  const int row = warp * 32 + lane;
  const bool have = __all_sync(0xffffffffu, mbar_wait(done, 0, a.error_flag, &abort_flag));
  if (have) {
    tc_fence_after();
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll
    for (int cc = 0; cc < MP / 32; ++cc) {
      float v[32];
      tmem_ld32(lane_base + cc * 32, v);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) red[(cc * 32 + c) * kLnRows + row] = v[c];
    }
  }
  tc_fence_before();
  cluster_barrier();  // every partial of the cluster is in shared memory

  pdl_wait();  // (returns at once: the producer's wait has passed) orders the writes below
  // This CTA reduces batch rows kz, kz + ks, ...; warp w takes every 4th of them and each
  // lane 4 consecutive tile rows (128 rows = 32 lanes x 4).
  const uint32_t red_base = smem_addr(red);
  for (int c = kz + warp * ks; c < a.m; c += 4 * ks) {
    // all ks loads in flight before the first add (one DSMEM round trip, not ks)
    const uint32_t at = red_base + (c * kLnRows + lane * 4) * 4;
    float4 part[kLnMaxSplit];
#pragma unroll
    for (int j = 0; j < kLnMaxSplit; ++j)
      if (j < ks) part[j] = ld_dsmem_f4(at, static_cast<uint32_t>(j));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < kLnMaxSplit; ++j) {
      if (j < ks) {
        acc.x += part[j].x;
        acc.y += part[j].y;
        acc.z += part[j].z;
        acc.w += part[j].w;
      }
    }
    if (!have) continue;
    if (a.silu_inner) {  // lanes 0-15: gate rows 0-63; lanes 16-31: the matching up rows
      const float ux = __shfl_down_sync(0xffffffffu, acc.x, 16);
      const float uy = __shfl_down_sync(0xffffffffu, acc.y, 16);
      const float uz = __shfl_down_sync(0xffffffffu, acc.z, 16);
      const float uw = __shfl_down_sync(0xffffffffu, acc.w, 16);
      if (lane < 16) {
        __nv_bfloat16 *dst = a.y + c * a.y_stride + tile * 64 + lane * 4;
        *reinterpret_cast<uint2 *>(dst) =
            make_uint2(pack2(silu_mul1(acc.x, ux), silu_mul1(acc.y, uy)),
                       pack2(silu_mul1(acc.z, uz), silu_mul1(acc.w, uw)));
      }
    } else {
      __nv_bfloat16 *dst = a.y + c * a.y_stride + tile * kLnRows + lane * 4;
      *reinterpret_cast<uint2 *>(dst) = make_uint2(pack2(acc.x, acc.y), pack2(acc.z, acc.w));
    }
  }
  cluster_barrier();  // peers finished reading this CTA's shared memory
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
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

template <int MP>
int launch_linear(const void *x, int64_t x_stride, int m, int k, const void *w, int n,
                  const LinearArgs &proto, int tiles, cudaStream_t stream) {
  using C = Ln<MP>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(linear_small_kernel<MP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(C::SMEM));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(linear_small_kernel<MP>,
                               cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
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
  const uint64_t xdims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
  const uint64_t xstr[1] = {static_cast<uint64_t>(x_stride) * 2};
  const uint32_t xbox[2] = {kLnBK, MP};
  if (!make_tmap_bf16(&tw, w, 2, wdims, wstr, wbox) || !make_tmap_bf16(&tx, x, 2, xdims, xstr, xbox))
    return B200ASR_ERR_CUDA;
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
  // Halve a split whose cluster cannot be resident (16 CTAs is a non-portable size).
  while (a.k_split > 1) {
    attr[0].val.clusterDim.x = a.k_split;
    cfg.gridDim = dim3(tiles * a.k_split, 1, 1);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, linear_small_kernel<MP>, &cfg) == cudaSuccess &&
        clusters > 0)
      break;
    cudaGetLastError();
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, linear_small_kernel<MP>, tw, tx, a);
  if (e != cudaSuccess) {
    set_error("linear_small: launch failed (%d x %d CTAs, cluster %d): %s", tiles, a.k_split,
              a.k_split, cudaGetErrorString(e));
    return B200ASR_ERR_CUDA;
  }
  return B200ASR_OK;
}

}  // namespace b200asr

using namespace b200asr;

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
  int tiles;
  if (silu_inner) {
    B200_REQUIRE(silu_inner > 0 && silu_inner % 64 == 0 && n == 2 * silu_inner,
                 "linear_small: SiLU*mul needs 2 x I weight rows with I %% 64 == 0 (I=%d, N=%d)",
                 silu_inner, n);
    B200_REQUIRE(y_row_stride >= silu_inner, "linear_small: output row stride too small");
    tiles = silu_inner / 64;
  } else {
    B200_REQUIRE(n > 0 && n % kLnRows == 0, "linear_small: N %d must be a multiple of %d", n,
                 kLnRows);
    B200_REQUIRE(y_row_stride >= n, "linear_small: output row stride too small");
    tiles = n / kLnRows;
  }
  LinearArgs a;
  a.m = m;
  a.steps = 0;
  a.k_split = linear_split(tiles, k / kLnBK);
  a.silu_inner = silu_inner;
  a.y = static_cast<__nv_bfloat16 *>(y);
  a.y_stride = y_row_stride;
  a.error_flag = error_flag;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return m <= 32 ? launch_linear<32>(x, x_row_stride, m, k, w, n, a, tiles, st)
                 : launch_linear<64>(x, x_row_stride, m, k, w, n, a, tiles, st);
}

