// Greedy sampler: argmax over the vocabulary of each row.
//
// Replaces the greedy branch of Sampler.forward (layers/sampler.py:16-20):
// logits.float().argmax(-1), which returns the FIRST index of the maximum and treats
// NaN as larger than every number.
//
// A row of 151,936 bf16 logits is 297 KiB. One CTA per row would leave most of the
// 148 SMs idle at decode batch sizes, so each row is split over a cluster of 8 CTAs;
// every CTA reduces its slice with 16-byte loads and a warp/block reduction, and the
// cluster leader combines the 8 partial results through distributed shared memory.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace b200asr {

constexpr int kArgmaxCluster = 8;
constexpr int kArgmaxThreads = 512;
constexpr int kArgmaxUnroll = 8;

struct Best {
  float v;
  int idx;
};

// True if (v, i) should replace (bv, bi): larger value, NaN beats numbers, ties and
// NaN-vs-NaN go to the lower index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  const bool vn = isnan(v), bn = isnan(bv);
  if (vn || bn) return vn && (!bn || i < bi);
  return v > bv || (v == bv && i < bi);
}

__global__ void __cluster_dims__(kArgmaxCluster, 1, 1) __launch_bounds__(kArgmaxThreads)
    greedy_argmax_kernel(const __nv_bfloat16 *__restrict__ logits, int64_t row_stride, int vocab,
                         int64_t *__restrict__ out_ids) {
  __shared__ Best warp_best[kArgmaxThreads / 32];
  __shared__ Best cta_best;
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.y;
  const __nv_bfloat16 *x = logits + row * row_stride;

  // Slice [lo, hi) of this CTA, in multiples of 8 elements.
  const int n8 = (vocab + 7) / 8;
  const int per = (n8 + kArgmaxCluster - 1) / kArgmaxCluster;
  const int lo8 = rank * per, hi8 = min(n8, lo8 + per);

  float bv = -INFINITY;
  int bi = INT_MAX;
  const bool vec_ok = (row_stride % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  // kArgmaxUnroll 16-byte loads per thread are in flight before the first compare (the
  // slice is a handful of loads per thread, so issuing them one by one would serialise
  // that many DRAM round trips). Ties resolve by index, so the visiting order is free.
  for (int c0 = lo8 + threadIdx.x; c0 < hi8; c0 += kArgmaxUnroll * blockDim.x) {
    uint4 raw[kArgmaxUnroll];
#pragma unroll
    for (int u = 0; u < kArgmaxUnroll; ++u) {
      const int c = c0 + u * static_cast<int>(blockDim.x);
      if (vec_ok && c < hi8 && c * 8 + 8 <= vocab)
        raw[u] = __ldg(reinterpret_cast<const uint4 *>(x + c * 8));
    }
#pragma unroll
    for (int u = 0; u < kArgmaxUnroll; ++u) {
      const int c = c0 + u * static_cast<int>(blockDim.x);
      if (c >= hi8) break;
      const int base = c * 8;
      float v[8];
      if (vec_ok && base + 8 <= vocab) {
        unpack8(raw[u], v);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = base + e < vocab ? bf2f(x[base + e]) : -INFINITY;
      }
      // Fast reject: a thread visits its indices in increasing order, so a vector can only
      // change its best if it holds a strictly larger number or a NaN.
      float m = v[0];
      bool nan = v[0] != v[0];
#pragma unroll
      for (int e = 1; e < 8; ++e) {
        m = fmaxf(m, v[e]);
        nan |= v[e] != v[e];
      }
      if (!nan && !(m > bv)) continue;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (base + e < vocab && better(v[e], base + e, bv, bi)) {
          bv = v[e];
          bi = base + e;
        }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) warp_best[warp] = {bv, bi};
  __syncthreads();
  if (warp == 0) {
    Best b = lane < kArgmaxThreads / 32 ? warp_best[lane] : Best{-INFINITY, INT_MAX};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, b.v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, b.idx, o);
      if (better(ov, oi, b.v, b.idx)) b = {ov, oi};
    }
    if (lane == 0) cta_best = b;
  }
  cluster.sync();
  if (rank == 0 && warp == 0) {
    // lane r < 8 reads CTA r's result (the remote reads in flight together), then a
    // shuffle reduction; better() orders by value and index, so the order is free
    Best b{-INFINITY, INT_MAX};
    if (lane < kArgmaxCluster) b = *cluster.map_shared_rank(&cta_best, lane);
#pragma unroll
    for (int o = kArgmaxCluster / 2; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, b.v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, b.idx, o);
      if (better(ov, oi, b.v, b.idx)) b = {ov, oi};
    }
    if (lane == 0) out_ids[row] = b.idx == INT_MAX ? 0 : b.idx;
  }
  cluster.sync();  // keep every CTA's shared memory alive until the leader has read it
}

}  // namespace b200asr

using namespace b200asr;

extern "C" int b200asr_greedy_argmax(const void *logits, int64_t row_stride, int32_t batch,
                                     int32_t vocab, int64_t *out_ids, b200asr_stream_t stream) {
  B200_REQUIRE(batch >= 0 && vocab >= 1 && row_stride >= vocab,
               "greedy_argmax: bad sizes (batch %d, vocab %d, stride %lld)", batch, vocab,
               (long long)row_stride);
  if (batch == 0) return B200ASR_OK;
  B200_REQUIRE(batch <= 65535, "greedy_argmax: batch %d too large", batch);
  B200_REQUIRE(logits && out_ids, "greedy_argmax: null pointer");
  dim3 grid(kArgmaxCluster, batch);
  B200_LAUNCH_CHECK_ERR(launch_kernel(greedy_argmax_kernel, grid, dim3(kArgmaxThreads), 0,
                                      stream, true, 1, static_cast<const __nv_bfloat16 *>(logits),
                                      row_stride, vocab, out_ids),
                        "greedy_argmax");
  return B200ASR_OK;
}
