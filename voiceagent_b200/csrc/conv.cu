// Encoder convolutional front on sm_100a: Conv2d(kernel 3, stride 2, padding 1) + bias +
// GELU, the three convolutions of the audio tower's downsampler (models/audio_encoder.py:
// 145-175: conv2d1 -> gelu -> conv2d2 -> gelu -> conv2d3 -> gelu over 100-frame chunks).
//
// Layout: activations channels-last, x [N][H][W][C_in] bf16; the output is written to
// y[n * sn + oy * sy + ox * sx + c] (channels contiguous), so conv3 can emit its pixels in
// the order conv_out reads them ([n][t = ox][f = oy][c]) without a transpose.
//
// Rounding follows the reference module by module: the convolution's output is bf16, the
// bias is added to it in fp32 and rounded again (cuDNN convolution, then the bias add),
// and GELU (erf form, torch.nn.functional.gelu's default) is evaluated in fp32 on that
// value and rounded.
//
//  * conv1 (C_in = 1): a direct stencil on CUDA cores -- 9 multiply-adds per output, far
//    too few for a tensor-core GEMM; each thread owns 8 output channels (their 72
//    weights in registers) of one pixel and writes them as one 16-byte store.
//  * conv2, conv3 (C_in = C_out = 480 for Qwen3-ASR): implicit GEMM on tcgen05, one
//    persistent CTA per SM. Output pixels of all chunks are flattened into one row space
//    and cut into tiles of 128 pixels x NT output channels; K runs over C_in in 64-channel
//    blocks x the 9 taps. The A operand (the 3x3 / stride-2 gather of the input) is built
//    by four warps with 16-byte cp.async copies, eight lanes per 128-byte input row --
//    zero-filled where the tap falls into the padding or past C_in -- straight into the
//    128-byte-swizzled K-major layout; each thread's copies arrive on the stage's full
//    barrier when they land (cp.async.mbarrier.arrive), so the gather never stalls on
//    its own copies. The weights arrive by TMA from a [C_out][9][C_pad] repacking; one
//    thread issues the MMAs into one of two TMEM accumulators while four epilogue warps
//    run bias + GELU on the other (the previous tile).
#include "common.cuh"

namespace b200asr {

// ------------------------------------------------------------------ epilogue math

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
}

// bf16 convolution output, bias added and rounded, GELU (the caller rounds the result)
__device__ __forceinline__ float conv_out_value(float acc, float bias) {
  const float y = __bfloat162float(__float2bfloat16_rn(acc));
  return gelu_erf(__bfloat162float(__float2bfloat16_rn(y + bias)));
}

// ------------------------------------------------------------- conv1: one channel

struct Conv1Args {
  const __nv_bfloat16 *x;  // [N][H][W] (one input channel)
  int n, h, w, ho, wo, c;
  const __nv_bfloat16 *wt;  // [C][9]
  const __nv_bfloat16 *bias;
  __nv_bfloat16 *y;
  int64_t sn, sy, sx;
};

__global__ void __launch_bounds__(256) conv1_gelu_kernel(const Conv1Args a) {
  const int groups = a.c / 8;
  const int per_pass = blockDim.x / groups;
  const int g = threadIdx.x % groups, slot = threadIdx.x / groups;
  if (slot >= per_pass) return;
  float wv[8][9], bv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    bv[i] = __bfloat162float(a.bias[8 * g + i]);
#pragma unroll
    for (int t = 0; t < 9; ++t) wv[i][t] = __bfloat162float(a.wt[(8 * g + i) * 9 + t]);
  }
  const int64_t per_image = static_cast<int64_t>(a.ho) * a.wo;
  const int64_t total = per_image * a.n;
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * per_pass + slot; p < total;
       p += static_cast<int64_t>(gridDim.x) * per_pass) {
    const int img = static_cast<int>(p / per_image);
    const int rem = static_cast<int>(p - static_cast<int64_t>(img) * per_image);
    const int oy = rem / a.wo, ox = rem - (rem / a.wo) * a.wo;
    const __nv_bfloat16 *src = a.x + static_cast<int64_t>(img) * a.h * a.w;
    float in[9];
#pragma unroll
    for (int ky = 0; ky < 3; ++ky)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const int iy = 2 * oy + ky - 1, ix = 2 * ox + kx - 1;
        in[ky * 3 + kx] = (iy >= 0 && iy < a.h && ix >= 0 && ix < a.w)
                              ? __bfloat162float(src[iy * a.w + ix]) : 0.f;
      }
    float out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int t = 0; t < 9; ++t) acc = fmaf(wv[i][t], in[t], acc);
      out[i] = conv_out_value(acc, bv[i]);
    }
    uint4 v;
    v.x = pack2(out[0], out[1]);
    v.y = pack2(out[2], out[3]);
    v.z = pack2(out[4], out[5]);
    v.w = pack2(out[6], out[7]);
    *reinterpret_cast<uint4 *>(a.y + img * a.sn + oy * a.sy + ox * a.sx + 8 * g) = v;
  }
}

// ------------------------------------------------- conv2/conv3: tcgen05 implicit GEMM

constexpr int kCvBK = 64;         // input channels per K block (one 128-byte swizzle row)
constexpr int kCvRows = 128;      // pixels per tile = MMA M = TMEM lanes
constexpr int kCvThreads = 320;   // warps 0-3 A gather, 4-7 epilogue, 8 weights (TMA), 9 MMA
constexpr int kCvSmemBudget = 200 * 1024;

template <int NT>
struct Cv {
  static constexpr int A_BYTES = kCvRows * 128;  // 16 KiB: 128 pixels x 64 channels
  static constexpr int B_BYTES = NT * 128;       // NT output channels x 64 channels
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = kCvSmemBudget / STAGE < 8 ? kCvSmemBudget / STAGE : 8;
  static constexpr int ACC_STRIDE = NT <= 128 ? 128 : 256;  // TMEM columns per accumulator
  static constexpr uint32_t TMEM_COLS = 2 * ACC_STRIDE;      // two accumulators
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(STAGES) * STAGE + 256;
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "MMA N");
  static_assert(STAGE % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
  static_assert(STAGES >= 3, "pipeline depth");
  static_assert(2 * STAGES * 8 + 2 * 2 * 8 + 4 <= 256, "barriers fit their slot");
};

struct ConvArgs {
  const __nv_bfloat16 *x;  // [N][H][W][C_in]
  int n, h, w, ci, cblocks, ho, wo, co;
  int64_t pixels;          // N * ho * wo
  const __nv_bfloat16 *bias;
  __nv_bfloat16 *y;
  int64_t sn, sy, sx;
  int32_t *error_flag;
};

__device__ __forceinline__ void cp_async16_zfill(uint32_t saddr, const void *gptr, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(gptr), "r"(bytes)
               : "memory");
}
// Arrive on `bar` once all of this thread's earlier cp.async copies have landed; the
// arrival is part of the barrier's initial count (.noinc).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t c0,
                                            int32_t c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// Warp-collective TMEM load of 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// `count` (16 or 32) outputs of one pixel row: bias, GELU, bf16, 16-byte stores.
template <int COUNT>
__device__ __forceinline__ void conv_store(const float *acc, const __nv_bfloat16 *bias,
                                           __nv_bfloat16 *dst) {
#pragma unroll
  for (int i = 0; i < COUNT / 8; ++i) {
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = conv_out_value(acc[8 * i + j], __bfloat162float(bias[8 * i + j]));
    uint4 v;
    v.x = pack2(o[0], o[1]);
    v.y = pack2(o[2], o[3]);
    v.z = pack2(o[4], o[5]);
    v.w = pack2(o[6], o[7]);
    *reinterpret_cast<uint4 *>(dst + 8 * i) = v;
  }
}

// Persistent: one CTA per SM walks tiles t = blockIdx.x, + gridDim.x, ...; tile t is
// pixel tile t / ntiles (128 pixels) x output-channel tile t % ntiles (NT channels), so
// the channel tiles of one pixel tile run side by side and share the gathered input in
// L2. K runs channel-block-major (64 channels, then the 9 taps), which keeps the input
// rows of the SM-wide working set (~70 KB per tile) in L2 across the taps. Two TMEM
// accumulators: the epilogue warps drain tile i while the MMA warp accumulates tile i + 1.
template <int NT>
__global__ void __launch_bounds__(kCvThreads, 1)
    conv_gemm_gelu_kernel(const __grid_constant__ CUtensorMap tm_w, const ConvArgs a) {
  using C = Cv<NT>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * C::STAGE);
  uint64_t *empty = full + S;
  uint64_t *acc_full = empty + S;   // [2] accumulator b holds a finished tile
  uint64_t *acc_empty = acc_full + 2;  // [2] accumulator b drained by the epilogue
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kblocks = 9 * a.cblocks;
  const int ntiles = a.co / NT;
  const int64_t ptiles = (a.pixels + kCvRows - 1) / kCvRows;
  const int64_t tiles = ptiles * ntiles;
  const int64_t per_image = static_cast<int64_t>(a.ho) * a.wo;

  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], kCvRows + 1);  // 128 gather threads + the weights' TMA
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kCvRows);
    }
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) prefetch_tmap(&tm_w);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // -------------------------------------------------------- A operand (im2col gather)
    // Eight lanes per 128-byte input row (lane & 7 = 16-byte chunk), four rows per warp
    // instruction, so each copy instruction covers four whole lines. Thread (warp, lane)
    // gathers tile rows warp * 32 + (lane >> 3) + 4 i, i < 8; its copies arrive on the
    // stage's full barrier when they land, so it never waits for its own copies.
    const int chunk = lane & 7;
    uint32_t g = 0;  // K blocks issued so far (stage ring position)
    bool ok = true;
    for (int64_t t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
      const int64_t p0 = (t / ntiles) * kCvRows;
      int pix[8], iy0[8], ix0[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t p = p0 + warp * 32 + (lane >> 3) + 4 * i;
        if (p < a.pixels) {
          const int im = static_cast<int>(p / per_image);
          const int rem = static_cast<int>(p - im * per_image);
          const int oy = rem / a.wo;
          pix[i] = im * a.h * a.w;
          iy0[i] = 2 * oy - 1;
          ix0[i] = 2 * (rem - oy * a.wo) - 1;
        } else {  // past the last pixel: every tap reads as padding
          pix[i] = 0;
          iy0[i] = -(1 << 20);
          ix0[i] = 0;
        }
      }
      for (int cb = 0; cb < a.cblocks; ++cb) {
        const int c0 = cb * kCvBK;
        const bool have_c = c0 + 8 * chunk < a.ci;
        const __nv_bfloat16 *xc = a.x + c0 + 8 * chunk;
        for (int tap = 0; tap < 9; ++tap, ++g) {
          const int st = static_cast<int>(g % S);
          if (!mbar_wait(&empty[st], ((g / S) & 1) ^ 1, a.error_flag, &abort_flag)) {
            ok = false;
            break;
          }
          const int ky = tap / 3, kx = tap - ky * 3;
          const uint32_t stage_a = smem_addr(smem + st * C::STAGE);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = warp * 32 + (lane >> 3) + 4 * i;
            const int iy = iy0[i] + ky, ix = ix0[i] + kx;
            const bool in = have_c && static_cast<unsigned>(iy) < static_cast<unsigned>(a.h) &&
                            static_cast<unsigned>(ix) < static_cast<unsigned>(a.w);
            const __nv_bfloat16 *src =
                in ? xc + static_cast<int64_t>(pix[i] + iy * a.w + ix) * a.ci : a.x;
            cp_async16_zfill(stage_a + (r >> 3) * 1024 + (r & 7) * 128 + ((chunk ^ (r & 7)) << 4),
                             src, in ? 16u : 0u);
          }
          cp_async_mbar_arrive_noinc(&full[st]);
        }
        if (!ok) break;
      }
    }
    cp_async_wait<0>();  // nothing of this thread's is in flight past this point
  } else if (warp < 8) {
    // ------------------------------------------------------------ bias + GELU epilogue
    // Warp w reads TMEM lanes 32 (w - 4) .. + 31: thread = tile row (pixel).
    const int r = (warp - 4) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp - 4) * 32) << 16;
    uint32_t i = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int b = static_cast<int>(i & 1);
      if (!mbar_wait(&acc_full[b], (i >> 1) & 1, a.error_flag, &abort_flag)) break;
      tc_fence_after();
      const int64_t p = (t / ntiles) * kCvRows + r;
      const int n0 = static_cast<int>(t % ntiles) * NT;
      const bool live = p < a.pixels;
      const int64_t pp = live ? p : 0;
      const int im = static_cast<int>(pp / per_image);
      const int rem = static_cast<int>(pp - im * per_image);
      const int oy = rem / a.wo, ox = rem - oy * a.wo;
      __nv_bfloat16 *dst = a.y + im * a.sn + oy * a.sy + ox * a.sx + n0;
      const uint32_t acc = tmem + lane_off + b * C::ACC_STRIDE;
#pragma unroll 1
      for (int col = 0; col + 32 <= NT; col += 32) {
        float v[32];
        tmem_ld32(acc + col, v);
        tmem_wait_ld();
        if (live) conv_store<32>(v, a.bias + n0 + col, dst + col);
      }
      if (NT % 32) {
        float v[16];
        tmem_ld16(acc + (NT - 16), v);
        tmem_wait_ld();
        if (live) conv_store<16>(v, a.bias + n0 + NT - 16, dst + NT - 16);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ weights (TMA)
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int n0 = static_cast<int>(t % ntiles) * NT;
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int st = static_cast<int>(g % S);
          if (!mbar_wait(&empty[st], ((g / S) & 1) ^ 1, a.error_flag, &abort_flag)) {
            ok = false;
            break;
          }
          const int cb = kb / 9, tap = kb - cb * 9;
          mbar_arrive_expect_tx(&full[st], C::B_BYTES);
          tma_load_2d(smem + st * C::STAGE + C::A_BYTES, &tm_w, tap * a.cblocks * kCvBK + cb * kCvBK,
                      n0, &full[st]);
        }
      }
      // after an abort: let the weight tiles already requested land before the CTA exits
      if (!ok)
        for (uint32_t k = g > static_cast<uint32_t>(S) ? g - S : 0; k < g; ++k)
          mbar_drain(&full[k % S], (k / S) & 1);
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kCvRows, NT, false, false);
      const uint32_t base = smem_addr(smem);
      uint32_t g = 0, i = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++i) {
        const int b = static_cast<int>(i & 1);
        if (!mbar_wait(&acc_empty[b], ((i >> 1) & 1) ^ 1, a.error_flag, &abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * C::ACC_STRIDE;
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int st = static_cast<int>(g % S);
          if (!mbar_wait(&full[st], (g / S) & 1, a.error_flag, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fence_proxy_async_smem();  // the A bytes came from cp.async (generic proxy)
          const uint32_t sa = base + st * C::STAGE, sb = sa + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < kCvBK / 16; ++k)
            umma_f16_ss(d, smem_desc_sw128(sa + k * 32, 16, 1024),
                        smem_desc_sw128(sb + k * 32, 16, 1024), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&acc_full[b]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Repack conv weights [C_out][C_in][3][3] into [C_out][9][C_pad] (C_pad = 64 * ceil(C_in /
// 64), zero past C_in): row n, column tap * C_pad + c of the GEMM's K-major B operand.
__global__ void conv_pack_weight_kernel(const __nv_bfloat16 *w, int co, int ci, int cpad,
                                        __nv_bfloat16 *packed) {
  const int64_t total = static_cast<int64_t>(co) * 9 * cpad;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % cpad);
    const int tap = static_cast<int>((i / cpad) % 9);
    const int n = static_cast<int>(i / (9 * static_cast<int64_t>(cpad)));
    packed[i] = c < ci ? w[(static_cast<int64_t>(n) * ci + c) * 9 + tap] : __float2bfloat16_rn(0.f);
  }
}

template <int NT>
int launch_conv_gemm(const ConvArgs &a, const void *packed, int co, int cpad, cudaStream_t stream) {
  using C = Cv<NT>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(conv_gemm_gelu_kernel<NT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(C::SMEM));
    if (e != cudaSuccess) {
      set_error("conv3x3s2_gelu: cannot reserve %zu bytes of shared memory: %s", C::SMEM,
                cudaGetErrorString(e));
      return B200ASR_ERR_CUDA;
    }
    configured = true;
  }
  CUtensorMap tw;
  const uint64_t dims[2] = {static_cast<uint64_t>(9) * cpad, static_cast<uint64_t>(co)};
  const uint64_t strides[1] = {static_cast<uint64_t>(9) * cpad * 2};
  const uint32_t box[2] = {kCvBK, NT};
  if (!make_tmap_bf16(&tw, packed, 2, dims, strides, box)) return B200ASR_ERR_CUDA;
  const int64_t tiles = (a.pixels + kCvRows - 1) / kCvRows * (co / NT);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms()));
  conv_gemm_gelu_kernel<NT><<<grid, kCvThreads, C::SMEM, stream>>>(tw, a);
  B200_CUDA_LAUNCH_CHECK("conv3x3s2_gelu");
  return B200ASR_OK;
}

}  // namespace b200asr

using namespace b200asr;

extern "C" size_t b200asr_conv_weight_bytes(int32_t c_out, int32_t c_in) {
  if (c_out <= 0 || c_in <= 0) return 0;
  if (c_in == 1) return static_cast<size_t>(c_out) * 9 * 2;
  const size_t cpad = static_cast<size_t>((c_in + kCvBK - 1) / kCvBK) * kCvBK;
  return static_cast<size_t>(c_out) * 9 * cpad * 2;
}

extern "C" int b200asr_conv_pack_weight(const void *weight, int32_t c_out, int32_t c_in,
                                        void *packed, b200asr_stream_t stream) {
  B200_REQUIRE(c_out > 0 && c_in > 0 && weight && packed, "conv_pack_weight: bad arguments");
  B200_REQUIRE(aligned16(packed), "conv_pack_weight: packed buffer must be 16-byte aligned");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (c_in == 1) {  // the direct kernel reads [C_out][9] as given
    cudaError_t e = cudaMemcpyAsync(packed, weight, static_cast<size_t>(c_out) * 9 * 2,
                                    cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) {
      set_error("conv_pack_weight: copy failed: %s", cudaGetErrorString(e));
      return B200ASR_ERR_CUDA;
    }
    return B200ASR_OK;
  }
  const int cpad = (c_in + kCvBK - 1) / kCvBK * kCvBK;
  conv_pack_weight_kernel<<<std::min<int64_t>(1024, (static_cast<int64_t>(c_out) * 9 * cpad + 255) / 256),
                            256, 0, s>>>(static_cast<const __nv_bfloat16 *>(weight), c_out, c_in,
                                         cpad, static_cast<__nv_bfloat16 *>(packed));
  B200_CUDA_LAUNCH_CHECK("conv_pack_weight");
  return B200ASR_OK;
}

extern "C" int b200asr_conv3x3s2_gelu(const void *x, int32_t n, int32_t h, int32_t w, int32_t c_in,
                                      const void *packed_weight, const void *bias, int32_t c_out,
                                      void *y, int64_t y_stride_n, int64_t y_stride_y,
                                      int64_t y_stride_x, int32_t *error_flag,
                                      b200asr_stream_t stream) {
  B200_REQUIRE(n >= 0 && h >= 1 && w >= 1 && c_in >= 1 && c_out >= 1,
               "conv3x3s2_gelu: bad sizes");
  if (n == 0) return B200ASR_OK;
  B200_REQUIRE(x && packed_weight && bias && y, "conv3x3s2_gelu: null pointer");
  B200_REQUIRE(c_out % 8 == 0 && aligned16(y) && y_stride_n % 8 == 0 && y_stride_y % 8 == 0 &&
                   y_stride_x % 8 == 0,
               "conv3x3s2_gelu: output channels and strides must keep 16-byte alignment");
  const int ho = (h - 1) / 2 + 1, wo = (w - 1) / 2 + 1;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (c_in == 1) {
    B200_REQUIRE(c_out <= 2048, "conv3x3s2_gelu: at most 2048 output channels for one input channel");
    Conv1Args a{};
    a.x = static_cast<const __nv_bfloat16 *>(x);
    a.n = n;
    a.h = h;
    a.w = w;
    a.ho = ho;
    a.wo = wo;
    a.c = c_out;
    a.wt = static_cast<const __nv_bfloat16 *>(packed_weight);
    a.bias = static_cast<const __nv_bfloat16 *>(bias);
    a.y = static_cast<__nv_bfloat16 *>(y);
    a.sn = y_stride_n;
    a.sy = y_stride_y;
    a.sx = y_stride_x;
    const int groups = c_out / 8;
    const int per_pass = std::max(1, 256 / groups);
    const int threads = groups * per_pass;
    const int64_t pixels = static_cast<int64_t>(n) * ho * wo;
    const int64_t blocks = std::min<int64_t>((pixels + per_pass - 1) / per_pass, 16LL * num_sms());
    conv1_gelu_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(a);
    B200_CUDA_LAUNCH_CHECK("conv3x3s2_gelu (one input channel)");
    return B200ASR_OK;
  }
  B200_REQUIRE(c_in % 8 == 0 && aligned16(x) && aligned16(packed_weight),
               "conv3x3s2_gelu: input channels must be a multiple of 8 and tensors 16-byte aligned");
  B200_REQUIRE(static_cast<int64_t>(n) * h * w < (int64_t{1} << 31),
               "conv3x3s2_gelu: at most 2^31 - 1 input pixels per call");
  ConvArgs a{};
  a.x = static_cast<const __nv_bfloat16 *>(x);
  a.n = n;
  a.h = h;
  a.w = w;
  a.ci = c_in;
  a.co = c_out;
  a.cblocks = (c_in + kCvBK - 1) / kCvBK;
  a.ho = ho;
  a.wo = wo;
  a.pixels = static_cast<int64_t>(n) * ho * wo;
  a.bias = static_cast<const __nv_bfloat16 *>(bias);
  a.y = static_cast<__nv_bfloat16 *>(y);
  a.sn = y_stride_n;
  a.sy = y_stride_y;
  a.sx = y_stride_x;
  a.error_flag = error_flag;
  const int cpad = a.cblocks * kCvBK;
  if (c_out % 240 == 0) return launch_conv_gemm<240>(a, packed_weight, c_out, cpad, s);
  if (c_out % 128 == 0) return launch_conv_gemm<128>(a, packed_weight, c_out, cpad, s);
  if (c_out % 32 == 0) return launch_conv_gemm<32>(a, packed_weight, c_out, cpad, s);
  set_error("conv3x3s2_gelu: %d output channels unsupported (needs a multiple of 32)", c_out);
  return B200ASR_ERR_UNSUPPORTED;
}
