// Shared helpers for the b200asr kernels: bf16 math, warp reductions, host-side
// error reporting, and thin inline-PTX wrappers for the sm_100a features the
// attention kernels use (mbarrier, bulk / tensor TMA copies, tcgen05 + TMEM).
//
// Every wait on an mbarrier is bounded by a wall-clock limit (kWaitLimitNs). On
// expiry the waiting thread records B200ASR_DEVERR_TIMEOUT in the kernel's error
// word and the kernel winds down instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/b200asr.h"

#define B200ASR_DEVERR_TIMEOUT 16

namespace b200asr {

// ----------------------------------------------------------------- host errors

void set_error(const char *fmt, ...);  // defined in capi.cu (thread-local message)

#define B200_REQUIRE(cond, ...)      \
  do {                               \
    if (!(cond)) {                   \
      ::b200asr::set_error(__VA_ARGS__); \
      return B200ASR_ERR_INVALID;    \
    }                                \
  } while (0)

#define B200_CUDA_LAUNCH_CHECK(what)                                            \
  do {                                                                          \
    cudaError_t err__ = cudaGetLastError();                                     \
    if (err__ != cudaSuccess) {                                                 \
      ::b200asr::set_error("%s: launch failed: %s", what, cudaGetErrorString(err__)); \
      return B200ASR_ERR_CUDA;                                                  \
    }                                                                           \
  } while (0)

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------- programmatic dependent launch
// With PDL on (b200asr_set_pdl), the decode-path kernels are launched with the
// programmatic-stream-serialization attribute: a kernel may start while its predecessor
// in the stream is still running. Each such kernel calls pdl_trigger() first (letting its
// own successor launch early) and pdl_wait() in every thread before it reads data that
// an earlier kernel produced or writes global memory; before that it only sets up shared
// memory, tensor maps, TMEM and loads of static data (weights). Without the attribute
// both instructions are no-ops.
bool pdl_enabled();  // defined in capi.cu
int num_sms();       // SMs of the current device (defined in paged_decode.cu)

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, bool pdl, unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl && pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

#define B200_LAUNCH_CHECK_ERR(err, what)                                             \
  do {                                                                             \
    cudaError_t e__ = (err);                                                       \
    if (e__ != cudaSuccess) {                                                      \
      ::b200asr::set_error("%s: launch failed: %s", what, cudaGetErrorString(e__)); \
      return B200ASR_ERR_CUDA;                                                     \
    }                                                                              \
  } while (0)

// ------------------------------------------------------------------ device math

__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

// Unpack 8 bf16 values held in a uint4 into floats.
__device__ __forceinline__ void unpack8(const uint4 &v, float *out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

// The two bf16 halves of a packed pair as floats (low element first).
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// bf16(a), bf16(b) as floats: one paired conversion instead of two.
__device__ __forceinline__ float2 round2_bf16(float a, float b) { return unpack2(pack2(a, b)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void raise_flag(int32_t *flag, int32_t bit) {
  if (flag != nullptr) atomicOr(flag, bit);
}

// -------------------------------------------------------------- shared memory

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate wait

// ------------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete; false (and flag raised) on timeout.
// `abort` is a CTA-shared word: once any thread times out, the others stop waiting.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int32_t *err,
                                          volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (globaltimer_ns() - start > kWaitLimitNs) {
      if (abort != nullptr) *abort = 1;
      raise_flag(err, B200ASR_DEVERR_TIMEOUT);
      return false;
    }
  }
}

// After a timed-out wait: give the copies this CTA already issued on `bar` (phase
// `parity`) up to kDrainLimitNs to land before the CTA exits, so no copy writes into the
// shared memory of a CTA that is later placed on the same SM. No abort check: the CTA
// has already given up; this only bounds its exit.
constexpr uint64_t kDrainLimitNs = 200000000ull;  // 0.2 s
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t start = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - start > kDrainLimitNs) return;
  }
}

// ------------------------------------------------------------------------- TMA

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 3-D tiled tensor load (no multicast) into shared memory.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int32_t c0,
                                            int32_t c1, int32_t c2, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (TMA/UMMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------- tcgen05/TMEM

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accum).
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

// Warp-collective TMEM load: 32 lanes x 32 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format) for a tile stored
// with the 128-byte swizzle: 8-row x 128-byte atoms, atom base 1024-byte aligned.
//   K-major operand : lbo ignored (16), sbo = byte stride between 8-row groups.
//   MN-major operand: lbo = byte stride between 64-element MN groups,
//                     sbo = byte stride between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3fffu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3fffu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16 with bf16 A/B, fp32 accumulator, dense.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n, bool a_mn_major,
                                                       bool b_mn_major) {
  return (1u << 4)                       // D format: f32
         | (1u << 7)                     // A format: bf16
         | (1u << 10)                    // B format: bf16
         | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

}  // namespace b200asr

// Host: resolve cuTensorMapEncodeTiled through the runtime (no -lcuda needed).
namespace b200asr {
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
// Tiled bf16 tensor map (128-byte swizzle, no interleave, zero OOB fill) of rank <= 5:
// dims[0] is contiguous; strides_bytes[i] is the byte stride of dims[i + 1] (any order).
bool make_tmap_bf16(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
                    const uint64_t *strides_bytes, const uint32_t *box);
EncodeTiledFn encode_tiled_fn();  // defined in capi.cu

// The TTS pool decode's bf16 / head_dim 128 / 16-token-page case on the stream-K decode
// kernel (paged_decode.cu). *taken is false (and nothing is launched) when the call does
// not fit it; b200asr_pool_paged_decode then runs its own kernel.
struct PoolStreamK {
  int batch, num_heads, num_kv_heads, head_dim;
  const void *query;
  int64_t q_stride_b, q_stride_h;
  void *key_pool, *value_pool;
  int num_pages, page_size;
  int64_t kv_stride_p, kv_stride_h, kv_stride_s;
  const int64_t *page_table;
  int64_t table_stride;
  int table_width;
  const int64_t *seq_lens;
  const uint8_t *valid;
  int64_t valid_stride;
  int valid_len;
  const void *new_key, *new_value;
  int64_t new_stride_b, new_stride_h;
  void *out;
  int64_t out_stride_b, out_stride_h;
  int max_seq_len;
  float scale;
  void *workspace;
  size_t workspace_bytes, workspace_head;  // head: bytes of counters the pool kernel keeps
  int32_t *error_flag;
  void *stream;
};
int pool_decode_stream_k(const PoolStreamK &p, bool *taken);

// 3-D bf16 tensor map: dims {d0 (contiguous), d1, d2}, strides in bytes for d1, d2,
// box {b0, b1, b2}, 128-byte swizzle. Returns false (error set) on failure.
bool make_tmap_3d_bf16(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1,
                       uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0,
                       uint32_t b1, uint32_t b2);
}  // namespace b200asr
