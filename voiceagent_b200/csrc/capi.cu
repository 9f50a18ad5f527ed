// C-ABI plumbing: error reporting, version, TMA tensor-map encoding.
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace b200asr {

static thread_local std::string g_last_error;
static std::atomic<int> g_pdl{0};

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

void set_error(const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_tmap_bf16(CUtensorMap *map, const void *base, int rank, const uint64_t *dims,
                    const uint64_t *strides_bytes, const uint32_t *box) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return false;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i > 0) st[i - 1] = strides_bytes[i - 1];
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void *>(base), d, st, bx,
                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for a rank-%d map", static_cast<int>(r), rank);
    return false;
  }
  return true;
}

bool make_tmap_3d_bf16(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                       uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                       uint32_t b2) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return false;
  }
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estrides[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides,
                  box, estrides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for dims {%llu,%llu,%llu} strides {%llu,%llu}",
              static_cast<int>(r), (unsigned long long)d0, (unsigned long long)d1,
              (unsigned long long)d2, (unsigned long long)stride1_bytes,
              (unsigned long long)stride2_bytes);
    return false;
  }
  return true;
}

}  // namespace b200asr

extern "C" int b200asr_version(void) { return 100; }

extern "C" void b200asr_set_pdl(int32_t enable) { b200asr::g_pdl.store(enable ? 1 : 0); }

extern "C" int32_t b200asr_pdl_enabled(void) { return b200asr::pdl_enabled() ? 1 : 0; }

extern "C" const char *b200asr_last_error(void) { return b200asr::g_last_error.c_str(); }
