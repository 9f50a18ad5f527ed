// Split-K paged decode attention (one query token per sequence).
//
// Replaces the decode use of flash_attn_varlen_func over the paged cache inside the
// CUDA-graph decode (layers/attention.py:96-107 with max_seqlen_q = 1, fed by
// engine/graph_runner.py:81-94): out[b, h] = softmax(q[b, h] K_b^T * scale) V_b with
// K_b, V_b the first len_b rows of sequence b gathered through its block table, and
// query head h reading KV head h / (H / H_kv).
//
// Design (HBM-bound; every KV row is read exactly once, for all query heads of its group):
//  * Stream-K split: the persistent grid (one CTA per SM) divides the batch's key tokens
//    -- all sequences laid end to end -- into equal contiguous ranges, so every CTA
//    streams the same number of bytes whatever the length mix. A range is cut into
//    segments at sequence ends and into stages of <= 16 tokens at KV-block ends.
//  * Producer warp: keeps a 3-deep ring of stages and publishes each stage's sequence,
//    token count and segment flags in shared memory. A stage is 2 x H_kv x 2
//    TMA boxes {64 dims, 1 head, 16 tokens} with the 128-byte swizzle (K and V, every
//    KV head, both halves of the head dim) -- one box per producer lane -- plus, on an
//    segment's first stage, a 1-D bulk copy of that sequence's query row.
//  * One consumer warp per KV head. Scores S = Q K^T and the update O += P V run on
//    mma.sync m16n8k16 (bf16 in, fp32 accumulate) with the group's query heads as the
//    MMA rows: a single-token GQA group has G (= 2) query rows, far below the 64-row
//    minimum of tcgen05, and the tensor-core fragments remove the shuffle reductions that
//    dominated a CUDA-core version. P is reused from the score registers as the A
//    operand (no shared-memory round trip); softmax statistics are fp32, base 2, and
//    need only a quad (4-lane) reduction per row.
//  * A segment covering a whole sequence writes bf16 output directly. A sequence split
//    across CTAs leaves one unnormalised fp32 partial plus (max, sum) per CTA in the
//    workspace; the CTA that publishes the last one (per-sequence counter in the
//    workspace header, reset by that CTA) merges them -- no second kernel.
#include <mutex>

#include "common.cuh"

namespace b200asr {

constexpr int kDecD = 128;
constexpr int kDecMaxGrid = 256;  // CTAs of the persistent grid (<= one per SM)
constexpr int kDecStage = 16;
constexpr int kDecStages = 3;
constexpr int kDecMaxBatch = 1024;
constexpr size_t kDecHeaderBytes = 4096;  // per-sequence merge counters (int32 x 1024)
constexpr int kDecBtCache = 1024;  // block-table entries kept in shared memory (B * bt_stride)
constexpr float kLog2e = 1.4426950408889634f;

template <int HKV, int G>
struct Dec {
  static constexpr int H = HKV * G;
  static constexpr int CONSUMERS = HKV * 32;           // one consumer warp per KV head
  static constexpr int THREADS = CONSUMERS + 32;       // + 1 producer warp
  static constexpr int HEAD_TILE = kDecStage * kDecD * 2;  // 16 tokens x 128 dims: 4 KiB
  static constexpr int KV_BYTES = HKV * HEAD_TILE;
  static constexpr int Q_BYTES = ((H * kDecD * 2 + 1023) / 1024) * 1024;
  static constexpr int STAGE_BYTES = 2 * KV_BYTES + Q_BYTES;
  static constexpr uint32_t TX_KV = 2 * KV_BYTES;
  static constexpr uint32_t TX_Q = H * kDecD * 2;
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(kDecStages) * STAGE_BYTES +
                                 4 * (kDecMaxBatch + 1) * 4 + kDecBtCache * 4 +
                                 2 * kDecStages * 8 + kDecStages * 32 + 64;
  static_assert(SMEM <= 232448, "dynamic shared memory above the 227 KB per-CTA limit");
  static_assert(G >= 1 && G <= 8, "group size");
  static_assert(HKV <= 8, "a stage box holds at most 8 KV heads");
};

struct DecodeArgs {
  const __nv_bfloat16 *q;
  int64_t q_stride;
  int num_blocks;
  int block_size;
  const int32_t *cu_seqlens_k;
  const int32_t *block_tables;
  int bt_stride;
  int batch;
  float scale_log2;
  __nv_bfloat16 *out;
  int64_t out_stride;
  int *counters;  // [kDecMaxBatch], zero between calls
  float *ws_ml;   // [parts_cap][H][2]
  float *ws_o;    // [parts_cap][H][128]
  int parts_cap;
  int32_t *error_flag;
  int early;  // launched with programmatic dependent launch: request stages before the wait
  // Page-pool layout (the TTS talker's [pages, kv_heads, 16, 128] pool; POOL kernels only):
  // lengths, page table and key-valid mask as b200asr_pool_paged_decode takes them, and
  // the current token's K/V, stored at position seq_len - 1 before its stage is loaded.
  const int64_t *seq_lens;
  int max_seq_len;
  const int64_t *page_table;
  int64_t table_stride;
  int table_width;
  const uint8_t *valid;
  int64_t valid_stride;
  int valid_len;
  const __nv_bfloat16 *nk, *nv;
  int64_t n_sb, n_sh;
  __nv_bfloat16 *kp, *vp;
  int64_t sp, sh, ss;  // pool element strides: page, head, position
};

// What the producer tells the consumers about a stage (written before the stage's
// mbarrier arrive, read after the matching wait).
struct StageInfo {
  int b;      // sequence, or -1 for the terminal stage
  int ntok;   // tokens of the sequence in the stage (1..16)
  int flags;  // 1: first stage of a segment (q attached), 2: last stage, 4: whole sequence
  int vbits;  // POOL: bit t set when token t is attended (in range, page valid, mask set)
  // POOL, the row's last stage with a current token: the stage row that holds it (-1:
  // none, or not attended) and its element offset in the pools (-1: page unusable)
  int new_row;
  int64_t new_off;
};

__device__ __forceinline__ void consumer_sync(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// Spin until the shared word *seq equals `want` (bounded like mbar_wait: false and the
// timeout bit raised after kWaitLimitNs, or at once when the CTA already aborted).
__device__ __forceinline__ bool slot_wait(volatile int *seq, int want, int32_t *err,
                                          volatile int *abort) {
  if (*seq == want) return true;
  const uint64_t start = globaltimer_ns();
  while (*seq != want) {
    if (*abort) return false;
    if (globaltimer_ns() - start > kWaitLimitNs) {
      *abort = 1;
      raise_flag(err, B200ASR_DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Largest b in [0, n) with v[b] <= x (v non-decreasing, v[0] <= x).
__device__ __forceinline__ int upper_index(const int *v, int n, int x) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (v[mid] <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                          uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16 bf16, rows) * B(16x8 bf16, cols) + D, fp32 accumulate.
__device__ __forceinline__ void mma16816(float *d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same MMA as a plain (reorderable) asm: a pure register operation.
__device__ __forceinline__ void mma16816_nv(float *d, uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose of an 8x8 bf16 matrix held one fragment register per lane.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled tile (1024-aligned).
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Stream-K partition: CTA c of g owns global key tokens [T*c/g, T*(c+1)/g).
__device__ __forceinline__ int part_begin(int64_t total, int c, int g) {
  return static_cast<int>(total * c / g);
}
// The CTA whose range contains global token x.
__device__ __forceinline__ int owner_cta(int64_t total, int x, int g) {
  const int64_t c = ((static_cast<int64_t>(x) + 1) * g - 1) / total;
  return static_cast<int>(c < g - 1 ? c : g - 1);
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// 4-D tiled tensor load (no multicast) into shared memory.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int32_t c0,
                                            int32_t c1, int32_t c2, int32_t c3, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_addr(bar))
      : "memory");
}

// 5-D tiled tensor load (no multicast) into shared memory.
__device__ __forceinline__ void tma_load_5d(void *dst, const CUtensorMap *map, int32_t c0,
                                            int32_t c1, int32_t c2, int32_t c3, int32_t c4,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_addr(bar))
      : "memory");
}

// The same box, into L2 only (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_4d(const CUtensorMap *map, int32_t c0, int32_t c1,
                                                int32_t c2, int32_t c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// Merge the n_parts split-K partials of sequence b (workspace slots first..first+n_parts-1)
// for the G query heads of KV head w (one warp each). Runs after this CTA's last stage,
// when the stage buffers are free: all consumer threads stage a chunk of partials --
// (max, sum) rows and fp32 accumulators, contiguous in the workspace -- with 16-byte
// cp.async.cg (L2, never a stale L1 line: other SMs wrote them), so a chunk costs one L2
// round trip. Lane l owns dims 4l..4l+3 of every head; the online rescale carries
// across chunks, so any number of partials merges.
template <class C, bool POOL>
__device__ __forceinline__ void merge_staged(const DecodeArgs &a, uint8_t *buf, int first,
                                             int n_parts, int b, int w, int lane, int tid) {
  constexpr int H = C::H;
  constexpr int NT = C::CONSUMERS;
  constexpr int G = H / (NT / 32);
  constexpr int PART_BYTES = H * (kDecD + 2) * 4;
  constexpr int CAP = kDecStages * C::STAGE_BYTES / PART_BYTES;
  const uint32_t sbuf = smem_addr(buf);
  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
    acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
  }
  for (int c0 = 0; c0 < n_parts; c0 += CAP) {
    const int n = min(CAP, n_parts - c0);
    const int ml_bytes = n * H * 8, o_bytes = n * H * kDecD * 4;
    const uint8_t *gml = reinterpret_cast<const uint8_t *>(a.ws_ml + static_cast<int64_t>(first + c0) * H * 2);
    const uint8_t *go = reinterpret_cast<const uint8_t *>(a.ws_o + static_cast<int64_t>(first + c0) * H * kDecD);
    for (int i = tid * 16; i < ml_bytes; i += NT * 16) cp_async16(sbuf + i, gml + i);
    for (int i = tid * 16; i < o_bytes; i += NT * 16) cp_async16(sbuf + ml_bytes + i, go + i);
    cp_async_wait_all();
    consumer_sync(NT);
    const float2 *sml = reinterpret_cast<const float2 *>(buf);
    const float4 *so = reinterpret_cast<const float4 *>(buf + ml_bytes);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int hh = w * G + g;
      float cm = -INFINITY;
      for (int i = lane; i < n; i += 32) cm = fmaxf(cm, sml[i * H + hh].x);
      const float mn = fmaxf(m[g], warp_max(cm));
      // POOL: a partial with every key masked has m = -inf (and l = 0, O = 0)
      const float mu = POOL && mn == -INFINITY ? 0.f : mn;
      const float sc = exp2f(m[g] - mu);
      l[g] *= sc;
      acc[g][0] *= sc;
      acc[g][1] *= sc;
      acc[g][2] *= sc;
      acc[g][3] *= sc;
      for (int i = 0; i < n; ++i) {
        const float2 st = sml[i * H + hh];
        const float wgt = exp2f(st.x - mu);
        const float4 v = so[(i * H + hh) * (kDecD / 4) + lane];
        l[g] += st.y * wgt;
        acc[g][0] += v.x * wgt;
        acc[g][1] += v.y * wgt;
        acc[g][2] += v.z * wgt;
        acc[g][3] += v.w * wgt;
      }
      m[g] = mn;
    }
    consumer_sync(NT);  // the next chunk (or merge) overwrites the buffer
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float inv = POOL && l[g] == 0.f ? 0.f : 1.f / l[g];  // no attended key: zeros
    __nv_bfloat16 *dst = a.out + b * a.out_stride + (w * G + g) * kDecD + lane * 4;
    *reinterpret_cast<uint2 *>(dst) = make_uint2(pack2(acc[g][0] * inv, acc[g][1] * inv),
                                                 pack2(acc[g][2] * inv, acc[g][3] * inv));
  }
}

template <int HKV, int G, bool POOL = false>
__global__ void __launch_bounds__(Dec<HKV, G>::THREADS, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const DecodeArgs a) {
  using C = Dec<HKV, G>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *stages = smem;
  int *s_cuk = reinterpret_cast<int *>(smem + kDecStages * C::STAGE_BYTES);  // [B + 1]
  int *s_sp = s_cuk + kDecMaxBatch + 1;      // [B + 1] first stage of each sequence
  int *s_parts = s_sp + kDecMaxBatch + 1;    // [B + 1] first partial slot of each sequence
  int *s_first = s_parts + kDecMaxBatch + 1;  // [B] first CTA of each sequence
  int *s_bt = s_first + kDecMaxBatch + 1;     // [B * bt_stride] block tables, when they fit
  uint64_t *full = reinterpret_cast<uint64_t *>(
      (reinterpret_cast<uintptr_t>(s_bt + kDecBtCache) + 7) & ~uintptr_t(7));
  uint64_t *empty = full + kDecStages;
  StageInfo *info = reinterpret_cast<StageInfo *>(empty + kDecStages);
  __shared__ int abort_flag;
  __shared__ int s_pending[2];  // sequences this CTA merges after its last stage
  __shared__ int s_npending;
  __shared__ int slot_last[kDecStages];  // stage number last issued into each ring slot

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = a.batch;

  pdl_trigger();
  if (tid == 0) {
    abort_flag = 0;
    s_npending = 0;
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HKV);
      slot_last[s] = -1;
    }
    fence_barrier_init();
  }
  if (warp == HKV && lane == 0) {
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  // The lengths, block tables and every cached row but each sequence's newest come from
  // launches that finished before the step's decoder kernels (the packer, earlier
  // steps): with programmatic dependent launch they are read, and the first ring of
  // stages requested, before the wait on the kernel that wrote q and the newest K/V.
  // Lengths and (when B * bt_stride entries fit) the block tables are loaded in the same
  // round trip -- every thread issues its loads before storing any -- so the first TMA
  // request waits for one global-memory latency instead of two.
  const int n_bt = POOL ? 0 : B * a.bt_stride;
  const bool bt_cached = !POOL && n_bt <= kDecBtCache;
  if constexpr (POOL) {
    // Row b attends positions < min(seq_lens[b], max_seq_len); s_cuk becomes the
    // exclusive prefix of those lengths (warp 0 scans after the loads).
    for (int i = tid; i < B; i += blockDim.x) {
      const int64_t sq = a.seq_lens[i];
      s_cuk[i + 1] = sq <= 0 ? 0 : static_cast<int>(sq < a.max_seq_len ? sq : a.max_seq_len);
      if (blockIdx.x == 0 && (sq <= 0 || sq > a.max_seq_len))
        raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);
    }
    __syncthreads();
    if (warp == 0) {
      int carry = 0;
      for (int b0 = 0; b0 < B; b0 += 32) {
        const int b = b0 + lane;
        const int v = b < B ? s_cuk[b + 1] : 0;
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        if (b < B) s_cuk[b + 1] = carry + incl;
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) s_cuk[0] = 0;
    }
  }
  for (int base = 0; !POOL && (base <= B || (bt_cached && base < n_bt)); base += 4 * blockDim.x) {
    int cu_v[4], bt_v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = base + k * blockDim.x + tid;
      cu_v[k] = i <= B ? a.cu_seqlens_k[i] : 0;
      bt_v[k] = bt_cached && i < n_bt ? a.block_tables[i] : 0;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = base + k * blockDim.x + tid;
      if (i <= B) s_cuk[i] = cu_v[k];
      if (bt_cached && i < n_bt) s_bt[i] = bt_v[k];
    }
  }
  __syncthreads();

  if (warp == HKV) {
    // ------------------------------------------------------------------ producer
    // Stage prefix: sequence b owns ceil(len_b / 16) stages, laid end to end. Published
    // to the consumers through named barrier 2 (arrive here, sync there).
    int carry = 0;
    for (int b0 = 0; b0 < B; b0 += 32) {
      const int b = b0 + lane;
      const int len = b < B ? s_cuk[b + 1] - s_cuk[b] : 0;
      const int ns = len > 0 ? (len + kDecStage - 1) / kDecStage : 0;
      int incl = ns;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (b < B) s_sp[b] = carry + incl - ns;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_sp[B] = carry;
    __syncwarp();
    asm volatile("bar.arrive 2, %0;" ::"r"(C::THREADS) : "memory");

    uint32_t it_stage = 0;
    auto acquire = [&](int &st) -> bool {
      st = it_stage % kDecStages;
      const uint32_t ph = (it_stage / kDecStages) & 1;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[st], ph ^ 1, a.error_flag, &abort_flag);
      if (ok && lane == 0) slot_last[st] = static_cast<int>(it_stage);
      return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    // After an abort, wait (bounded) for the copies of every slot's last stage to land
    // before the CTA exits.
    auto drain = [&]() {
      if (lane != 0 || !abort_flag) return;
      for (int s = 0; s < kDecStages; ++s)
        if (slot_last[s] >= 0) mbar_drain(&full[s], (slot_last[s] / kDecStages) & 1);
    };
    // Before the wait: stages up to the first one holding a sequence's newest token, at
    // most one ring (no acquire blocks). Their q copies are issued after the wait, on the
    // same stage barriers (which already count q's bytes).
    bool waited = a.early == 0;  // without PDL the wait returns at once: no early phase
    int n_early = 0, n_dq = 0;
    int dq_st[kDecStages], dq_b[kDecStages];
    auto wait_prev = [&]() {
      if (waited) return;
      pdl_wait();
      waited = true;
      if (lane == 2)
        for (int i = 0; i < n_dq; ++i)
          bulk_g2s(stages + dq_st[i] * C::STAGE_BYTES + 2 * C::KV_BYTES,
                   a.q + dq_b[i] * a.q_stride, C::TX_Q, &full[dq_st[i]]);
    };
    const int S = carry;
    const int geff = S < 1 ? 1 : (S < static_cast<int>(gridDim.x) ? S : static_cast<int>(gridDim.x));
    if (S > 0 && static_cast<int>(blockIdx.x) < geff) {
      const int c = blockIdx.x;
      const int j0 = part_begin(S, c, geff), j1 = part_begin(S, c + 1, geff);
      for (int wb = j0; wb < j1; wb += 32) {
        // Lane i describes stage wb + i: sequence, token count, flags and cache slot
        // (the block-table reads of 32 stages are in flight together).
        const int j = wb + lane;
        int d_b = 0, d_n = 0, d_fl = 0, d_slot = 0, d_end = 0, d_vb = 0, d_nrow = -1;
        int64_t d_noff = -1;
        if (j < j1) {
          const int b = upper_index(s_sp, B + 1, j);  // s_sp[b] <= j < s_sp[b + 1]
          const int len = s_cuk[b + 1] - s_cuk[b];
          const int t0 = (j - s_sp[b]) * kDecStage;
          d_n = min(kDecStage, len - t0);
          d_end = t0 + d_n == len;  // holds the sequence's newest token
          const bool first = t0 == 0 || j == j0, last = t0 + d_n == len || j == j1 - 1;
          const bool whole = s_sp[b] >= j0 && s_sp[b + 1] <= j1;
          d_b = b;
          d_fl = (first ? 1 : 0) | (last ? 2 : 0) | (whole ? 4 : 0);
          if constexpr (POOL) {
            // one stage = one 16-token page; an unusable page is loaded from page 0 with
            // none of its tokens attended
            const int col = t0 / kDecStage;
            int64_t page = -1;
            if (col < a.table_width) page = a.page_table[static_cast<int64_t>(b) * a.table_stride + col];
            const bool page_ok = page >= 0 && page < a.num_blocks;
            if (!page_ok) raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
            d_slot = page_ok ? static_cast<int>(page) : 0;
            int bits = 0;
            if (page_ok) {
              const uint8_t *vrow = a.valid + static_cast<int64_t>(b) * a.valid_stride;
#pragma unroll
              for (int t = 0; t < kDecStage; ++t) {
                const int pos = t0 + t;
                const bool on = t < d_n && (a.valid == nullptr || pos >= a.valid_len || vrow[pos] != 0);
                bits |= on ? (1 << t) : 0;
              }
            }
            // the current token (position seq_len - 1): its pool slot, and its row here
            // when this stage holds it and it is attended (the consumers copy it in)
            if (d_end && a.nk != nullptr) {
              const int64_t pos = a.seq_lens[b] - 1;
              const int64_t pcol = pos / kDecStage;
              int64_t npage = -1;
              if (pos >= 0 && pcol < a.table_width)
                npage = a.page_table[static_cast<int64_t>(b) * a.table_stride + pcol];
              if (npage >= 0 && npage < a.num_blocks) {
                d_noff = npage * a.sp + (pos - pcol * kDecStage) * a.ss;
              } else if (pos >= 0) {
                raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
              }
              const int64_t r = pos - t0;
              if (r >= 0 && r < d_n &&
                  (a.valid == nullptr || pos >= a.valid_len ||
                   a.valid[static_cast<int64_t>(b) * a.valid_stride + pos] != 0)) {
                d_nrow = static_cast<int>(r);
                bits |= 1 << d_nrow;  // attended from new_key / new_value even on a bad page
              }
            }
            d_vb = bits;
          } else {
            const int col = t0 / a.block_size;
            int blk = 0;
            if (col >= a.bt_stride) {  // context longer than its block-table row
              raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);
            } else {
              const int64_t at = static_cast<int64_t>(b) * a.bt_stride + col;
              blk = bt_cached ? s_bt[at] : a.block_tables[at];
              if (blk < 0 || blk >= a.num_blocks) {
                raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
                blk = 0;
              }
            }
            d_slot = blk * a.block_size + t0 % a.block_size;
          }
        }
        const int nw = min(32, j1 - wb);
        for (int i = 0; i < nw; ++i) {
          const int b = __shfl_sync(0xffffffffu, d_b, i);
          const int n = __shfl_sync(0xffffffffu, d_n, i);
          const int fl = __shfl_sync(0xffffffffu, d_fl, i);
          const int slot = __shfl_sync(0xffffffffu, d_slot, i);
          const int vb = __shfl_sync(0xffffffffu, d_vb, i);
          const int nrow = __shfl_sync(0xffffffffu, d_nrow, i);
          const int64_t noff = __shfl_sync(0xffffffffu, d_noff, i);
          const int end = __shfl_sync(0xffffffffu, d_end, i);
          if (end || n_early == kDecStages) wait_prev();
          int st;
          if (!acquire(st)) {
            wait_prev();
            drain();
            return;
          }
          if (lane == 0) {
            info[st] = StageInfo{b, n, fl, vb, nrow, noff};
            mbar_arrive_expect_tx(&full[st], C::TX_KV + ((fl & 1) ? C::TX_Q : 0));
          }
          __syncwarp();
          uint8_t *stage = stages + st * C::STAGE_BYTES;
          // One box per operand: 16 tokens x every KV head x both 64-dim halves (32 KiB).
          if constexpr (POOL) {
            if (lane < 2) tma_load_5d(stage + lane * C::KV_BYTES, lane ? &tm_v : &tm_k, 0, 0, 0, 0, slot, &full[st]);
          } else {
            if (lane < 2) tma_load_4d(stage + lane * C::KV_BYTES, lane ? &tm_v : &tm_k, 0, slot, 0, 0, &full[st]);
          }
          if (fl & 1) {
            if (!waited) {
              dq_st[n_dq] = st;
              dq_b[n_dq] = b;
              ++n_dq;
            } else if (lane == 2) {
              bulk_g2s(stage + 2 * C::KV_BYTES, a.q + b * a.q_stride, C::TX_Q, &full[st]);
            }
          }
          if (!waited) ++n_early;
          ++it_stage;
        }
      }
    }
    wait_prev();
    int st;  // terminal stage: tells the consumers to stop
    if (!acquire(st)) {
      drain();
      return;
    }
    if (lane == 0) {
      info[st] = StageInfo{-1, 0, 0, 0, -1, -1};
      mbar_arrive(&full[st]);
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  pdl_wait();  // partials, counters and outputs are written after the previous kernel
  asm volatile("bar.sync 2, %0;" ::"r"(C::THREADS) : "memory");  // stage prefix ready
  const int S = s_sp[B];
  const int geff = S < 1 ? 1 : (S < static_cast<int>(gridDim.x) ? S : static_cast<int>(gridDim.x));
  if (warp == 0) {  // per sequence: first owning CTA + prefix of partial slots
    int carry = 0;
    for (int b0 = 0; b0 < B; b0 += 32) {
      const int b = b0 + lane;
      int parts = 0, first = 0;
      if (b < B && s_sp[b + 1] > s_sp[b]) {
        first = owner_cta(S, s_sp[b], geff);
        parts = owner_cta(S, s_sp[b + 1] - 1, geff) - first + 1;
      }
      int incl = parts;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (b < B) {
        s_parts[b] = carry + incl - parts;
        s_first[b] = first;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_parts[B] = carry;  // <= B + geff - 1 <= parts_cap by construction
      if (carry > a.parts_cap) raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);
    }
  }
  consumer_sync(C::CONSUMERS);
  const bool parts_ok = s_parts[B] <= a.parts_cap;
  const int w = warp;               // KV head of this warp
  const int row = lane >> 2;        // MMA row = query head within the group (valid if < G)
  const int quad = lane & 3;
  const bool row_valid = row < G;
  const uint32_t stage_base = smem_addr(stages);
  const int lm_mat = lane >> 3, lm_row = lane & 7;  // ldmatrix: matrix and row of this lane

  if (blockIdx.x == 0) {  // rows with no keys: zeros (nothing else writes them)
    for (int b = w; b < B; b += HKV) {
      if (s_cuk[b + 1] - s_cuk[b] <= 0) {
        for (int i = lane; i < C::H * kDecD / 8; i += 32)
          reinterpret_cast<uint4 *>(a.out + b * a.out_stride)[i] = make_uint4(0, 0, 0, 0);
      }
    }
  }

  uint32_t qa[8][2];
  float o[16][4];
  float m_run = -INFINITY, l_run = 0.f;
  for (uint32_t it_stage = 0;; ++it_stage) {
    const int st = it_stage % kDecStages;
    const uint32_t ph = (it_stage / kDecStages) & 1;
    if (!mbar_wait(&full[st], ph, a.error_flag, &abort_flag)) return;
    const StageInfo si = info[st];
    if (si.b < 0) break;
    const int ntok = si.ntok;
    const uint32_t k_tile = stage_base + st * C::STAGE_BYTES + w * C::HEAD_TILE;
    const uint32_t v_tile = k_tile + C::KV_BYTES;

    if (si.flags & 1) {  // first stage of a segment: fresh state + this sequence's query
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
      m_run = -INFINITY;
      l_run = 0.f;
      const uint8_t *qs = stages + st * C::STAGE_BYTES + 2 * C::KV_BYTES +
                          (w * G + (row_valid ? row : 0)) * kDecD * 2;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t lo = *reinterpret_cast<const uint32_t *>(qs + (kk * 16 + quad * 2) * 2);
        const uint32_t hi = *reinterpret_cast<const uint32_t *>(qs + (kk * 16 + 8 + quad * 2) * 2);
        qa[kk][0] = row_valid ? lo : 0u;
        qa[kk][1] = row_valid ? hi : 0u;
      }
    }
    const int vbits = POOL ? si.vbits : (1 << ntok) - 1;
    if constexpr (POOL) {
      // The current token of the row: this warp's KV head row of new_key / new_value goes
      // into the stage (when attended here) and into the pools (when its page is usable).
      if (si.new_row >= 0 || si.new_off >= 0) {
        const int c = lane & 15, is_v = lane >> 4;
        const uint4 val = *reinterpret_cast<const uint4 *>((is_v ? a.nv : a.nk) + si.b * a.n_sb +
                                                           w * a.n_sh + c * 8);
        if (si.new_row >= 0) {
          uint8_t *tile = stages + st * C::STAGE_BYTES + is_v * C::KV_BYTES + w * C::HEAD_TILE;
          *reinterpret_cast<uint4 *>(tile + (c >> 3) * 2048 + swz(si.new_row, c & 7)) = val;
        }
        if (si.new_off >= 0)
          *reinterpret_cast<uint4 *>((is_v ? a.vp : a.kp) + si.new_off + w * a.sh + c * 8) = val;
        __syncwarp();
      }
    }
    if (vbits != (1 << kDecStage) - 1) {  // clear V rows not attended: 0 * stale bytes stays 0
      uint8_t *vt = stages + st * C::STAGE_BYTES + C::KV_BYTES + w * C::HEAD_TILE;
      for (int i = lane; i < kDecStage * 16; i += 32) {
        const int r = i / 16, ch = i % 16;
        if (!((vbits >> r) & 1))
          *reinterpret_cast<uint4 *>(vt + (ch >> 3) * 2048 + swz(r, ch & 7)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }

    // S = Q K^T for tokens 0-7 (n-tile 0) and 8-15 (n-tile 1).
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {  // k-steps 2kp, 2kp+1 = 16-byte chunks 4kp..4kp+3
        const int chunk = 4 * kp + lm_mat;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(k_tile + (chunk >> 3) * 2048 + swz(nt * 8 + lm_row, chunk & 7), b0, b1, b2, b3);
        mma16816(s[nt], qa[2 * kp][0], 0u, qa[2 * kp][1], 0u, b0, b1);
        mma16816(s[nt], qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u, b2, b3);
      }
    }
    // Online softmax on rows (one query head per quad), base 2.
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = nt * 8 + quad * 2 + e;
        s[nt][e] = ((vbits >> t) & 1) ? s[nt][e] * a.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[nt][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);  // ASR: token 0 of every stage is valid: finite
    // POOL: every key so far masked leaves m = -inf: exponentiate against 0 (all zeros)
    const float m_use = POOL && m_new == -INFINITY ? 0.f : m_new;
    const float alpha = exp2f(m_run - m_use);
    float p[2][2], sum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[nt][e] = exp2f(s[nt][e] - m_use);
        sum += p[nt][e];
      }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l_run = l_run * alpha + sum;
    m_run = m_new;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= alpha;
      o[j][1] *= alpha;
    }
    // O += P V: P (16 rows x 16 tokens) straight from the score registers.
    const uint32_t pa0 = row_valid ? pack2(p[0][0], p[0][1]) : 0u;
    const uint32_t pa2 = row_valid ? pack2(p[1][0], p[1][1]) : 0u;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {  // 16 head dims = chunks 2nd, 2nd+1
      const int chunk = 2 * nd + (lm_mat >> 1);
      const int trow = (lm_mat & 1) * 8 + lm_row;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(v_tile + (chunk >> 3) * 2048 + swz(trow, chunk & 7), b0, b1, b2, b3);
      mma16816(o[2 * nd], pa0, 0u, pa2, 0u, b0, b1);
      mma16816(o[2 * nd + 1], pa0, 0u, pa2, 0u, b2, b3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (!(si.flags & 2)) continue;

    // ---------------------------------------------------------- segment epilogue
    const int b = si.b;
    const int h = w * G + row;
    if (si.flags & 4) {
      if (row_valid) {
        const float inv = POOL && l_run == 0.f ? 0.f : 1.f / l_run;  // no attended key: zeros
        __nv_bfloat16 *dst = a.out + b * a.out_stride + h * kDecD + quad * 2;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          *reinterpret_cast<uint32_t *>(dst + j * 8) = pack2(o[j][0] * inv, o[j][1] * inv);
      }
      continue;
    }
    if (!parts_ok) continue;
    const int part = s_parts[b] + (static_cast<int>(blockIdx.x) - s_first[b]);
    if (row_valid) {
      float *dst = a.ws_o + (static_cast<int64_t>(part) * C::H + h) * kDecD + quad * 2;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<float2 *>(dst + j * 8) = make_float2(o[j][0], o[j][1]);
      if (quad == 0)
        *reinterpret_cast<float2 *>(a.ws_ml + (static_cast<int64_t>(part) * C::H + h) * 2) =
            make_float2(m_run, l_run);
    }
    const int n_parts = s_parts[b + 1] - s_parts[b];
    consumer_sync(C::CONSUMERS);
    if (tid == 0) {
      // Release this CTA's partial (cumulative over the barrier) and count it; the CTA
      // that brings the count to n_parts has acquired every other partial and merges
      // them after its last stage. A CTA's only partial segments are its first and last.
      int done;
      asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                   : "=r"(done)
                   : "l"(a.counters + b)
                   : "memory");
      if (done == n_parts - 1) {
        a.counters[b] = 0;  // every partial has arrived: ready for the next call
        if (s_npending < 2) s_pending[s_npending++] = b;
      }
    }
  }
  consumer_sync(C::CONSUMERS);  // all stages consumed: the stage buffers are free
  for (int k = 0; k < s_npending; ++k) {
    const int b = s_pending[k];
    merge_staged<C, POOL>(a, stages, s_parts[b], s_parts[b + 1] - s_parts[b], b, w, lane, tid);
  }
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

// =============================================================================
// Short contexts: one CTA per (sequence, KV head), no cross-CTA merge.
//
// With contexts of a few hundred tokens (the decode steps of ASR requests) the stream-K
// split above leaves every CTA a couple of stages and nearly every sequence split, so the
// partial writes, the counter round trip and the merge dominate the launch. Here a work
// unit is one KV head of one sequence: stages of 64 tokens of that head (one 16 KiB TMA
// box for K and one for V: {64 dims, 64 tokens, 2 halves, 1 head}), four consumer warps
// taking 16 tokens each with the same mma.sync QK^T / PV as above, and at the unit's end
// the four warps' softmax states combine in shared memory and the G query rows are
// written directly. B x H_kv units (256 for 32 sequences) keep the SMs busy without
// splitting any sequence's softmax across CTAs.
// =============================================================================
constexpr int kShortTok = 64;
constexpr int kShortStages = 3;
constexpr int kShortWarps = 4;    // consumer warps of one group: 16 tokens of a stage each
constexpr int kShortMaxCtx = 512;  // the host picks this kernel for max_seqlen_k <= 512
// Two consumer groups where two CTAs still fit an SM (G <= 2: scratch of 8 warps x G rows).
template <int G>
constexpr int short_groups() { return G <= 2 ? 2 : 1; }

// GR consumer groups of four warps: group g takes the stages j of a unit with j % GR == g,
// so GR stages of one unit are processed at once; every group keeps its own softmax state
// and the groups' states are combined at the unit's end. Each of the first GR stages of a
// unit carries the unit's query rows (one copy per group).
template <int G, int GR>
struct Short {
  static constexpr int HALF = kShortTok * 128;  // 64 tokens x 64 dims x 2 B = 8 KiB
  static constexpr int KV_BYTES = 2 * HALF;     // one head's K (or V) stage: 16 KiB
  static constexpr int Q_BYTES = ((G * kDecD * 2 + 1023) / 1024) * 1024;
  static constexpr int STAGE_BYTES = 2 * KV_BYTES + Q_BYTES;
  static constexpr int WARPS = kShortWarps * GR;  // consumer warps
  static constexpr int CONSUMERS = WARPS * 32;
  static constexpr int THREADS = CONSUMERS + 32;
  static constexpr int SCRATCH_BYTES = WARPS * G * (kDecD + 2) * 4;
  static constexpr size_t SMEM = 1024 + static_cast<size_t>(kShortStages) * STAGE_BYTES +
                                 SCRATCH_BYTES + 2 * kShortStages * 8 + kShortStages * 4 + 64;
  static_assert(GR == 1 || GR == 2, "one or two consumer groups");
  static_assert(2 * (SMEM + 1024) <= 233472, "two CTAs per SM");
};

template <int G, int GR>
__global__ void __launch_bounds__(Short<G, GR>::THREADS, 2)
    paged_decode_short_kernel(const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v, const DecodeArgs a,
                              int hkv) {
  using C = Short<G, GR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *stages = smem;
  float *scratch = reinterpret_cast<float *>(smem + kShortStages * C::STAGE_BYTES);
  uint64_t *full = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(scratch) + C::SCRATCH_BYTES);
  uint64_t *empty = full + kShortStages;
  // slot_seq[s]: number of the stage the producer last placed in ring slot s (-1: none).
  // With two groups, a group may reach its wait for stage q while the other group's stage
  // q - 3 still occupies the slot, possibly not yet landed: a parity wait would then match
  // the slot's older completed phase and pass early. A consumer therefore first waits
  // until slot_seq shows its own stage -- the producer writes it only after acquiring the
  // slot, i.e. after stage q - 3 was consumed -- and only then waits on the parity.
  volatile int *slot_seq = reinterpret_cast<volatile int *>(empty + kShortStages);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = a.batch, units = a.batch * hkv;
  pdl_trigger();
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < kShortStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kShortWarps);  // one group consumes each stage
      slot_seq[s] = -1;
    }
    fence_barrier_init();
  }
  if (warp == C::WARPS && lane == 0) {
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  __syncthreads();

  if (warp == C::WARPS) {
    // ------------------------------------------------------------------ producer
    // With programmatic dependent launch this CTA may start while the kernel before it
    // (the step's K/V store and q) still runs. The batch metadata and every cached row
    // but each sequence's newest come from launches that finished before the step's
    // decoder kernels began (the packer, earlier steps), so the first unit's stages
    // except its last -- the one holding the newest token -- are requested before the
    // wait; q and the last stage after it.
    uint32_t it_stage = 0;
    bool waited = a.early == 0;  // without PDL the wait returns at once: no early phase
    auto wait_prev = [&]() {
      if (!waited) pdl_wait();
      waited = true;
    };
    auto acquire = [&](int &st) -> bool {
      st = it_stage % kShortStages;
      const uint32_t ph = (it_stage / kShortStages) & 1;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[st], ph ^ 1, a.error_flag, &abort_flag);
      return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    // After an abort, wait (bounded) for the copies of every slot's last stage to land.
    auto drain = [&]() {
      if (lane != 0 || !abort_flag) return;
      for (int s = 0; s < kShortStages; ++s)
        if (slot_seq[s] >= 0) mbar_drain(&full[s], (slot_seq[s] / kShortStages) & 1);
    };
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const bool first_unit = u == static_cast<int>(blockIdx.x);
      if (!first_unit) wait_prev();
      const int b = u / hkv, h = u - (u / hkv) * hkv;
      // Lane i's block-table entry for stage i is read together with the length (the
      // column is in the row whatever the length; it is used only if stage i exists),
      // so the first TMA request waits for one global-memory latency, not two.
      const int col0 = lane * kShortTok / a.block_size;
      const int64_t row = static_cast<int64_t>(b) * a.bt_stride;
      const int c_lo = a.cu_seqlens_k[b], c_hi = a.cu_seqlens_k[b + 1];
      const int blk0 = col0 < a.bt_stride ? a.block_tables[row + col0] : 0;
      const int len = c_hi - c_lo;
      if (len <= 0) continue;  // zero rows: written by CTA 0's consumers
      const int nst = (len + kShortTok - 1) / kShortTok;
      const __nv_bfloat16 *q_src = a.q + b * a.q_stride + h * G * kDecD;
      // stages [0, early) go out before the wait (a fresh ring: no acquire blocks)
      const int early = waited ? 0 : min(nst - 1, kShortStages);
      int q_slots[GR], n_q = 0;  // early stages whose barrier also counts q (sent after the wait)
      for (int wb = 0; wb < nst; wb += 32) {
        // lane i: cache slot of stage wb + i (block-table reads in flight together)
        const int s = wb + lane;
        int d_slot = 0;
        if (s < nst) {
          const int t0 = s * kShortTok;
          const int col = t0 / a.block_size;
          int blk = 0;
          if (col >= a.bt_stride) {
            raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);
          } else {
            blk = wb == 0 ? blk0 : a.block_tables[row + col];
            if (blk < 0 || blk >= a.num_blocks) {
              raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
              blk = 0;
            }
          }
          d_slot = blk * a.block_size + t0 % a.block_size;
        }
        // Before the wait, the stages the ring cannot take yet -- and the one holding the
        // newest token, which the previous kernel writes through L2 -- are requested into
        // L2, so their loads after the wait are L2 hits.
        if (!waited && s < nst && s >= early) {
          tma_prefetch_4d(&tm_k, 0, d_slot, 0, h);
          tma_prefetch_4d(&tm_v, 0, d_slot, 0, h);
        }
        const int nw = min(32, nst - wb);
        for (int i = 0; i < nw; ++i) {
          const int j = wb + i;
          const int slot = __shfl_sync(0xffffffffu, d_slot, i);
          const bool with_q = j < GR;  // the first stage of each group carries q
          if (j >= early) wait_prev();
          int st;
          if (!acquire(st)) {
            wait_prev();
            drain();
            return;
          }
          if (lane == 0) {
            slot_seq[st] = static_cast<int>(it_stage);  // the slot's previous stage is consumed
            mbar_arrive_expect_tx(&full[st], 2 * C::KV_BYTES + (with_q ? G * kDecD * 2 : 0));
          }
          __syncwarp();
          uint8_t *stage = stages + st * C::STAGE_BYTES;
          if (lane < 2) tma_load_4d(stage + lane * C::KV_BYTES, lane ? &tm_v : &tm_k, 0, slot, 0, h, &full[st]);
          if (with_q) {
            if (j < early) {
              q_slots[n_q++] = st;
            } else if (lane == 2) {
              bulk_g2s(stage + 2 * C::KV_BYTES, q_src, G * kDecD * 2, &full[st]);
            }
          }
          ++it_stage;
          if (j == early - 1) {  // the early stages are out: wait, then their q copies
            wait_prev();
            if (lane == 2)
              for (int k = 0; k < n_q; ++k)
                bulk_g2s(stages + q_slots[k] * C::STAGE_BYTES + 2 * C::KV_BYTES, q_src,
                         G * kDecD * 2, &full[q_slots[k]]);
          }
        }
      }
    }
    wait_prev();
    drain();
    return;
  }

  // -------------------------------------------------------------------- consumers
  // Every consumer warp walks the CTA's units and their stages in the producer's order
  // (stage number = ring position), taking the stages of its group.
  pdl_wait();  // the output and the zero rows are written after the previous kernel
  const int w = warp % kShortWarps;  // token slice [16w, 16w + 16) of the group's stages
  const int grp = warp / kShortWarps;
  const int row = lane >> 2;         // MMA row = query head within the group (valid if < G)
  const int quad = lane & 3;
  const bool row_valid = row < G;
  const uint32_t stage_base = smem_addr(stages);
  const int lm_mat = lane >> 3, lm_row = lane & 7;
  constexpr int H = G;  // query rows of a unit

  if (blockIdx.x == 0) {  // rows with no keys: zeros
    for (int b = warp; b < B; b += C::WARPS) {
      if (a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b] <= 0) {
        for (int i = lane; i < hkv * G * kDecD / 8; i += 32)
          reinterpret_cast<uint4 *>(a.out + b * a.out_stride)[i] = make_uint4(0, 0, 0, 0);
      }
    }
  }

  // Token-major MMAs: with G = 1-4 query rows per unit, putting the 16 tokens of a
  // warp's slice on the MMA's M side (S^T = K Q^T, O^T += V^T P^T) halves the MMAs of
  // the row-major form (where 12-15 of every 16 query rows are padding), halves the
  // accumulator registers, and the QK^T sum runs as two independent chains. Lane
  // (g = lane / 4, c = lane % 4) holds S^T for tokens g and g + 8 and queries 2c, 2c + 1
  // (valid when < G), and O^T for dims 16 mt + g (+ 8) of the same queries.
  uint32_t qa[8][2];  // Q as the B operand: Q[g][16 kk + 2c ..], Q[g][16 kk + 8 + 2c ..]
  float o[8][4];
  float m_run[2], l_run[2];
  bool live = true;  // false once a wait timed out: skip work, keep taking part in barriers
  uint32_t it_stage = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int b = u / hkv, h = u - (u / hkv) * hkv;
    const int len = a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b];
    if (len <= 0) continue;
    const int nst = (len + kShortTok - 1) / kShortTok;
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    m_run[0] = m_run[1] = -INFINITY;
    l_run[0] = l_run[1] = 0.f;
    for (int js = 0; js < nst; ++js, ++it_stage) {
      if (js % GR != grp) continue;
      const int st = it_stage % kShortStages;
      const uint32_t ph = (it_stage / kShortStages) & 1;
      if (live && !slot_wait(&slot_seq[st], static_cast<int>(it_stage), a.error_flag, &abort_flag))
        live = false;
      if (live && !mbar_wait(&full[st], ph, a.error_flag, &abort_flag)) live = false;
      if (!live) continue;
      const int ntok = min(16, max(0, min(kShortTok, len - js * kShortTok) - 16 * w));
      const uint32_t k_tile = stage_base + st * C::STAGE_BYTES + w * 16 * 128;
      const uint32_t v_tile = k_tile + C::KV_BYTES;

      if (js < GR) {  // this group's first stage of the unit: the unit's query rows
        const uint8_t *qs = stages + st * C::STAGE_BYTES + 2 * C::KV_BYTES + (row_valid ? row : 0) * kDecD * 2;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t lo = *reinterpret_cast<const uint32_t *>(qs + (kk * 16 + quad * 2) * 2);
          const uint32_t hi = *reinterpret_cast<const uint32_t *>(qs + (kk * 16 + 8 + quad * 2) * 2);
          qa[kk][0] = row_valid ? lo : 0u;
          qa[kk][1] = row_valid ? hi : 0u;
        }
      }
      if (ntok > 0) {
        if (ntok < 16) {  // clear V rows past the end so 0 * stale bytes stays 0
          uint8_t *vt = stages + st * C::STAGE_BYTES + C::KV_BYTES + w * 16 * 128;
          for (int i = lane; i < (16 - ntok) * 16; i += 32) {
            const int r = ntok + i / 16, ch = i % 16;
            *reinterpret_cast<uint4 *>(vt + (ch >> 3) * C::HALF + swz(r, ch & 7)) = make_uint4(0, 0, 0, 0);
          }
          __syncwarp();
        }
        // S^T[16 tokens][8 queries] = K (A, 16 x 16 per step) x Q^T (B): even / odd steps
        // accumulate separately
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
        const int kt = (lm_mat & 1) * 8 + lm_row;  // ldmatrix row: token
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int chunk = 2 * kk + (lm_mat >> 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(k_tile + (chunk >> 3) * C::HALF + swz(kt, chunk & 7), a0, a1, a2, a3);
          mma16816_nv((kk & 1) ? sb : sa, a0, a1, a2, a3, qa[kk][0], qa[kk][1]);
        }
        // lane: tokens t0 = g, t1 = g + 8; queries 2c + e
        float sv[2][2];  // [token][e]
        const int t0 = row, t1 = row + 8;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          sv[0][e] = t0 < ntok ? (sa[e] + sb[e]) * a.scale_log2 : -INFINITY;
          sv[1][e] = t1 < ntok ? (sa[2 + e] + sb[2 + e]) * a.scale_log2 : -INFINITY;
        }
        float alpha[2], pr[2][2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float mx = fmaxf(sv[0][e], sv[1][e]);  // over the 16 tokens: lanes of equal c
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float m_new = fmaxf(m_run[e], mx);  // token 0 of the slice is valid: finite
          alpha[e] = exp2f(m_run[e] - m_new);
          pr[0][e] = exp2f(sv[0][e] - m_new);
          pr[1][e] = exp2f(sv[1][e] - m_new);
          float sum = pr[0][e] + pr[1][e];
          sum += __shfl_xor_sync(0xffffffffu, sum, 4);
          sum += __shfl_xor_sync(0xffffffffu, sum, 8);
          sum += __shfl_xor_sync(0xffffffffu, sum, 16);
          l_run[e] = l_run[e] * alpha[e] + sum;
          m_run[e] = m_new;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j][0] *= alpha[0];
          o[j][1] *= alpha[1];
          o[j][2] *= alpha[0];
          o[j][3] *= alpha[1];
        }
        // P^T (tokens x queries) as two 8x8 blocks in accumulator layout -> transposed into
        // the B fragments of O^T += V^T P^T (k = token, n = query)
        const uint32_t pb0 = movmatrix_t(pack2(pr[0][0], pr[0][1]));  // tokens 0-7
        const uint32_t pb1 = movmatrix_t(pack2(pr[1][0], pr[1][1]));  // tokens 8-15
        const int vt_row = (lm_mat >> 1) * 8 + lm_row;  // ldmatrix row: token
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int chunk = 2 * mt + (lm_mat & 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(v_tile + (chunk >> 3) * C::HALF + swz(vt_row, chunk & 7), a0, a1, a2, a3);
          mma16816_nv(o[mt], a0, a1, a2, a3, pb0, pb1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // ----------------------------------------- unit end: combine every warp's state
    float *sm = scratch + warp * H * (kDecD + 2);  // [H][2] (m, l) then [H][128] o
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int q = 2 * quad + e;
      if (q >= H) continue;
      if (row == 0) {
        sm[q * 2] = m_run[e];
        sm[q * 2 + 1] = l_run[e];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sm[2 * H + q * kDecD + j * 16 + row] = o[j][e];
        sm[2 * H + q * kDecD + j * 16 + row + 8] = o[j][2 + e];
      }
    }
    consumer_sync(C::CONSUMERS);
    for (int idx = threadIdx.x; live && idx < H * kDecD / 2; idx += C::CONSUMERS) {
      const int g = idx / (kDecD / 2), d = (idx % (kDecD / 2)) * 2;
      float mm = -INFINITY;
#pragma unroll
      for (int v = 0; v < C::WARPS; ++v) mm = fmaxf(mm, scratch[v * H * (kDecD + 2) + g * 2]);
      float l = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int v = 0; v < C::WARPS; ++v) {
        const float *sv = scratch + v * H * (kDecD + 2);
        const float wgt = exp2f(sv[g * 2] - mm);  // 0 for a warp that saw no token
        l += sv[g * 2 + 1] * wgt;
        o0 += sv[2 * H + g * kDecD + d] * wgt;
        o1 += sv[2 * H + g * kDecD + d + 1] * wgt;
      }
      const float inv = 1.f / l;
      *reinterpret_cast<uint32_t *>(a.out + b * a.out_stride + (h * G + g) * kDecD + d) =
          pack2(o0 * inv, o1 * inv);
    }
    consumer_sync(C::CONSUMERS);  // scratch is reused by the next unit
  }
  // A consumer that gave up leaves stages unconsumed: let their copies land before exit.
  if (threadIdx.x == 0 && abort_flag)
    for (int s = 0; s < kShortStages; ++s)
      if (slot_seq[s] >= 0) mbar_drain(&full[s], (slot_seq[s] / kShortStages) & 1);
}

template <int G, int GR>
int launch_decode_short(const DecodeArgs &a, int hkv, const void *k_cache, const void *v_cache,
                        int64_t num_slots, cudaStream_t stream) {
  using C = Short<G, GR>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(paged_decode_short_kernel<G, GR>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(C::SMEM));
    if (e != cudaSuccess) {
      set_error("paged_decode: cannot reserve %zu bytes of shared memory: %s", C::SMEM,
                cudaGetErrorString(e));
      return B200ASR_ERR_CUDA;
    }
    configured = true;
  }
  // {64 dims, slots, 2 halves, hkv heads}; box {64, 64 tokens, 2, 1 head} lands as
  // [half][token][64 dims] with the 128-byte swizzle: one head's 64-token K or V tile.
  CUtensorMap tk, tv;
  const uint64_t dims[4] = {64, static_cast<uint64_t>(num_slots), 2, static_cast<uint64_t>(hkv)};
  const uint64_t strides[3] = {static_cast<uint64_t>(hkv) * kDecD * 2, 128, 256};
  const uint32_t box[4] = {64, kShortTok, 2, 1};
  if (!make_tmap_bf16(&tk, k_cache, 4, dims, strides, box) ||
      !make_tmap_bf16(&tv, v_cache, 4, dims, strides, box))
    return B200ASR_ERR_CUDA;
  const int units = a.batch * hkv;
  const int grid = std::min(units, 2 * num_sms());
  B200_LAUNCH_CHECK_ERR(launch_kernel(paged_decode_short_kernel<G, GR>, dim3(grid), dim3(C::THREADS),
                                      C::SMEM, stream, true, 1, tk, tv, a, hkv),
                        "paged_decode (short contexts)");
  return B200ASR_OK;
}

template <int HKV, int G>
int launch_decode(const DecodeArgs &a, const void *k_cache, const void *v_cache,
                  int64_t num_slots, cudaStream_t stream) {
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
  // The cache [slots][HKV][128] bf16 viewed as {64 dims, slots, 2 halves, HKV heads}: one
  // box of {64, 16, 2, HKV} lands in shared memory as [head][half][token][64 dims], i.e.
  // per head a 16 x 128 K (or V) tile in two 128-byte-swizzled halves. A single large box
  // per operand matters: an SM keeps only a limited number of TMA boxes in flight, and
  // with 2 boxes per stage (rather than 4 * HKV) all stages of the ring stream at once.
  CUtensorMap tk, tv;
  const uint64_t dims[4] = {64, static_cast<uint64_t>(num_slots), 2, HKV};
  const uint64_t strides[3] = {HKV * kDecD * 2ull, 128, 256};
  const uint32_t box[4] = {64, kDecStage, 2, HKV};
  if (!make_tmap_bf16(&tk, k_cache, 4, dims, strides, box) ||
      !make_tmap_bf16(&tv, v_cache, 4, dims, strides, box))
    return B200ASR_ERR_CUDA;
  const int grid = std::min(num_sms(), kDecMaxGrid);
  B200_LAUNCH_CHECK_ERR(launch_kernel(paged_decode_kernel<HKV, G>, dim3(grid), dim3(C::THREADS),
                                      C::SMEM, stream, true, 1, tk, tv, a),
                        "paged_decode");
  return B200ASR_OK;
}

// Partials: every sequence contributes at most one per CTA boundary it straddles plus one.
size_t decode_parts_cap(int batch) { return static_cast<size_t>(batch) + kDecMaxGrid; }

template <int HKV, int G>
int launch_decode_pool(const DecodeArgs &a, const CUtensorMap &tk, const CUtensorMap &tv,
                       cudaStream_t stream) {
  using C = Dec<HKV, G>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(paged_decode_kernel<HKV, G, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(C::SMEM));
    if (e != cudaSuccess) {
      set_error("pool_paged_decode: cannot reserve %zu bytes of shared memory: %s", C::SMEM,
                cudaGetErrorString(e));
      return B200ASR_ERR_CUDA;
    }
    configured = true;
  }
  const int grid = std::min(num_sms(), kDecMaxGrid);
  B200_LAUNCH_CHECK_ERR(launch_kernel(paged_decode_kernel<HKV, G, true>, dim3(grid),
                                      dim3(C::THREADS), C::SMEM, stream, false, 1, tk, tv, a),
                        "pool_paged_decode (stream-K)");
  return B200ASR_OK;
}

int pool_decode_stream_k(const PoolStreamK &p, bool *taken) {
  *taken = false;
  const int hq = p.num_heads, hkv = p.num_kv_heads;
  const bool heads = (hkv == 8 && (hq == 16 || hq == 8)) || (hkv == 4 && (hq == 16 || hq == 8)) ||
                     (hkv == 2 && hq == 4);
  if (!heads || p.head_dim != kDecD || p.page_size != kDecStage || p.batch > kDecMaxBatch ||
      p.q_stride_h != kDecD || p.out_stride_h != kDecD || p.q_stride_b % 8 != 0 ||
      p.out_stride_b % 4 != 0 || p.kv_stride_s % 8 != 0 || p.kv_stride_h % 8 != 0 ||
      p.kv_stride_p % 8 != 0 || p.kv_stride_s < kDecD || p.num_pages <= 0)
    return B200ASR_OK;
  const size_t parts = decode_parts_cap(p.batch);
  const size_t base = (p.workspace_head + 255) / 256 * 256 > kDecHeaderBytes
                          ? (p.workspace_head + 255) / 256 * 256 : kDecHeaderBytes;
  if (p.workspace_bytes < base + parts * hq * (kDecD + 2) * sizeof(float)) return B200ASR_OK;
  // Pool [pages][heads][16][128] bf16 as {64 dims, 16 positions, 2 halves, heads, pages}: a
  // box {64, 16, 2, HKV, 1} lands as [head][half][token][64 dims], the stage layout the
  // stream-K consumers read.
  CUtensorMap tk, tv;
  const uint64_t dims[5] = {64, kDecStage, 2, static_cast<uint64_t>(hkv),
                            static_cast<uint64_t>(p.num_pages)};
  const uint64_t strides[4] = {static_cast<uint64_t>(p.kv_stride_s) * 2, 128,
                               static_cast<uint64_t>(p.kv_stride_h) * 2,
                               static_cast<uint64_t>(p.kv_stride_p) * 2};
  const uint32_t box[5] = {64, kDecStage, 2, static_cast<uint32_t>(hkv), 1};
  if (!make_tmap_bf16(&tk, p.key_pool, 5, dims, strides, box) ||
      !make_tmap_bf16(&tv, p.value_pool, 5, dims, strides, box))
    return B200ASR_ERR_CUDA;
  DecodeArgs a{};
  a.q = static_cast<const __nv_bfloat16 *>(p.query);
  a.q_stride = p.q_stride_b;
  a.num_blocks = p.num_pages;
  a.block_size = kDecStage;
  a.batch = p.batch;
  a.scale_log2 = p.scale * kLog2e;
  a.out = static_cast<__nv_bfloat16 *>(p.out);
  a.out_stride = p.out_stride_b;
  a.parts_cap = static_cast<int>(parts);
  a.counters = static_cast<int *>(p.workspace);  // zero at rest, like the pool kernel's
  a.ws_ml = reinterpret_cast<float *>(static_cast<uint8_t *>(p.workspace) + base);
  a.ws_o = a.ws_ml + parts * hq * 2;
  a.error_flag = p.error_flag;
  a.early = 0;
  a.seq_lens = p.seq_lens;
  a.max_seq_len = p.max_seq_len;
  a.page_table = p.page_table;
  a.table_stride = p.table_stride;
  a.table_width = p.table_width;
  a.valid = p.valid;
  a.valid_stride = p.valid_stride;
  a.valid_len = p.valid ? p.valid_len : 0;
  a.nk = static_cast<const __nv_bfloat16 *>(p.new_key);
  a.nv = static_cast<const __nv_bfloat16 *>(p.new_value);
  a.n_sb = p.new_stride_b;
  a.n_sh = p.new_stride_h;
  a.kp = static_cast<__nv_bfloat16 *>(p.key_pool);
  a.vp = static_cast<__nv_bfloat16 *>(p.value_pool);
  a.sp = p.kv_stride_p;
  a.sh = p.kv_stride_h;
  a.ss = p.kv_stride_s;
  *taken = true;
  const cudaStream_t st = static_cast<cudaStream_t>(p.stream);
  if (hkv == 8 && hq == 16) return launch_decode_pool<8, 2>(a, tk, tv, st);
  if (hkv == 8 && hq == 8) return launch_decode_pool<8, 1>(a, tk, tv, st);
  if (hkv == 4 && hq == 16) return launch_decode_pool<4, 4>(a, tk, tv, st);
  if (hkv == 4 && hq == 8) return launch_decode_pool<4, 2>(a, tk, tv, st);
  return launch_decode_pool<2, 2>(a, tk, tv, st);
}

}  // namespace b200asr

using namespace b200asr;

extern "C" size_t b200asr_paged_decode_workspace_size(int32_t batch, int32_t max_seqlen_k,
                                                      int32_t num_heads, int32_t head_dim) {
  if (batch <= 0 || num_heads <= 0 || head_dim <= 0) return 0;
  (void)max_seqlen_k;  // the stream-K split bounds the partials by batch + grid, not length
  const size_t parts = decode_parts_cap(batch);
  return kDecHeaderBytes + parts * num_heads * (static_cast<size_t>(head_dim) + 2) * sizeof(float);
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
  B200_REQUIRE(block_size >= kDecStage && block_size % kDecStage == 0,
               "paged_decode: block_size %d must be a multiple of %d", block_size, kDecStage);
  B200_REQUIRE(num_blocks >= 1 && bt_stride >= 1 && max_seqlen_k >= 1,
               "paged_decode: bad table geometry");
  B200_REQUIRE(q && k_cache && v_cache && cu_seqlens_k && block_tables && out && workspace,
               "paged_decode: null pointer");
  B200_REQUIRE(q_row_stride >= static_cast<int64_t>(num_heads) * head_dim && q_row_stride % 8 == 0 &&
                   out_row_stride % 4 == 0 && aligned16(q) && aligned16(k_cache) &&
                   aligned16(v_cache) && aligned16(workspace) &&
                   (reinterpret_cast<uintptr_t>(out) & 7) == 0,
               "paged_decode: misaligned tensor (q rows must be contiguous and 16-byte aligned)");
  const size_t need = b200asr_paged_decode_workspace_size(batch, max_seqlen_k, num_heads, head_dim);
  if (workspace_bytes < need) {
    set_error("paged_decode: workspace %zu bytes < %zu needed", workspace_bytes, need);
    return B200ASR_ERR_WORKSPACE;
  }
  DecodeArgs a{};
  a.q = static_cast<const __nv_bfloat16 *>(q);
  a.q_stride = q_row_stride;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.cu_seqlens_k = cu_seqlens_k;
  a.block_tables = block_tables;
  a.bt_stride = bt_stride;
  a.batch = batch;
  a.scale_log2 = scale * kLog2e;
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.out_stride = out_row_stride;
  a.parts_cap = static_cast<int>(decode_parts_cap(batch));
  a.counters = static_cast<int *>(workspace);
  a.ws_ml = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kDecHeaderBytes);
  a.ws_o = a.ws_ml + static_cast<size_t>(a.parts_cap) * num_heads * 2;
  a.error_flag = error_flag;
  a.early = pdl_enabled() ? 1 : 0;
  const int64_t slots = static_cast<int64_t>(num_blocks) * block_size;
  // Contexts of at most kShortMaxCtx tokens: one CTA per (sequence, KV head).
  if (max_seqlen_k <= kShortMaxCtx && block_size % kShortTok == 0 &&
      num_heads % num_kv_heads == 0 && num_kv_heads <= 8) {
    const int g = num_heads / num_kv_heads;
    if (g == 1) return launch_decode_short<1, short_groups<1>()>(a, num_kv_heads, k_cache, v_cache, slots, stream);
    if (g == 2) return launch_decode_short<2, short_groups<2>()>(a, num_kv_heads, k_cache, v_cache, slots, stream);
    if (g == 4) return launch_decode_short<4, short_groups<4>()>(a, num_kv_heads, k_cache, v_cache, slots, stream);
  }
  if (num_kv_heads == 8 && num_heads == 16) return launch_decode<8, 2>(a, k_cache, v_cache, slots, stream);
  if (num_kv_heads == 8 && num_heads == 8) return launch_decode<8, 1>(a, k_cache, v_cache, slots, stream);
  if (num_kv_heads == 4 && num_heads == 16) return launch_decode<4, 4>(a, k_cache, v_cache, slots, stream);
  if (num_kv_heads == 4 && num_heads == 8) return launch_decode<4, 2>(a, k_cache, v_cache, slots, stream);
  if (num_kv_heads == 2 && num_heads == 4) return launch_decode<2, 2>(a, k_cache, v_cache, slots, stream);
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
// use the symbol's name as a device address, so the first call on each device (with that
// device current) resolves it once with cudaGetSymbolAddress and caches the pointer. That
// first call may load the module, so it should come before any stream capture.
//
// The per-sequence merge counters at the head of the array must be zero when a launch
// starts. Every call therefore clears them with cudaMemsetAsync on the caller's stream,
// right before its kernel: the clear is ordered with the launch on any stream (a
// non-blocking one included), and counters that a call whose waits timed out left
// behind do not leak into the next call. No call allocates. All calls share the one
// array, so two calls whose kernels overlap on the GPU -- different streams, or graphs
// replayed concurrently -- race on it and must be serialised by the caller.

static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[B200ASR_NOALLOC_SCRATCH_BYTES];

namespace b200asr {

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
      set_error("paged_decode_noalloc: set-up of the static scratch failed on device %d: %s", dev,
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
    set_error("paged_decode_noalloc: batch %d x %d heads needs %zu bytes of scratch, more than "
              "the built-in %zu; use b200asr_paged_decode with a workspace",
              batch, num_heads, need,
              static_cast<size_t>(B200ASR_NOALLOC_SCRATCH_BYTES));
    return B200ASR_ERR_WORKSPACE;
  }
  if (batch == 0) return B200ASR_OK;
  int status = B200ASR_OK;
  void *scratch = noalloc_scratch(&status);
  if (scratch == nullptr) return status;
  // Merge counters to zero on the caller's stream, ordered before this call's kernel.
  const cudaError_t e = cudaMemsetAsync(scratch, 0, kDecHeaderBytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("paged_decode_noalloc: clearing the merge counters failed: %s", cudaGetErrorString(e));
    return B200ASR_ERR_CUDA;
  }
  return b200asr_paged_decode(q, q_row_stride, k_cache, v_cache, num_blocks, block_size,
                              num_heads, num_kv_heads, head_dim, cu_seqlens_k, block_tables,
                              bt_stride, batch, max_seqlen_k, scale, out, out_row_stride, scratch,
                              B200ASR_NOALLOC_SCRATCH_BYTES, error_flag, stream);
}
