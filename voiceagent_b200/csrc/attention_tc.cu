// Tensor-core (tcgen05 / TMEM / TMA) attention kernels for sm_100a.
//
// paged_prefill    <- PagedAttention.forward prefill/mixed rows (layers/attention.py:87-107):
//                     flash_attn_varlen_func(..., causal=True, block_table=...) over the
//                     paged cache, causal mask aligned bottom-right.
// varlen_attention <- VarlenSelfAttention.forward (layers/attention.py:121-139) for the
//                     audio encoder's 104-token windows, causal=False.
//
// Common structure (one CTA = 6 warps):
//   warps 0-3  softmax / correction / epilogue; thread i owns accumulator row i (TMEM
//              lane i), so row max and row sum need no shuffles;
//   warp 4     TMA producer (one elected lane);
//   warp 5     TMEM allocator and tcgen05.mma issuer (one elected lane).
// Operands live in shared memory in the 128-byte-swizzled layout TMA writes and the
// UMMA descriptors read (8-row x 128-byte atoms, 1024-byte aligned). Q and K are
// K-major; V is read as an MN-major B operand straight from its [key][dim] tile; P is
// written by the softmax threads in the same swizzled K-major layout.
#include "common.cuh"

namespace b200asr {

constexpr int kTcThreads = 192;
constexpr float kTcLog2e = 1.4426950408889634f;

__device__ __forceinline__ int named_bar_softmax() { return 128; }
__device__ __forceinline__ void softmax_bar() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Store one 64-column bf16 row (from fp32 `p`) into a K-major SW128 tile at row r.
__device__ __forceinline__ void store_p_row64(uint8_t *tile, int r, const float *p) {
  uint8_t *row = tile + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 v;
    v.x = pack2(p[8 * c + 0], p[8 * c + 1]);
    v.y = pack2(p[8 * c + 2], p[8 * c + 3]);
    v.z = pack2(p[8 * c + 4], p[8 * c + 5]);
    v.w = pack2(p[8 * c + 6], p[8 * c + 7]);
    *reinterpret_cast<uint4 *>(row + ((c ^ (r & 7)) << 4)) = v;
  }
}

// =============================================================================
// Paged causal GQA prefill, head_dim 128, query heads = 2 x KV heads.
// Work item = (64 query tokens of one sequence) x (one KV head g): M rows 0-63 are query
// head 2g, rows 64-127 query head 2g+1, tokens t = row & 63.
//
// Persistent: the grid is at most two CTAs per SM and CTA c takes items c, c + grid, ...
// (item = query tile * KV heads + g, query tiles numbered sequence by sequence). TMEM
// (S in two 64-column buffers, O in 128 columns) and the barriers are set up once per
// CTA. Only the producer warp locates an item (a warp scan over the query lengths, the
// lengths and the block ids of its KV tiles): it runs ahead, and hands the item's
// parameters to the MMA and softmax warps through a two-slot shared-memory ring. The
// next item's Q and first K/V tiles load while the current item's last P V and epilogue
// run; its first P V waits until the epilogue has read O.
// =============================================================================

constexpr int kPfBN = 64;                      // keys per KV tile
constexpr int kPfQBytes = 128 * 128 * 2;       // 32 KiB: 2 d-halves x [128 rows x 128 B]
constexpr int kPfKVBytes = kPfBN * 128 * 2;    // 16 KiB: 2 d-halves x [64 rows x 128 B]
constexpr int kPfPBytes = 128 * kPfBN * 2;     // 16 KiB: [128 rows x 128 B]
constexpr int kPfStages = 2;
// P of tile j is written over K of tile j (same stage, same 16 KiB): S = Q K^T has
// completed when the softmax reads S, and the stage is refilled only after P V of tile j.
// Without a separate P buffer the CTA needs ~97 KB, so two CTAs share an SM.
static_assert(kPfPBytes == kPfKVBytes, "P reuses its tile's K buffer");
constexpr int kPfSmem = 1024 /*align slack*/ + kPfQBytes + 2 * kPfStages * kPfKVBytes + 512;
// Online softmax with lazy rescaling (the conditional rescale of FlashAttention-4): the
// running maximum a row exponentiates against only moves when a tile's maximum exceeds it
// by more than kPfRescaleLog2 (base 2), so P stays below 2^8 and O in TMEM is rescaled
// (a TMEM round trip of 128 columns) on few tiles instead of most. The final O / l uses
// the same maximum for both, so the result is the softmax whichever maximum was used.
constexpr float kPfRescaleLog2 = 8.f;

struct PrefillArgs {
  const int32_t *cu_seqlens_q;
  const int32_t *cu_seqlens_k;
  const int32_t *block_tables;
  int bt_stride;
  int batch;
  int num_blocks;
  int block_size;
  int num_kv_heads;
  int items;  // upper bound of (query tile, KV head) items
  float scale_log2;
  __nv_bfloat16 *out;
  int64_t out_stride;
  int32_t *error_flag;
};

// An item's parameters as the producer publishes them (one ring slot).
struct PfItem {
  int q0, nq, p_first, n_kv, n_tiles, g;  // n_tiles < 0: no more items
};

__global__ void __launch_bounds__(kTcThreads, 2)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sQ = smem;
  uint8_t *sK = sQ + kPfQBytes;                  // [stage] 16 KiB each
  uint8_t *sV = sK + kPfStages * kPfKVBytes;     // [stage] 16 KiB each
  uint64_t *bars = reinterpret_cast<uint64_t *>(sV + kPfStages * kPfKVBytes);
  uint64_t *q_full = bars + 0;     // Q of the item landed (one phase per item)
  uint64_t *q_empty = bars + 1;    // the item's last S = Q K^T done: Q may be refilled
  uint64_t *kv_full = bars + 2;    // [2] per KV tile (global tile count)
  uint64_t *kv_empty = bars + 4;   // [2]
  uint64_t *s_full = bars + 6;     // [2]
  uint64_t *s_free = bars + 8;     // [2] (128 arrivals)
  uint64_t *p_full = bars + 10;    // [2] (128 arrivals)
  uint64_t *o_done = bars + 12;    // one phase per P V tile
  uint64_t *o_last = bars + 13;    // one phase per item: its last P V
  uint64_t *o_free = bars + 14;    // one phase per item: O read by the epilogue (128)
  uint64_t *meta_full = bars + 15;   // [2] ring slot written
  uint64_t *meta_empty = bars + 17;  // [2] ring slot read by the MMA thread and the softmax
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 19);
  PfItem *ring = reinterpret_cast<PfItem *>(bars + 20);  // [2]
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    abort_flag = 0;
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
      mbar_init(&p_full[s], 128);
      mbar_init(&meta_full[s], 1);
      mbar_init(&meta_empty[s], 129);
    }
    mbar_init(o_done, 1);
    mbar_init(o_last, 1);
    mbar_init(o_free, 128);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer (whole warp)
    // Query tiles are located by a warp scan over the sequences' tile counts; the items
    // of this CTA come in increasing order, so the scan resumes where it stopped.
    int scan_b0 = 0, scan_carry = 0;
    auto locate = [&](int t, int &b, int &qtile) -> bool {
      while (scan_b0 < a.batch) {
        const int bb = scan_b0 + lane;
        int n = 0;
        if (bb < a.batch) n = (a.cu_seqlens_q[bb + 1] - a.cu_seqlens_q[bb] + 63) / 64;
        int incl = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        if (t < scan_carry + total) {
          const int excl = scan_carry + incl - n;
          const unsigned ball = __ballot_sync(0xffffffffu, bb < a.batch && t >= excl && t < excl + n);
          const int src = __ffs(ball) - 1;
          b = scan_b0 + src;
          qtile = t - __shfl_sync(0xffffffffu, excl, src);
          return true;
        }
        scan_carry += total;
        scan_b0 += 32;
      }
      return false;
    };
    uint32_t it = 0, jg = 0;  // items published, KV tiles issued
    bool ok = true;
    // publish ring slot it & 1 (after its previous readers are done)
    auto publish = [&](const PfItem &item) -> bool {
      const int slot = it & 1;
      int good = 1;
      if (lane == 0) {
        good = it < 2 || mbar_wait(&meta_empty[slot], ((it >> 1) & 1) ^ 1, a.error_flag, &abort_flag);
        if (good) {
          volatile PfItem *r = ring + slot;
          r->q0 = item.q0;
          r->nq = item.nq;
          r->p_first = item.p_first;
          r->n_kv = item.n_kv;
          r->n_tiles = item.n_tiles;
          r->g = item.g;
          mbar_arrive(&meta_full[slot]);
        }
      }
      return __shfl_sync(0xffffffffu, good, 0) != 0;
    };
    for (int i = blockIdx.x; ok && i < a.items; i += gridDim.x) {
      const int t = i / a.num_kv_heads, g = i - t * a.num_kv_heads;
      int b, qtile;
      if (!locate(t, b, qtile)) break;  // past the last query tile
      const int q_len = a.cu_seqlens_q[b + 1] - a.cu_seqlens_q[b];
      const int k_len = a.cu_seqlens_k[b + 1] - a.cu_seqlens_k[b];
      PfItem item;
      item.q0 = a.cu_seqlens_q[b] + qtile * 64;
      item.nq = min(64, q_len - qtile * 64);
      const int offset = k_len - q_len;  // bottom-right alignment
      item.p_first = offset + qtile * 64;
      item.n_kv = min(k_len, item.p_first + item.nq);
      item.n_tiles = item.n_kv > 0 ? (item.n_kv + kPfBN - 1) / kPfBN : 0;
      item.g = g;
      if (offset < 0) {
        if (lane == 0) raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);
        continue;
      }
      if (item.n_tiles == 0) continue;
      if (!publish(item)) {
        ok = false;
        break;
      }
      // Q: after the previous item's last S = Q K^T
      if (lane == 0) {
        if (it > 0 && !mbar_wait(q_empty, (it - 1) & 1, a.error_flag, &abort_flag)) ok = false;
        if (ok) {
          mbar_arrive_expect_tx(q_full, kPfQBytes);
          for (int hh = 0; hh < 2; ++hh)
            for (int dh = 0; dh < 2; ++dh)
              tma_load_3d(sQ + dh * 16384 + hh * 8192, &tm_q, dh * 64, 2 * g + hh, item.q0, q_full);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++it;
      // K/V tiles: lane l reads the cache slot of tile w0 + l (reads in flight together)
      const int64_t bt_row = static_cast<int64_t>(b) * a.bt_stride;
      for (int w0 = 0; ok && w0 < item.n_tiles; w0 += 32) {
        int slot = 0;
        if (w0 + lane < item.n_tiles) {
          const int key0 = (w0 + lane) * kPfBN;
          int block = a.block_tables[bt_row + key0 / a.block_size];
          if (block < 0 || block >= a.num_blocks) {
            raise_flag(a.error_flag, B200ASR_DEVERR_BLOCK);
            block = 0;
          }
          slot = block * a.block_size + (key0 % a.block_size);
        }
        const int nw = min(32, item.n_tiles - w0);
        for (int l = 0; l < nw; ++l, ++jg) {
          const int sl = __shfl_sync(0xffffffffu, slot, l);
          if (lane == 0) {
            const int st = jg & 1;
            if (!mbar_wait(&kv_empty[st], ((jg >> 1) & 1) ^ 1, a.error_flag, &abort_flag)) {
              ok = false;
            } else {
              mbar_arrive_expect_tx(&kv_full[st], 2 * kPfKVBytes);
              uint8_t *k_dst = sK + st * kPfKVBytes;
              uint8_t *v_dst = sV + st * kPfKVBytes;
              for (int dh = 0; dh < 2; ++dh) {
                tma_load_3d(k_dst + dh * 8192, &tm_k, dh * 64, g, sl, &kv_full[st]);
                tma_load_3d(v_dst + dh * 8192, &tm_v, dh * 64, g, sl, &kv_full[st]);
              }
            }
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          if (!ok) break;
        }
      }
    }
    if (ok) {  // end marker
      PfItem end{};
      end.n_tiles = -1;
      publish(end);
    }
    // after an abort: let the copies already requested land before the CTA exits
    if (lane == 0 && abort_flag) {
      if (it > 0) mbar_drain(q_full, (it - 1) & 1);
      for (uint32_t k = jg > 2 ? jg - 2 : 0; k < jg; ++k) mbar_drain(&kv_full[k & 1], (k >> 1) & 1);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, kPfBN, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128, false, true);
      const uint32_t q_base = smem_addr(sQ), k_base = smem_addr(sK), v_base = smem_addr(sV);
      // P V of global tile jj, tile j of the item (j == 0 overwrites O)
      auto issue_pv = [&](uint32_t jj, int j, bool last) {
        const uint32_t vb = v_base + (jj & 1) * kPfKVBytes;
        const uint32_t pb = k_base + (jj & 1) * kPfKVBytes;  // P(jj) over K(jj)
#pragma unroll
        for (int k = 0; k < kPfBN / 16; ++k) {
          const uint64_t ad = smem_desc_sw128(pb + k * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(vb + k * 2048, 8192, 1024);
          umma_f16_ss(tmem + 128, ad, bd, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[jj & 1]);
        umma_commit(o_done);
        if (last) umma_commit(o_last);
      };
      uint32_t jg = 0;
      bool ok = true;
      for (uint32_t it = 0; ok; ++it) {
        const int slot = it & 1;
        if (!mbar_wait(&meta_full[slot], (it >> 1) & 1, a.error_flag, &abort_flag)) break;
        const int n_tiles = ring[slot].n_tiles;
        tc_fence_before();
        mbar_arrive(&meta_empty[slot]);
        if (n_tiles < 0) break;
        if (!mbar_wait(q_full, it & 1, a.error_flag, &abort_flag)) break;
        // the item's first P V overwrites O: the previous item's epilogue must have read it
        bool o_ready = it == 0;
        auto wait_o = [&]() -> bool {
          if (!o_ready) o_ready = mbar_wait(o_free, (it - 1) & 1, a.error_flag, &abort_flag);
          return o_ready;
        };
        for (int j = 0; j < n_tiles; ++j, ++jg) {
          const int st = jg & 1;
          if (!mbar_wait(&kv_full[st], (jg >> 1) & 1, a.error_flag, &abort_flag)) { ok = false; break; }
          if (jg >= 2 && !mbar_wait(&s_free[st], ((jg - 2) >> 1) & 1, a.error_flag, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t kb = k_base + st * kPfKVBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
            const uint32_t koff = (k >> 2) * 8192 + (k & 3) * 32;
            const uint64_t ad = smem_desc_sw128(q_base + off, 16, 1024);
            const uint64_t bd = smem_desc_sw128(kb + koff, 16, 1024);
            umma_f16_ss(tmem + st * kPfBN, ad, bd, idesc_s, k > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[st]);
          if (j == n_tiles - 1) umma_commit(q_empty);  // Q of this item no longer read
          if (j >= 1) {
            const uint32_t jp = jg - 1;
            if (!mbar_wait(&p_full[jp & 1], (jp >> 1) & 1, a.error_flag, &abort_flag) ||
                (j == 1 && !wait_o())) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(jp, j - 1, false);
          }
        }
        if (!ok) break;
        const uint32_t jl = jg - 1;
        if (!mbar_wait(&p_full[jl & 1], (jl >> 1) & 1, a.error_flag, &abort_flag) || !wait_o()) break;
        tc_fence_after();
        issue_pv(jl, n_tiles - 1, true);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax (warps 0-3)
    const int r = tid;                   // accumulator row == TMEM lane
    const int t = r & 63;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    uint32_t jg = 0;
    for (uint32_t it = 0;; ++it) {
      const int slot = it & 1;
      if (!mbar_wait(&meta_full[slot], (it >> 1) & 1, a.error_flag, &abort_flag)) break;
      const PfItem item = *const_cast<const PfItem *>(ring + slot);
      tc_fence_before();
      mbar_arrive(&meta_empty[slot]);
      if (item.n_tiles < 0) break;
      const int head = 2 * item.g + (r >> 6);
      const int p_row = item.p_first + t;  // last key this row may attend
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < item.n_tiles; ++j, ++jg) {
        const int st = jg & 1;
        if (!mbar_wait(&s_full[st], (jg >> 1) & 1, a.error_flag, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        float s[kPfBN];
        tmem_ld32(lane_base + st * kPfBN, s);
        tmem_ld32(lane_base + st * kPfBN + 32, s + 32);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_free[st]);
        const int key0 = j * kPfBN;
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < kPfBN; ++c) {
          s[c] = (key0 + c <= p_row) ? s[c] * a.scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
        // Tile 0 sets the maximum (key 0 is visible to every row: finite). Later tiles
        // move it only past the threshold; O then needs its rescale, after P V of the
        // previous tile. At tile j that P V is the only one that can be outstanding (S of
        // tile j was issued after P V of tile j - 2), so the parity wait is exact.
        const bool move = j == 0 || mx > m + kPfRescaleLog2;
        const float m_new = move ? fmaxf(m, mx) : m;
        const float alpha = exp2f(m - m_new);  // m = -inf on the first tile -> 0
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < kPfBN; ++c) {
          s[c] = exp2f(s[c] - m_new);
          sum += s[c];
        }
        l = l * alpha + sum;
        m = m_new;
        if (j > 0 && __any_sync(0xffffffffu, move)) {
          if (!mbar_wait(o_done, (jg - 1) & 1, a.error_flag, &abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            float o[32];
            tmem_ld32(lane_base + 128 + cc * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(lane_base + 128 + cc * 32, o);
          }
          tmem_wait_st();
        }
        store_p_row64(sK + st * kPfKVBytes, r, s);  // P(j) over K(j)
        // Keys from n_kv on get P = 0 in every row, but their V rows hold whatever the
        // cache pages hold past the sequence (never-written memory may be NaN or Inf, and
        // 0 * NaN poisons the row sums): clear those V rows of the last tile. Thread r owns
        // key t of d-half r >> 6.
        if (j == item.n_tiles - 1 && key0 + t >= item.n_kv) {
          fence_proxy_async_smem();  // after the tile's TMA bytes, before these stores
          uint4 *row = reinterpret_cast<uint4 *>(sV + st * kPfKVBytes + (r >> 6) * 8192 +
                                                 (t >> 3) * 1024 + (t & 7) * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) row[c] = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[st]);
      }
      if (!ok || !mbar_wait(o_last, it & 1, a.error_flag, &abort_flag)) break;
      tc_fence_after();
      float o[4][32];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld32(lane_base + 128 + cc * 32, o[cc]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(o_free);  // the next item's first P V may overwrite O
      if (t < item.nq) {
        const float inv = 1.f / l;
        __nv_bfloat16 *dst = a.out + static_cast<int64_t>(item.q0 + t) * a.out_stride + head * 128;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 v;
            v.x = pack2(o[cc][8 * i + 0] * inv, o[cc][8 * i + 1] * inv);
            v.y = pack2(o[cc][8 * i + 2] * inv, o[cc][8 * i + 3] * inv);
            v.z = pack2(o[cc][8 * i + 4] * inv, o[cc][8 * i + 5] * inv);
            v.w = pack2(o[cc][8 * i + 6] * inv, o[cc][8 * i + 7] * inv);
            *reinterpret_cast<uint4 *>(dst + cc * 32 + i * 8) = v;
          }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// =============================================================================
// Windowed bidirectional attention, head_dim 64, segments of at most 128 tokens.
// Work item = (segment, head): S = Q K^T (128x128, K=64), softmax over the whole row
// (no online rescaling needed), O = P V (128x64, K=128).
//
// Persistent pipeline: the grid is at most two CTAs per SM, and CTA c takes items c,
// c + grid, ... (item = segment * heads + head). TMEM (S in columns 0-127, O of items
// i & 1 in 128-191 / 192-255) and the barriers are set up once per CTA. Shared memory
// holds two (Q, K, V) buffers: the producer loads item i + 1 into one while item i
// computes from the other, the MMA warp issues S of item i + 1 as soon as the softmax has
// read S of item i out of TMEM, and P of item i (two 64-key K-major halves) is written
// over Q and K of its buffer once S is done (the buffer is refilled only after P V of
// item i). The softmax warps write item i's output after item i + 1's softmax, so P V
// of item i runs under that softmax instead of stalling the warps.
// =============================================================================

constexpr int kWinTile = 16384;                   // [128 rows x 128 B]
constexpr int kWinBuf = 3 * kWinTile;             // Q | K | V of one item
constexpr int kWinSmem = 1024 + 2 * kWinBuf + 256;

struct WindowArgs {
  const int32_t *cu_seqlens;
  int num_segments;
  int num_heads;
  float scale_log2;
  __nv_bfloat16 *out;
  int64_t out_stride;
  int32_t *error_flag;
};

// Rows and head of item `item`; false for an empty or over-long segment (skipped by every
// role alike, so all roles see the same sequence of items).
__device__ __forceinline__ bool window_item(const WindowArgs &a, int item, int &row0, int &len,
                                            int &head) {
  const int seg = item / a.num_heads;
  head = item - seg * a.num_heads;
  row0 = a.cu_seqlens[seg];
  len = a.cu_seqlens[seg + 1] - row0;
  return len > 0 && len <= 128;
}

__global__ void __launch_bounds__(kTcThreads, 2)
    varlen_window_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const WindowArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + 2 * kWinBuf);
  uint64_t *ld_full = bars;       // [2] item's Q, K, V landed in buffer b
  uint64_t *ld_empty = bars + 2;  // [2] buffer b free (P V of its item done)
  uint64_t *s_full = bars + 4;    // S in TMEM
  uint64_t *s_free = bars + 5;    // S read out by the softmax (128 arrivals)
  uint64_t *p_full = bars + 6;    // [2] P of item i written (128 arrivals), by i & 1
  uint64_t *o_full = bars + 8;    // [2] O of item i in TMEM
  uint64_t *o_free = bars + 10;   // [2] O of item i read out (128 arrivals)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 12);
  // meta[b] = {row0, len, head} of the item in buffer b, written by the producer before
  // the item's loads (published by ld_full[b]); len < 0 marks the end of the CTA's items.
  volatile int *meta = reinterpret_cast<volatile int *>(bars + 13);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int items = a.num_segments * a.num_heads;
  if (tid == 0) {
    abort_flag = 0;
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ld_full[b], 1);
      mbar_init(&ld_empty[b], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&p_full[b], 128);
      mbar_init(&o_full[b], 1);
      mbar_init(&o_free[b], 128);
    }
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    // The only role that reads the segment bounds from global memory: it runs ahead of
    // the others (loads of item i + 1 overlap item i), so those reads leave the chain.
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < items; item += gridDim.x) {
        int row0, len, head;
        if (!window_item(a, item, row0, len, head)) {
          if (len > 128) raise_flag(a.error_flag, B200ASR_DEVERR_LENGTH);
          continue;
        }
        const int b = it & 1;
        if (!mbar_wait(&ld_empty[b], ((it >> 1) & 1) ^ 1, a.error_flag, &abort_flag)) {
          ok = false;
          break;
        }
        meta[4 * b] = row0;
        meta[4 * b + 1] = len;
        meta[4 * b + 2] = head;
        uint8_t *buf = smem + b * kWinBuf;
        mbar_arrive_expect_tx(&ld_full[b], kWinBuf);
        tma_load_3d(buf, &tm_q, 0, head, row0, &ld_full[b]);
        tma_load_3d(buf + kWinTile, &tm_k, 0, head, row0, &ld_full[b]);
        tma_load_3d(buf + 2 * kWinTile, &tm_v, 0, head, row0, &ld_full[b]);
        ++it;
      }
      // end marker through the same pipeline: the next buffer's phase completes with no
      // bytes and len = -1
      const int b = it & 1;
      if (ok && mbar_wait(&ld_empty[b], ((it >> 1) & 1) ^ 1, a.error_flag, &abort_flag)) {
        meta[4 * b + 1] = -1;
        mbar_arrive(&ld_full[b]);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 64, false, true);
      const uint32_t base = smem_addr(smem);
      // S of item `it` (buffer it & 1) into TMEM columns 0-127; 0 at the end marker,
      // -1 on a timed-out wait
      auto issue_s = [&](uint32_t it) -> int {
        const uint32_t b = it & 1;
        if (!mbar_wait(&ld_full[b], (it >> 1) & 1, a.error_flag, &abort_flag)) return -1;
        if (meta[4 * b + 1] < 0) return 0;
        if (it > 0 && !mbar_wait(s_free, (it - 1) & 1, a.error_flag, &abort_flag)) return -1;
        tc_fence_after();
        const uint32_t qb = base + b * kWinBuf, kb = qb + kWinTile;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ss(tmem, smem_desc_sw128(qb + k * 32, 16, 1024),
                      smem_desc_sw128(kb + k * 32, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        return 1;
      };
      int have = issue_s(0);
      for (uint32_t it = 0; have > 0; ++it) {
        have = issue_s(it + 1);  // overlaps the softmax of item `it`
        if (have < 0) break;
        const int ob = it & 1;
        if (!mbar_wait(&p_full[ob], (it >> 1) & 1, a.error_flag, &abort_flag)) break;
        // O buffer ob last held item it - 2: its output must have been read
        if (it >= 2 && !mbar_wait(&o_free[ob], ((it - 2) >> 1) & 1, a.error_flag, &abort_flag)) break;
        tc_fence_after();
        const uint32_t pb = base + (it & 1) * kWinBuf;  // P over Q | K
        const uint32_t vb = pb + 2 * kWinTile;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_f16_ss(tmem + 128 + 64 * ob,
                      smem_desc_sw128(pb + (k >> 2) * kWinTile + (k & 3) * 32, 16, 1024),
                      smem_desc_sw128(vb + k * 2048, kWinTile, 1024), idesc_o, k > 0 ? 1u : 0u);
        umma_commit(&o_full[ob]);
        umma_commit(&ld_empty[it & 1]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int r = tid;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    // the previous item, whose output is written after this item's softmax
    int p_row0 = 0, p_len = 0, p_head = 0;
    float p_sum = 1.f;
    auto epilogue = [&](uint32_t pi) -> bool {
      const int ob = pi & 1;
      if (!mbar_wait(&o_full[ob], (pi >> 1) & 1, a.error_flag, &abort_flag)) return false;
      tc_fence_after();
      float o[64];
      tmem_ld32(lane_base + 128 + 64 * ob, o);
      tmem_ld32(lane_base + 160 + 64 * ob, o + 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&o_free[ob]);
      if (r < p_len) {
        const float inv = 1.f / p_sum;
        __nv_bfloat16 *dst = a.out + static_cast<int64_t>(p_row0 + r) * a.out_stride + p_head * 64;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint4 v;
          v.x = pack2(o[8 * i + 0] * inv, o[8 * i + 1] * inv);
          v.y = pack2(o[8 * i + 2] * inv, o[8 * i + 3] * inv);
          v.z = pack2(o[8 * i + 4] * inv, o[8 * i + 5] * inv);
          v.w = pack2(o[8 * i + 6] * inv, o[8 * i + 7] * inv);
          *reinterpret_cast<uint4 *>(dst + i * 8) = v;
        }
      }
      return true;
    };
    bool ended = false;
    uint32_t it = 0;
    for (;; ++it) {
      const int b = it & 1;
      // the item's bounds, published with its loads (the buffer cannot be refilled
      // before this item's P V, so the phase waited for is this item's)
      if (!mbar_wait(&ld_full[b], (it >> 1) & 1, a.error_flag, &abort_flag)) break;
      const int len = meta[4 * b + 1];
      if (len < 0) {
        ended = true;
        break;
      }
      const int row0 = meta[4 * b], head = meta[4 * b + 2];
      uint8_t *buf = smem + b * kWinBuf;
      if (!mbar_wait(s_full, it & 1, a.error_flag, &abort_flag)) break;
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld32(lane_base + cc * 32, s + cc * 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_free);  // the MMA warp may now compute S of the next item
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        s[c] = c < len ? s[c] * a.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        s[c] = exp2f(s[c] - mx);
        sum += s[c];
      }
      store_p_row64(buf, r, s);
      store_p_row64(buf + kWinTile, r, s + 64);
      // Keys from len on belong to other segments (or lie past the tensor): P = 0 there,
      // and their V rows are cleared so that a NaN or Inf outside the segment stays out
      // of it. Thread r owns key r.
      if (r >= len) {
        fence_proxy_async_smem();  // after the item's TMA bytes, before these stores
        uint4 *row = reinterpret_cast<uint4 *>(buf + 2 * kWinTile + (r >> 3) * 1024 + (r & 7) * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) row[c] = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[b]);
      if (it > 0 && !epilogue(it - 1)) break;
      p_row0 = row0;
      p_len = len;
      p_head = head;
      p_sum = sum;
    }
    if (ended && it > 0) epilogue(it - 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

int set_smem_attr(const void *fn, int bytes, const char *what) {
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_error("%s: cannot reserve %d bytes of shared memory: %s", what, bytes, cudaGetErrorString(e));
    return B200ASR_ERR_CUDA;
  }
  return B200ASR_OK;
}

}  // namespace b200asr

using namespace b200asr;

extern "C" int b200asr_paged_prefill(const void *q, int64_t q_row_stride, const void *k_cache,
                                     const void *v_cache, int32_t num_blocks, int32_t block_size,
                                     int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                     const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                                     const int32_t *block_tables, int32_t bt_stride, int32_t batch,
                                     int32_t total_q, int32_t max_seqlen_q, float scale, void *out,
                                     int64_t out_row_stride, int32_t *error_flag,
                                     b200asr_stream_t stream) {
  B200_REQUIRE(head_dim == 128, "paged_prefill: head_dim %d unsupported (needs 128)", head_dim);
  B200_REQUIRE(num_kv_heads >= 1 && num_heads == 2 * num_kv_heads,
               "paged_prefill: needs num_heads == 2 * num_kv_heads (got %d / %d)", num_heads,
               num_kv_heads);
  B200_REQUIRE(batch >= 0 && total_q >= 0, "paged_prefill: bad sizes");
  if (batch == 0 || total_q == 0) return B200ASR_OK;
  B200_REQUIRE(block_size >= 64 && block_size % 64 == 0,
               "paged_prefill: block_size %d must be a multiple of 64", block_size);
  B200_REQUIRE(q && k_cache && v_cache && cu_seqlens_q && cu_seqlens_k && block_tables && out,
               "paged_prefill: null pointer");
  B200_REQUIRE(aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out) &&
                   q_row_stride % 8 == 0 && out_row_stride % 8 == 0,
               "paged_prefill: tensors and row strides must be 16-byte aligned");
  CUtensorMap tq, tk, tv;
  const uint64_t slots = static_cast<uint64_t>(num_blocks) * block_size;
  if (!make_tmap_3d_bf16(&tq, q, 128, num_heads, total_q, 256, q_row_stride * 2, 64, 1, 64) ||
      !make_tmap_3d_bf16(&tk, k_cache, 128, num_kv_heads, slots, 256, num_kv_heads * 256ull, 64, 1, 64) ||
      !make_tmap_3d_bf16(&tv, v_cache, 128, num_kv_heads, slots, 256, num_kv_heads * 256ull, 64, 1, 64))
    return B200ASR_ERR_CUDA;
  static bool configured = false;
  if (!configured) {
    int rc = set_smem_attr(reinterpret_cast<const void *>(paged_prefill_kernel), kPfSmem,
                           "paged_prefill");
    if (rc) return rc;
    configured = true;
  }
  PrefillArgs a{};
  a.cu_seqlens_q = cu_seqlens_q;
  a.cu_seqlens_k = cu_seqlens_k;
  a.block_tables = block_tables;
  a.bt_stride = bt_stride;
  a.batch = batch;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.num_kv_heads = num_kv_heads;
  a.scale_log2 = scale * kTcLog2e;
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.out_stride = out_row_stride;
  a.error_flag = error_flag;
  (void)max_seqlen_q;
  const int64_t tiles = static_cast<int64_t>(total_q) / 64 + batch;  // >= sum of ceil(q_len / 64)
  B200_REQUIRE(tiles * num_kv_heads < (int64_t{1} << 31), "paged_prefill: too many query tiles");
  a.items = static_cast<int>(tiles * num_kv_heads);
  const int grid = static_cast<int>(std::min<int64_t>(a.items, 2 * num_sms()));
  paged_prefill_kernel<<<grid, kTcThreads, kPfSmem, stream>>>(tq, tk, tv, a);
  B200_CUDA_LAUNCH_CHECK("paged_prefill");
  return B200ASR_OK;
}

extern "C" int b200asr_varlen_attention(const void *q, int64_t q_row_stride, const void *k,
                                        int64_t k_row_stride, const void *v, int64_t v_row_stride,
                                        const int32_t *cu_seqlens, int32_t num_segments,
                                        int32_t total_tokens, int32_t max_seqlen, int32_t num_heads,
                                        int32_t head_dim, float scale, void *out,
                                        int64_t out_row_stride, int32_t *error_flag,
                                        b200asr_stream_t stream) {
  B200_REQUIRE(head_dim == 64, "varlen_attention: head_dim %d unsupported (needs 64)", head_dim);
  B200_REQUIRE(max_seqlen <= 128, "varlen_attention: segments up to 128 tokens (got %d)", max_seqlen);
  B200_REQUIRE(num_segments >= 0 && total_tokens >= 0 && num_heads >= 1, "varlen_attention: bad sizes");
  if (num_segments == 0 || total_tokens == 0) return B200ASR_OK;
  B200_REQUIRE(q && k && v && cu_seqlens && out, "varlen_attention: null pointer");
  B200_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) &&
                   q_row_stride % 8 == 0 && k_row_stride % 8 == 0 && v_row_stride % 8 == 0 &&
                   out_row_stride % 8 == 0,
               "varlen_attention: tensors and row strides must be 16-byte aligned");
  B200_REQUIRE(static_cast<int64_t>(num_segments) * num_heads <= 0x7fffffff,
               "varlen_attention: too many (segment, head) items");
  CUtensorMap tq, tk, tv;
  if (!make_tmap_3d_bf16(&tq, q, 64, num_heads, total_tokens, 128, q_row_stride * 2, 64, 1, 128) ||
      !make_tmap_3d_bf16(&tk, k, 64, num_heads, total_tokens, 128, k_row_stride * 2, 64, 1, 128) ||
      !make_tmap_3d_bf16(&tv, v, 64, num_heads, total_tokens, 128, v_row_stride * 2, 64, 1, 128))
    return B200ASR_ERR_CUDA;
  static bool configured = false;
  if (!configured) {
    int rc = set_smem_attr(reinterpret_cast<const void *>(varlen_window_kernel), kWinSmem,
                           "varlen_attention");
    if (rc) return rc;
    configured = true;
  }
  WindowArgs a{};
  a.cu_seqlens = cu_seqlens;
  a.num_segments = num_segments;
  a.num_heads = num_heads;
  a.scale_log2 = scale * kTcLog2e;
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.out_stride = out_row_stride;
  a.error_flag = error_flag;
  const int64_t items = static_cast<int64_t>(num_segments) * num_heads;
  const int grid = static_cast<int>(std::min<int64_t>(items, 2 * num_sms()));
  varlen_window_kernel<<<grid, kTcThreads, kWinSmem, stream>>>(tq, tk, tv, a);
  B200_CUDA_LAUNCH_CHECK("varlen_attention");
  return B200ASR_OK;
}
