// Sparse FlashAttention forward kernel (tcgen05 + TMA) and its host launcher.
// Design notes are at the top of attention.cuh.
#include "attention.cuh"
#include <cstring>

#include "host_util.h"

namespace mib200 {

// Lazy rescale: O and P stay relative to a running max m_used until a row's
// max exceeds it by more than 2^MI_RESCALE_LOG2 (P then stays below that
// power of two: representable in fp16 and bf16).
#ifndef MI_RESCALE_LOG2
#define MI_RESCALE_LOG2 12.0f
#endif

#ifdef MI_TRACE
// Debug builds only: (clock64, %globaltimer ns) at the first and the last
// softmax iteration of the traced CTA, for the effective SM clock.
__device__ unsigned long long g_trace_gt[8];  // [4..7]: kernel entry, setup done, loop done, exit
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Debug builds only (-DMI_TRACE): clock64 timeline of the CTA with blockIdx
// (0,0,0), [event][entry], read back with mi_debug_trace().
__device__ unsigned long long g_trace[10][4096];
#define MI_TR(ev, j) \
  do { if (trace_cta && (j) < 4096) g_trace[ev][j] = clock64(); } while (0)
#else
#define MI_TR(ev, j) do { } while (0)
#endif


// Softmax of one 64-key block for one query row, in registers.
// s: raw scores (overwritten).  Returns the block max of raw visible scores.
struct RowState {
  float m_used;  // running max (log2 domain) the current P and O are relative to
  float l;       // running sum of P
};

// SPLIT (block_sparse plans): each entry carries one key block per 64-row
// half of the tile.  S and O of the two halves are computed by two M=64 MMAs
// whose accumulators interleave in TMEM: the M=64 layout puts row m of the
// MMA at lane (m % 16) + 32 * (m / 16), and the second MMA, addressed at lane
// 16, fills the other 16 lanes of every 32-lane quadrant.  Query row r of
// the tile therefore sits at a lane where each quadrant holds 16 rows of
// each half; softmax thread L owns row split_row(L).
__device__ __forceinline__ int split_row(int L) {
  return ((L & 31) < 16) ? (L >> 5) * 16 + (L & 15) : 64 + (L >> 5) * 16 + (L & 15);
}

#ifndef MI_PLAN_AHEAD
#define MI_PLAN_AHEAD 1
#endif
template <typename DT, int D, bool SPLIT, bool GATHER>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_o,
                    const __grid_constant__ CUtensorMap tm_kr,
                    const __grid_constant__ CUtensorMap tm_vr,
                    const __grid_constant__ ReplicaMaps tm_rep, const AttnParams p) {
  using L = AttnSmem<D, SPLIT>;
  constexpr int NC = L::NC;
  constexpr int KS = L::KS, VS = L::VS;
  constexpr bool kBF16 = DType<DT>::kBF16;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* q_tmem = pv_done + 2;  // the softmax warps staged Q's first KQ dims in TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlotOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbortOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int t = p.t_lo + p.t_n - 1 - blockIdx.x;  // heavy (late) tiles first
  const int h = blockIdx.y;  // head of the call (plan and workspace index)
  const int b = blockIdx.z;
  const int bh = b * p.H + h;
  const int hv = p.head_index ? p.head_index[h] : h;  // head of the q/k/v/out views
#ifdef MI_TRACE
#ifndef MI_TRACE_HEAD
#define MI_TRACE_HEAD 0  // head whose heaviest tile is traced
#endif
  const bool trace_cta = blockIdx.x == 0 && blockIdx.y == MI_TRACE_HEAD && blockIdx.z == 0 &&
                         (threadIdx.x == 0 || threadIdx.x == 160);
  if (trace_cta && threadIdx.x == 0) g_trace_gt[4] = clock64();
#endif

  // ---- entry list of this tile -------------------------------------------
  EntrySource src;
  src.mode = p.mode;
  const int32_t* gcols = nullptr;  // gathered key positions of this tile
  int n_entries;
  if (p.mode == 0) {
    const long long a_lo = (long long)p.q_off + (long long)t * kBM;
    const long long last_row = min((long long)t * kBM + kBM - 1, (long long)p.Sq - 1);
    const long long a_hi = (long long)p.q_off + last_row;
    const long long key_hi = min(a_hi, (long long)p.Sk - 1);
    const int hi = (int)(key_hi / kBN);
    const long long sink_keys = min(p.n_init, key_hi + 1);
    const int nsb = sink_keys > 0 ? (int)((sink_keys + kBN - 1) / kBN) : 0;
    long long band_lo_key = a_lo - p.n_local + 1;
    if (band_lo_key < 0) band_lo_key = 0;
    const int band_lo = (int)(band_lo_key / kBN);
    const int band_start = max(band_lo, nsb);
    const int nband = (band_lo_key > key_hi) ? 0 : max(0, hi - band_start + 1);
    src.nsb = nsb;
    src.band_start = band_start;
    src.list = nullptr;
    n_entries = nsb + nband;
  } else {
    src.nsb = 0;
    src.band_start = 0;
    src.list = p.plan + (long long)bh * p.plan_head_stride + plan_offset(t, p.plan_cap);
    n_entries = p.plan_count[(long long)bh * p.T + t];
    if (GATHER) gcols = p.gcols + ((long long)bh * p.T + t) * p.gmax * 64;
  }

  // ---- one-time setup -------------------------------------------------------
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kBM);
      mbar_init(&pv_done[i], 1);
      if (i == 0) mbar_init(q_tmem, kBM);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // Constant chunk NC of every V stage: column 0 = 1, other columns 0 (64-byte
  // swizzled like the TMA-loaded chunks).  TMA never writes it.
  for (int i = threadIdx.x; i < VS * L::NB * kBN * 4; i += kThreads) {
    const int st = i / (kBN * 4), r = (i >> 2) % kBN, lu = i & 3;  // st: block slot of the V ring
    const uint16_t one = DType<DT>::kBF16 ? (uint16_t)0x3F80 : (uint16_t)0x3C00;
    const uint4 val = make_uint4(lu == 0 ? (uint32_t)one : 0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(smem + L::kVOff + st * L::kVBytes + NC * (kBN * 64) + r * 64 +
                              ((lu ^ ((r >> 1) & 3)) << 4)) = val;
  }
  fence_proxy_async_smem();
  if (warp == 5) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
#ifdef MI_TRACE
  if (trace_cta && threadIdx.x == 0) g_trace_gt[5] = clock64();
#endif

  if (warp == 4) {
    // ======================= TMA producer (one thread) =========================
    // Fixed order K0, K1, V0, K2, V1, ...: K runs one block ahead of V, and
    // each ring slot is reused once the MMA that read it has completed.
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      if (GATHER) {
        tma_prefetch_desc(&tm_kr);
        tma_prefetch_desc(&tm_vr);
      }
      mbar_arrive_expect_tx(q_full, L::kQBytes);
      for (int c = 0; c < NC; ++c)
        tma_load_4d(smem + L::kQOff + c * (kBM * 64), &tm_q, q_full, c * 32, t * kBM, hv, b);
      // A stage holds one key block per entry, or two in a split tile
      // (the block of query rows [0,64), then the block of rows [64,128)).
      // A gathered group (kb < 0; GATHER kernels only) loads its up to 64 key
      // rows four at a time through the 2-D row view; empty slots load key 0
      // of the head, which the group's masks leave invisible.
      const long long row0 = (long long)b * p.grow_b + (long long)hv * p.grow_h;
      auto gather_rows = [&](uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int g) {
        const int4* cols = reinterpret_cast<const int4*>(gcols + g * 64);
        // all 16 loads first: the TMA issues below are ordered memory
        // operations, so a load placed between them would wait out its full
        // latency before the next issue
        int4 cv[kBN / 4];
#pragma unroll
        for (int rg = 0; rg < kBN / 4; ++rg) cv[rg] = cols[rg];
#pragma unroll
        for (int rg = 0; rg < kBN / 4; ++rg) {
          const int4 c = cv[rg];
          const int r0 = (int)(row0 + max(c.x, 0)), r1 = (int)(row0 + max(c.y, 0));
          const int r2 = (int)(row0 + max(c.z, 0)), r3 = (int)(row0 + max(c.w, 0));
          for (int cc = 0; cc < NC; ++cc)
            tma_gather4_2d(dst + cc * (kBN * 64) + rg * 256, map, bar, cc * 32, r0, r1, r2, r3);
        }
      };
      // Key blocks of the entries, read kAhead entries before they are needed
      // (a plan entry is a global load; read at the point of use its latency
      // would stall every load issue).
      constexpr int kAhead = MI_PLAN_AHEAD;
      int2 ahead[kAhead + 1];  // entries j-1 .. j+kAhead-1 of the current step
      auto fetch = [&](int j) -> int2 {
        int2 r = make_int2(0, 0);
        if (j >= 0 && j < n_entries) {
          uint64_t m0, m1;
          src.get(j, r.x, r.y, m0, m1);
        }
        return r;
      };
#pragma unroll
      for (int i = 0; i <= kAhead; ++i) ahead[i] = fetch(i - 1);
      auto load_k = [&](int j, int2 e) -> bool {
        const int st = j % KS, use = j / KS;
        if (use > 0 && !mbar_wait(&k_empty[st], (use - 1) & 1, 101)) return false;
        const int kb[2] = {e.x, e.y};
        uint8_t* dst = smem + L::kKOff + st * L::kKStage;
        mbar_arrive_expect_tx(&k_full[st], L::kKStage);
        if (GATHER && kb[0] < 0) {
          gather_rows(dst, &tm_kr, &k_full[st], -1 - kb[0]);
          return true;
        }
        for (int hb = 0; hb < L::NB; ++hb)
          for (int c = 0; c < NC; ++c)
            tma_load_4d(dst + hb * L::kKVBytes + c * (kBN * 64), &tm_k, &k_full[st], c * 32,
                        kb[hb] * kBN, hv, b);
        return true;
      };
      auto load_v = [&](int j, int2 e) -> bool {
        const int st = j % VS, use = j / VS;
        if (use > 0 && !mbar_wait(&v_empty[st], (use - 1) & 1, 103)) return false;
        const int kb[2] = {e.x, e.y};
        uint8_t* dst = smem + L::kVOff + st * L::kVStage;
        mbar_arrive_expect_tx(&v_full[st], L::NB * L::kKVBytes);
        if (GATHER && kb[0] < 0) {
          gather_rows(dst, &tm_vr, &v_full[st], -1 - kb[0]);
          return true;
        }
        for (int hb = 0; hb < L::NB; ++hb)
          for (int c = 0; c < NC; ++c)
            tma_load_4d(dst + hb * L::kVBytes + c * (kBN * 64), &tm_v, &v_full[st], c * 32,
                        kb[hb] * kBN, hv, b);
        return true;
      };
      bool ok = true;
      for (int j = 0; ok && j < n_entries; ++j) {
        if (*abort_flag) break;
        ok = load_k(j, ahead[1]);
        if (ok && j >= 1) ok = load_v(j - 1, ahead[0]);
#pragma unroll
        for (int i = 0; i < kAhead; ++i) ahead[i] = ahead[i + 1];
        ahead[kAhead] = fetch(j + kAhead);
      }
      if (ok && n_entries > 0 && !*abort_flag) ok = load_v(n_entries - 1, ahead[0]);
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 5) {
    // ======================= MMA issuer (whole warp) ===========================
    // The warp runs converged and an elected lane issues: a tcgen05.mma issue
    // takes about as long as the MMA, so every wait and branch between MMAs
    // is tensor-pipe idle time, and a lone lane in a divergent branch issues
    // at about half the converged rate.
    // Split tiles: two M=64 MMAs per step; the second (query rows [64,128),
    // its own key block) accumulates at TMEM lane 16.
    constexpr int kM = SPLIT ? 64 : kBM;
    constexpr uint32_t idesc_qk = make_idesc_f16(kBF16, kM, kBN, false, false);
    constexpr uint32_t idesc_pv = make_idesc_f16(kBF16, kM, L::kOCols, false, true);
    constexpr uint32_t kLane16 = 16u << 16;
    const uint64_t qd0 = make_desc_sw64(smem_u32(smem + L::kQOff), 16, 512);
    const uint64_t kd0 = make_desc_sw64(smem_u32(smem + L::kKOff), 16, 512);
    const uint64_t vd0 = make_desc_sw64(smem_u32(smem + L::kVOff), kBN * 64, 512);
    const uint32_t tmem_o = tmem_base + 128;

    auto issue_qk = [&](int j) -> bool {
      const int st = j % KS;
      if (!__all_sync(0xffffffffu, mbar_wait(&k_full[st], (j / KS) & 1, 104))) return false;
      tc_fence_after();
      MI_TR(9, j);
      if (elect_one_sync()) {
        const uint64_t kd = kd0 + (uint64_t)((st * L::kKStage) >> 4);
        const uint32_t tmem_s = tmem_base + (j & 1) * kBN;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t koff = (ks & 1) * 32;
          const uint64_t qd = qd0 + (((ks >> 1) * (kBM * 64) + koff) >> 4);
          const uint64_t kdk = kd + (((ks >> 1) * (kBN * 64) + koff) >> 4);
          if (ks < L::KQ / 16) {  // A = Q from TMEM (staged by the softmax warps)
            const uint32_t tq = tmem_base + L::kQCol + ks * 8;
            umma_f16_ts(tmem_s, tq, kdk, idesc_qk, ks > 0 ? 1u : 0u);
            if constexpr (SPLIT)
              umma_f16_ts(tmem_s + kLane16, tq + kLane16, kdk + (L::kKVBytes >> 4), idesc_qk,
                          ks > 0 ? 1u : 0u);
          } else {
            umma_f16_ss(tmem_s, qd, kdk, idesc_qk, ks > 0 ? 1u : 0u);
            if constexpr (SPLIT)  // Q rows [64,128) start 64 rows (4096 B) into each chunk
              umma_f16_ss(tmem_s + kLane16, qd + ((64 * 64) >> 4), kdk + (L::kKVBytes >> 4),
                          idesc_qk, ks > 0 ? 1u : 0u);
          }
        }
        umma_commit(&s_full[j & 1]);
        umma_commit(&k_empty[st]);
      }
      __syncwarp();
      MI_TR(5, j);
      return true;
    };
    bool ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0, 102) && mbar_wait(q_tmem, 0, 111));
    if (ok && n_entries > 0) ok = issue_qk(0);
    for (int j = 0; ok && j < n_entries; ++j) {
      if (*abort_flag) { ok = false; break; }
      // S buffer (j+1)&1 last held P(j-1), consumed by PV(j-1), issued earlier by this
      // warp: tcgen05.mma from one thread execute in issue order.
      if (j + 1 < n_entries && !issue_qk(j + 1)) { ok = false; break; }
      const int st = j % VS;
      if (!__all_sync(0xffffffffu, mbar_wait(&p_full[j & 1], (j >> 1) & 1, 105))) { ok = false; break; }
      MI_TR(6, j);
      if (!__all_sync(0xffffffffu, mbar_wait(&v_full[st], (j / VS) & 1, 106))) { ok = false; break; }
      tc_fence_after();
      MI_TR(8, j);
      if (elect_one_sync()) {
        const uint64_t vd = vd0 + (uint64_t)((st * L::kVStage) >> 4);
        const uint32_t tmem_p = tmem_base + (j & 1) * kBN;
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks) {
          const uint64_t vdk = vd + (uint64_t)((ks * 1024) >> 4);
          umma_f16_ts(tmem_o, tmem_p + ks * 8, vdk, idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
          if constexpr (SPLIT)  // P and O of rows [64,128) at lane 16; their V block second
            umma_f16_ts(tmem_o + kLane16, tmem_p + kLane16 + ks * 8, vdk + (L::kVBytes >> 4),
                        idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[j & 1]);
        umma_commit(&v_empty[st]);
      }
      __syncwarp();
      MI_TR(7, j);
    }
    if (!ok && lane == 0) *abort_flag = 1;
  } else {
    // ======================= softmax warps 0-3 ================================
    // Thread = TMEM lane; the query row it owns (identity unless SPLIT).
    const int row = SPLIT ? split_row(threadIdx.x) : threadIdx.x;
    const uint32_t lane_base = tmem_base + ((uint32_t)(warp * 32) << 16);
    const long long a = (long long)p.q_off + (long long)t * kBM + row;  // absolute position
    // Lowest and highest absolute positions among the warp's 32 rows.
    const long long tile_a0 = (long long)p.q_off + (long long)t * kBM;
    const long long a_w0 = SPLIT ? tile_a0 + warp * 16 : a - lane;
    const long long a_w1 = SPLIT ? tile_a0 + 64 + warp * 16 + 15 : a - lane + 31;
    const float NEG_INF = -INFINITY;
    const float sc = p.scale_log2;
    float m_used = NEG_INF;
    bool ok = true;

    // Stage this row's first KQ dims of Q in this thread's TMEM lane (the
    // A operand of the first KQ/16 QK K-steps).  Shared-memory Q is 64-byte
    // swizzled: 16-byte unit u of row r in chunk c sits at unit u ^ ((r>>1)&3).
    if (mbar_wait(q_full, 0, 112)) {
      const uint8_t* qrow = smem + L::kQOff + row * 64;
      const uint32_t sw = (row >> 1) & 3;
#pragma unroll
      for (int c = 0; c < L::KQ / 32; ++c) {
        uint32_t w[16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 x = *reinterpret_cast<const uint4*>(qrow + c * (kBM * 64) + ((u ^ sw) << 4));
          w[4 * u + 0] = x.x;
          w[4 * u + 1] = x.y;
          w[4 * u + 2] = x.z;
          w[4 * u + 3] = x.w;
        }
        tmem_st16u(lane_base + L::kQCol + c * 16, w);
      }
      tmem_wait_st();
    } else {
      ok = false;
    }
    tc_fence_before();
    mbar_arrive(q_tmem);

    int kb_n = 0, kb1_n = 0;
    uint64_t m0_n = 0, m1_n = 0;
    if (n_entries > 0) src.get(0, kb_n, kb1_n, m0_n, m1_n);
    for (int j = 0; ok && j < n_entries; ++j) {
      const int kb = (row < 64) ? kb_n : kb1_n;  // this row's key block
      const int kb_lo = min(kb_n, kb1_n), kb_hi = max(kb_n, kb1_n);
      const uint64_t mask = (row < 64) ? m0_n : m1_n;
      const bool masks_full = (m0_n & m1_n) == ~0ull;
      if (j + 1 < n_entries) src.get(j + 1, kb_n, kb1_n, m0_n, m1_n);  // prefetch next entry

      MI_TR(0, j);
#ifdef MI_TRACE
      if (trace_cta && threadIdx.x == 0 && (j == 0 || j == n_entries - 1)) {
        g_trace_gt[j == 0 ? 0 : 2] = clock64();
        g_trace_gt[j == 0 ? 1 : 3] = globaltimer_ns();
      }
#endif
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, 107)) { ok = false; break; }
      tc_fence_after();
      MI_TR(1, j);

      // A gathered group has kb < 0, so key0 <= -64: with n_init = 0 and the
      // unbounded n_local of mode 1 every positional term below is all ones
      // and its visibility is its mask alone.
      const long long key0 = (long long)kb * kBN;
      // Visible keys of this row inside the block:
      //   mask AND key <= a AND key < Sk AND (key < n_init OR key > a - n_local).
      // Warp-uniform shortcut for blocks wholly visible to the warp's 32 rows
      // (evaluated on both halves' masks and key blocks, so it is uniform in
      // split tiles too, where a warp holds rows of both halves).
      const long long klo = (long long)kb_lo * kBN, khi = (long long)kb_hi * kBN;
      const bool fast_full = masks_full && khi + kBN - 1 <= a_w0 && khi + kBN - 1 < p.Sk &&
                             (klo > a_w1 - p.n_local || khi + kBN - 1 < p.n_init);
      uint64_t vis = ~0ull;
      bool all_full = true, all_empty = false;
      if (!fast_full) {
        vis = mask & bits_below(a - key0 + 1) & bits_below((long long)p.Sk - key0) &
              (bits_below(p.n_init - key0) | ~bits_below(a - p.n_local - key0 + 1));
        all_full = __all_sync(0xffffffffu, vis == ~0ull);
        all_empty = __all_sync(0xffffffffu, vis == 0ull);
      }
      const uint32_t tmem_s = lane_base + (j & 1) * kBN;

      float s[kBN];
      if (!all_empty) {
        tmem_ld32(tmem_s, *reinterpret_cast<float(*)[32]>(&s[0]));
        tmem_ld32(tmem_s + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
        tmem_wait_ld();
        if (!all_full) {
#pragma unroll
          for (int c = 0; c < kBN; ++c) s[c] = ((vis >> c) & 1ull) ? s[c] : NEG_INF;
        }
      }
      auto row_max = [&]() -> float {
        float mx0 = fmax3(s[0], s[1], s[2]);
        float mx1 = fmax3(s[3], s[4], s[5]);
        float mx2 = fmax3(s[6], s[7], s[8]);
        float mx3 = fmax3(s[9], s[10], s[11]);
#pragma unroll
        for (int c = 12; c < 60; c += 8) {
          mx0 = fmax3(mx0, s[c], s[c + 1]);
          mx1 = fmax3(mx1, s[c + 2], s[c + 3]);
          mx2 = fmax3(mx2, s[c + 4], s[c + 5]);
          mx3 = fmax3(mx3, s[c + 6], s[c + 7]);
        }
        return fmaxf(fmax3(mx0, mx1, fmax3(s[60], s[61], s[62])), fmax3(mx2, mx3, s[63]));
      };
      // P = 2^(s*scale_log2 - m_used), packed in pairs.
      uint32_t pk[kBN / 2];
      auto exp_block = [&](float nm) {
#pragma unroll
        for (int c = 0; c < kBN / 2; ++c) {
          const float x0 = __fmaf_rn(s[2 * c], sc, nm);
          const float x1 = __fmaf_rn(s[2 * c + 1], sc, nm);
          pk[c] = DType<DT>::pack2(fast_exp2(x0), fast_exp2(x1));
        }
      };
      // With the lazy rescale, P is relative to the running max m_used, which
      // rarely moves after the first blocks.  So P is computed against m_used
      // straight away, with the block max taken alongside (ALU work that
      // overlaps the MUFU exp2) instead of before it; only if some row's max
      // grew past the threshold does the warp rescale O and recompute P.  The
      // result is the same as computing the max first.
      const bool spec = j > 0 && !all_empty && __all_sync(0xffffffffu, m_used != NEG_INF);
      float tmax = NEG_INF;
      if (spec) {
        exp_block(-m_used);
        tmax = row_max();
      } else if (!all_empty) {
        tmax = row_max();
      }
      MI_TR(2, j);
      const float m_new = fmaxf(m_used, tmax * sc);
      const bool need = m_new > m_used + MI_RESCALE_LOG2;
      bool fresh = !spec;  // P still to be computed (or recomputed)
      if (j == 0) {
        m_used = m_new;
      } else if (__any_sync(0xffffffffu, need)) {
        // O must hold PV(j-1) before it is rescaled.
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, 108)) { ok = false; break; }
        tc_fence_after();
        const float f = need ? ((m_used == NEG_INF) ? 0.f : fast_exp2(m_used - m_new)) : 1.f;
#pragma unroll
        for (int c = 0; c < L::kOCols / 16; ++c) {
          float o[16];
          tmem_ld16(lane_base + 128 + c * 16, o);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 16; ++x) o[x] *= f;
          tmem_st16(lane_base + 128 + c * 16, o);
        }
        tmem_wait_st();
        if (need) m_used = m_new;
        fresh = true;
      }
      // Rows with nothing visible yet keep P = 0.  The row sums of P come out
      // of the PV MMA (column D of O).
      if (fresh) {
        if (all_empty || m_used == NEG_INF) {
#pragma unroll
          for (int c = 0; c < kBN / 2; ++c) pk[c] = 0u;
        } else {
          exp_block(-m_used);
        }
      }
      MI_TR(3, j);
      // P(j) overwrites the first 32 columns of S buffer (j & 1).
      tmem_st32u(tmem_s, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
      MI_TR(4, j);
    }

#ifdef MI_TRACE
    if (trace_cta && threadIdx.x == 0) g_trace_gt[6] = clock64();
#endif
    // ---- epilogue: O / l -> shared (Q tile area, swizzled) -> TMA store -----
    if (!ok) *abort_flag = 1;
    bool have_o = false;
    float o[D];
    float l = 0.f;
    if (ok && n_entries > 0) {
      const int jl = n_entries - 1;
      if (mbar_wait(&pv_done[jl & 1], (jl >> 1) & 1, 109)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          tmem_ld32(lane_base + 128 + c * 32, *reinterpret_cast<float(*)[32]>(&o[c * 32]));
        float lc[16];
        tmem_ld16(lane_base + 128 + D, lc);
        tmem_wait_ld();
        l = lc[0];
        have_o = true;
      } else {
        ok = false;
      }
    } else if (ok) {
      ok = mbar_wait(q_full, 0, 110);  // the Q tile area must be idle before reuse
    }
    if (!ok) *abort_flag = 1;
    const float inv = (have_o && l > 0.f) ? 1.f / l : 0.f;
    const uint32_t sw = (row >> 1) & 3;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = c * 32 + u * 8;
        uint4 val;
        val.x = DType<DT>::pack2(have_o ? o[e + 0] * inv : 0.f, have_o ? o[e + 1] * inv : 0.f);
        val.y = DType<DT>::pack2(have_o ? o[e + 2] * inv : 0.f, have_o ? o[e + 3] * inv : 0.f);
        val.z = DType<DT>::pack2(have_o ? o[e + 4] * inv : 0.f, have_o ? o[e + 5] * inv : 0.f);
        val.w = DType<DT>::pack2(have_o ? o[e + 6] * inv : 0.f, have_o ? o[e + 7] * inv : 0.f);
        *reinterpret_cast<uint4*>(smem + L::kQOff + c * (kBM * 64) + row * 64 + ((u ^ sw) << 4)) =
            val;
      }
    }
    fence_proxy_async_smem();
    named_barrier(1, kBM);
    if (row == 0 && !*abort_flag) {
      for (int c = 0; c < NC; ++c)
        tma_store_4d(&tm_o, smem + L::kQOff + c * (kBM * 64), c * 32, t * kBM, hv, b);
      // the same tile into every output replica (e.g. the peers' buffers)
      for (int r = 0; r < p.n_replica; ++r)
        for (int c = 0; c < NC; ++c)
          tma_store_4d(&tm_rep.m[r], smem + L::kQOff + c * (kBM * 64), c * 32, t * kBM, hv, b);
      bulk_commit();
      bulk_wait_read0();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
#ifdef MI_TRACE
  if (trace_cta && threadIdx.x == 0) g_trace_gt[7] = clock64();
#endif
}

// ---------------------------------------------------------------------------
// Host launcher
// ---------------------------------------------------------------------------
template <typename DT, int D, bool SPLIT, bool GATHER>
static int launch_attn_t(const mi_tensor4& q, const mi_tensor4& k, const mi_tensor4& v,
                         const mi_tensor4& out, AttnParams prm, cudaStream_t stream) {
  using L = AttnSmem<D, SPLIT>;
  CUtensorMap tq, tk, tv, to;
  int rc;
  if ((rc = make_bnsd_map(&tq, q, prm.B, prm.H, prm.Sq, D, 32, kBM)) != MI_OK) return rc;
  if ((rc = make_bnsd_map(&tk, k, prm.B, prm.H, prm.Sk, D, 32, kBN)) != MI_OK) return rc;
  if ((rc = make_bnsd_map(&tv, v, prm.B, prm.H, prm.Sk, D, 32, kBN)) != MI_OK) return rc;
  if ((rc = make_bnsd_map(&to, out, prm.B, prm.H, prm.Sq, D, 32, kBM)) != MI_OK) return rc;
  CUtensorMap tkr, tvr;  // 2-D row views of K and V (gathered groups only)
  memset(&tkr, 0, sizeof(tkr));
  memset(&tvr, 0, sizeof(tvr));
  if (GATHER) {
    const long long nh = k.head_index ? k.head_extent : prm.H;
    const long long rows = (long long)(prm.B - 1) * prm.grow_b + (nh - 1) * prm.grow_h + prm.Sk;
    if ((rc = make_rows_map(&tkr, k.ptr, rows, k.stride_s, D, 32)) != MI_OK) return rc;
    if ((rc = make_rows_map(&tvr, v.ptr, rows, v.stride_s, D, 32)) != MI_OK) return rc;
  }
  ReplicaMaps trep;
  memset(&trep, 0, sizeof(trep));
  for (int r = 0; r < prm.n_replica; ++r) {
    mi_tensor4 o = out;
    o.ptr = out.replica[r];
    if ((rc = make_bnsd_map(&trep.m[r], o, prm.B, prm.H, prm.Sq, D, 32, kBM)) != MI_OK) return rc;
  }
  auto kern = attn_fwd_kernel<DT, D, SPLIT, GATHER>;
  const int alloc = L::kAlloc;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, alloc);
  if (e == cudaSuccess) {
    dim3 grid(prm.t_n, prm.H, prm.B);
    kern<<<grid, kThreads, alloc, stream>>>(tq, tk, tv, to, tkr, tvr, trep, prm);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    debug_launch_failure("attn_fwd_kernel", reinterpret_cast<const void*>(kern), e, kThreads,
                         alloc);
    return MI_ERR_LAUNCH;
  }
  return MI_OK;
}

int launch_attention(const mi_tensor4& q, const mi_tensor4& k, const mi_tensor4& v,
                     const mi_tensor4& out, int64_t D, int dtype, AttnParams prm,
                     cudaStream_t stream) {
  // one head table for q, k, v and out (see mi_tensor4)
  if (k.head_index != q.head_index || v.head_index != q.head_index ||
      out.head_index != q.head_index)
    return MI_ERR_SHAPE;
  prm.head_index = q.head_index;
  if (out.n_replica < 0 || out.n_replica > MI_MAX_REPLICAS ||
      (out.n_replica > 0 && !out.replica))
    return MI_ERR_SHAPE;
  prm.n_replica = (int)out.n_replica;
  prm.out = out.ptr;
  prm.os_b = out.stride_b;
  prm.os_h = out.stride_h;
  prm.os_s = out.stride_s;
  if (prm.t_n == 0 && prm.t_lo == 0) prm.t_n = prm.T;  // default: every tile
  if (prm.t_lo < 0 || prm.t_n < 0 || prm.t_lo + prm.t_n > prm.T) return MI_ERR_SHAPE;
  if (prm.t_n == 0 || prm.H == 0 || prm.B == 0) return MI_OK;
  const bool bf = dtype == MI_BF16;
  const bool split = prm.split != 0;
  if (split && prm.mode != 1) return MI_ERR_SHAPE;
  const bool gather = prm.gather != 0;
  if (gather && (split || prm.mode != 1)) return MI_ERR_SHAPE;
#define MI_ATTN_CASE(DD)                                                                  \
  if (D == DD) {                                                                         \
    if (split)                                                                           \
      return bf ? launch_attn_t<__nv_bfloat16, DD, true, false>(q, k, v, out, prm, stream) \
                : launch_attn_t<__half, DD, true, false>(q, k, v, out, prm, stream);      \
    if (gather)                                                                          \
      return bf ? launch_attn_t<__nv_bfloat16, DD, false, true>(q, k, v, out, prm, stream) \
                : launch_attn_t<__half, DD, false, true>(q, k, v, out, prm, stream);      \
    return bf ? launch_attn_t<__nv_bfloat16, DD, false, false>(q, k, v, out, prm, stream)  \
              : launch_attn_t<__half, DD, false, false>(q, k, v, out, prm, stream);        \
  }
  MI_ATTN_CASE(64)
  MI_ATTN_CASE(96)
  MI_ATTN_CASE(128)
#undef MI_ATTN_CASE
  return MI_ERR_SHAPE;
}

}  // namespace mib200

#ifdef MI_TRACE
extern "C" int mi_debug_trace_gt(unsigned long long* host_out) {
  return cudaMemcpyFromSymbol(host_out, mib200::g_trace_gt, sizeof(mib200::g_trace_gt)) ==
                 cudaSuccess
             ? 0
             : 4;
}
extern "C" int mi_debug_trace(unsigned long long* host_out) {
  return cudaMemcpyFromSymbol(host_out, mib200::g_trace, sizeof(mib200::g_trace)) == cudaSuccess
             ? 0
             : 4;
}
#endif
