// Sparse FlashAttention forward kernel (tcgen05 + TMA) and its host launcher.
// Design notes are at the top of attention.cuh.
#include "attention.cuh"
#include "host_util.h"

namespace mib200 {

template <typename DT, int D>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  using L = AttnSmem<D>;
  constexpr int NC = L::NC;
  constexpr bool kBF16 = DType<DT>::kBF16;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 1 + kStages;
  uint64_t* s_full = bars + 1 + 2 * kStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = s_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlotOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbortOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int t = p.T - 1 - blockIdx.x;  // heavy (late) tiles first
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int bh = b * p.H + h;

  // ---- entry list of this tile -------------------------------------------
  EntrySource src;
  src.mode = p.mode;
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
  }

  // ---- one-time setup -------------------------------------------------------
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kBM);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4) {
    // ======================= TMA producer =====================================
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      uint8_t* sq = smem + L::kQOff;
      mbar_arrive_expect_tx(q_full, L::kQBytes);
      for (int c = 0; c < NC; ++c)
        tma_load_4d(sq + c * (kBM * 64), &tm_q, q_full, c * 32, t * kBM, h, b);
      for (int j = 0; j < n_entries; ++j) {
        const int st = j % kStages;
        const int use = j / kStages;
        if (use > 0) {
          if (!mbar_wait(&kv_empty[st], (use - 1) & 1, 101)) { *abort_flag = 1; break; }
        }
        if (*abort_flag) break;
        int kb;
        uint64_t m0, m1;
        src.get(j, kb, m0, m1);
        uint8_t* sk = smem + L::kKOff + st * L::kKVBytes;
        uint8_t* sv = smem + L::kVOff + st * L::kKVBytes;
        mbar_arrive_expect_tx(&kv_full[st], 2 * L::kKVBytes);
        for (int c = 0; c < NC; ++c) {
          tma_load_4d(sk + c * (kBN * 64), &tm_k, &kv_full[st], c * 32, kb * kBN, h, b);
          tma_load_4d(sv + c * (kBN * 64), &tm_v, &kv_full[st], c * 32, kb * kBN, h, b);
        }
      }
    }
  } else if (warp == 5) {
    // ======================= MMA issuer =======================================
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kBF16, kBM, kBN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBF16, kBM, D, false, true);
      const uint32_t sq = smem_u32(smem + L::kQOff);
      const uint32_t sk0 = smem_u32(smem + L::kKOff);
      const uint32_t sv0 = smem_u32(smem + L::kVOff);
      const uint32_t sp0 = smem_u32(smem + L::kPOff);
      const uint32_t tmem_o = tmem_base + 128;

      auto issue_qk = [&](int j) {
        const int st = j % kStages;
        const uint32_t sk = sk0 + st * L::kKVBytes;
        const uint32_t tmem_s = tmem_base + (j & 1) * kBN;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t koff = (ks & 1) * 32;
          const uint64_t ad = make_desc_sw64(sq + (ks >> 1) * (kBM * 64) + koff, 16, 512);
          const uint64_t bd = make_desc_sw64(sk + (ks >> 1) * (kBN * 64) + koff, 16, 512);
          umma_f16_ss(tmem_s, ad, bd, idesc_qk, ks > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
      };
      bool ok = mbar_wait(q_full, 0, 102);
      if (ok && n_entries > 0) {
        ok = mbar_wait(&kv_full[0], 0, 103);
        if (ok) {
          tc_fence_after();
          issue_qk(0);
        }
      }
      for (int j = 0; ok && j < n_entries; ++j) {
        if (*abort_flag) break;
        if (j + 1 < n_entries) {
          const int st = (j + 1) % kStages;
          if (!mbar_wait(&kv_full[st], ((j + 1) / kStages) & 1, 104)) { ok = false; break; }
          tc_fence_after();
          issue_qk(j + 1);
        }
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, 105)) { ok = false; break; }
        tc_fence_after();
        const int st = j % kStages;
        const uint32_t sv = sv0 + st * L::kKVBytes;
        const uint32_t sp = sp0 + (j & 1) * L::kPBytes;
#pragma unroll
        for (int ks = 0; ks < kBN / 16; ++ks) {
          const uint64_t ad = make_desc_sw64(sp + (ks >> 1) * (kBM * 64) + (ks & 1) * 32, 16, 512);
          const uint64_t bd = make_desc_sw64(sv + ks * 1024, kBN * 64, 512);
          umma_f16_ss(tmem_o, ad, bd, idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[j & 1]);
        umma_commit(&kv_empty[st]);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ======================= softmax warps 0-3 ================================
    const int row = threadIdx.x;  // 0..127
    const uint32_t lane_base = tmem_base + ((uint32_t)(warp * 32) << 16);
    const long long a = (long long)p.q_off + (long long)t * kBM + row;  // absolute position
    const float NEG_INF = -INFINITY;
    float m_used = NEG_INF;
    float l = 0.f;
    uint8_t* sp_base = smem + L::kPOff;
    bool ok = true;

    for (int j = 0; j < n_entries; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, 106)) { ok = false; break; }
      tc_fence_after();
      float s[kBN];
      tmem_ld32(lane_base + (j & 1) * kBN, *reinterpret_cast<float(*)[32]>(&s[0]));
      tmem_ld32(lane_base + (j & 1) * kBN + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
      tmem_wait_ld();

      int kb;
      uint64_t m0, m1;
      src.get(j, kb, m0, m1);
      const uint64_t mask = (row < 64) ? m0 : m1;
      const long long key0 = (long long)kb * kBN;
      // Visible keys of this row inside the block form: mask AND key <= a AND key < Sk AND
      // (key < n_init OR key > a - n_local).  Fast path when all 64 are visible.
      const bool full = (mask == ~0ull) && (key0 + kBN - 1 <= a) && (key0 + kBN - 1 < p.Sk) &&
                        (key0 > a - p.n_local || key0 + kBN - 1 < p.n_init);
      float tmax = NEG_INF;
      if (full) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          s[c] *= p.scale_log2;
          tmax = fmaxf(tmax, s[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          const long long key = key0 + c;
          const bool vis = ((mask >> c) & 1ull) && key <= a && key < p.Sk &&
                           (key < p.n_init || key > a - p.n_local);
          s[c] = vis ? s[c] * p.scale_log2 : NEG_INF;
          tmax = fmaxf(tmax, s[c]);
        }
      }
      const float m_new = fmaxf(m_used, tmax);
      const bool need = m_new > m_used + 8.0f;
      if (j == 0) {
        m_used = m_new;
      } else if (__any_sync(0xffffffffu, need)) {
        // O must hold PV(j-1) before it is rescaled.
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, 107)) { ok = false; break; }
        tc_fence_after();
        const float f = need ? ((m_used == NEG_INF) ? 0.f : fast_exp2(m_used - m_new)) : 1.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(lane_base + 128 + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) o[x] *= f;
          tmem_st32(lane_base + 128 + c * 32, o);
        }
        tmem_wait_st();
        if (need) {
          l *= f;
          m_used = m_new;
        }
      }
      // P = exp2(s - m_used); rows with nothing visible yet keep P = 0.
      float lsum = 0.f;
      uint32_t pk[kBN / 2];
      if (m_used == NEG_INF) {
#pragma unroll
        for (int c = 0; c < kBN / 2; ++c) pk[c] = 0u;
      } else {
#pragma unroll
        for (int c = 0; c < kBN / 2; ++c) {
          const float p0 = fast_exp2(s[2 * c] - m_used);
          const float p1 = fast_exp2(s[2 * c + 1] - m_used);
          lsum += p0 + p1;
          pk[c] = DType<DT>::pack2(p0, p1);
        }
      }
      l += lsum;
      // P buffer (j & 1) was last read by PV(j-2).
      if (j >= 2) {
        if (!mbar_wait(&pv_done[j & 1], ((j - 2) >> 1) & 1, 108)) { ok = false; break; }
      }
      uint8_t* sp = sp_base + (j & 1) * L::kPBytes;
      const uint32_t sw = (row >> 1) & 3;
#pragma unroll
      for (int pc = 0; pc < 2; ++pc) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 val = make_uint4(pk[pc * 16 + u * 4 + 0], pk[pc * 16 + u * 4 + 1],
                                 pk[pc * 16 + u * 4 + 2], pk[pc * 16 + u * 4 + 3]);
          *reinterpret_cast<uint4*>(sp + pc * (kBM * 64) + row * 64 + ((u ^ sw) << 4)) = val;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }

    // ---- epilogue: O / l -> out ---------------------------------------------
    if (!ok) *abort_flag = 1;
    const long long qrow = (long long)t * kBM + row;
    float o[D];
    bool have_o = false;
    if (ok && n_entries > 0 && !*abort_flag) {
      const int jl = n_entries - 1;
      if (mbar_wait(&pv_done[jl & 1], (jl >> 1) & 1, 109)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          tmem_ld32(lane_base + 128 + c * 32, *reinterpret_cast<float(*)[32]>(&o[c * 32]));
        tmem_wait_ld();
        have_o = true;
      } else {
        *abort_flag = 1;
      }
    }
    if (qrow < p.Sq) {
      const float inv = (have_o && l > 0.f) ? 1.f / l : 0.f;
      DT* dst = reinterpret_cast<DT*>(p.out) + (long long)b * p.os_b + (long long)h * p.os_h +
                qrow * p.os_s;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        uint4 val;
        val.x = DType<DT>::pack2(have_o ? o[8 * c + 0] * inv : 0.f, have_o ? o[8 * c + 1] * inv : 0.f);
        val.y = DType<DT>::pack2(have_o ? o[8 * c + 2] * inv : 0.f, have_o ? o[8 * c + 3] * inv : 0.f);
        val.z = DType<DT>::pack2(have_o ? o[8 * c + 4] * inv : 0.f, have_o ? o[8 * c + 5] * inv : 0.f);
        val.w = DType<DT>::pack2(have_o ? o[8 * c + 6] * inv : 0.f, have_o ? o[8 * c + 7] * inv : 0.f);
        *reinterpret_cast<uint4*>(dst + 8 * c) = val;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host launcher
// ---------------------------------------------------------------------------
template <typename DT, int D>
static int launch_attn_t(const mi_tensor4& q, const mi_tensor4& k, const mi_tensor4& v,
                         AttnParams prm, cudaStream_t stream) {
  using L = AttnSmem<D>;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_bnsd_map(&tq, q, prm.B, prm.H, prm.Sq, D, 32, kBM)) != MI_OK) return rc;
  if ((rc = make_bnsd_map(&tk, k, prm.B, prm.H, prm.Sk, D, 32, kBN)) != MI_OK) return rc;
  if ((rc = make_bnsd_map(&tv, v, prm.B, prm.H, prm.Sk, D, 32, kBN)) != MI_OK) return rc;
  auto kern = attn_fwd_kernel<DT, D>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc) !=
      cudaSuccess)
    return MI_ERR_LAUNCH;
  dim3 grid(prm.T, prm.H, prm.B);
  kern<<<grid, kThreads, L::kAlloc, stream>>>(tq, tk, tv, prm);
  return cudaGetLastError() == cudaSuccess ? MI_OK : MI_ERR_LAUNCH;
}

int launch_attention(const mi_tensor4& q, const mi_tensor4& k, const mi_tensor4& v,
                     const mi_tensor4& out, int64_t D, int dtype, AttnParams prm,
                     cudaStream_t stream) {
  prm.out = out.ptr;
  prm.os_b = out.stride_b;
  prm.os_h = out.stride_h;
  prm.os_s = out.stride_s;
  if (prm.T == 0 || prm.H == 0 || prm.B == 0) return MI_OK;
  if (out.stride_d != 1 || (reinterpret_cast<uintptr_t>(out.ptr) & 15) || (out.stride_s * 2) % 16 ||
      (out.stride_h * 2) % 16 || (out.stride_b * 2) % 16)
    return MI_ERR_ALIGN;
  const bool bf = dtype == MI_BF16;
#define MI_ATTN_CASE(DD)                                                            \
  if (D == DD)                                                                     \
    return bf ? launch_attn_t<__nv_bfloat16, DD>(q, k, v, prm, stream)             \
              : launch_attn_t<__half, DD>(q, k, v, prm, stream);
  MI_ATTN_CASE(64)
  MI_ATTN_CASE(96)
  MI_ATTN_CASE(128)
#undef MI_ATTN_CASE
  return MI_ERR_SHAPE;
}

}  // namespace mib200
