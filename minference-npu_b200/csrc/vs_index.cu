// vertical_and_slash pattern: index estimation (last-64-query softmax,
// column and diagonal sums, two top-k) and the attention plan built from the
// direct-mask semantics.
//
// Reference semantics:
//   minference/modules/minference_forward.py:124-167
//     qk = bf16(q[-64:] @ k^T) / sqrt(D) (rounded to the input dtype again),
//     last 64x64 causal mask, softmax in fp32, vertical = column sums,
//     slash = anti-diagonal sums (sum_all_diagonal_matrix), columns 0..29 and
//     the 100 most local diagonals forced in, two topk, v_idx ascending,
//     s_idx = S-1-diag descending.
//   minference/ops/vertical_slash_kernel_npu.py:255-369 (_build_vs_mask_direct)
//     query block bq, end_m = 64(bq+1): every slash s < end_m keeps keys
//     [re-64, re) with re = min(max(end_m - s, 64), S); vertical columns are
//     visible to every row; AND causal.
//
// Determinism: every floating-point reduction below has a fixed order and the
// exponential is an explicit Cody-Waite + degree-7 Taylor evaluation built
// from IEEE fma/mul/add only, so results are reproducible bit for bit by the
// C restatement used as the test oracle.
#include "attention.cuh"
#include "host_util.h"
#include "topk.cuh"

namespace mib200 {

// exp(y) for y <= 0 (y < -87 -> 0).  Cody & Waite argument reduction with the
// classic two-part ln2 split, then the Taylor polynomial of e^r to degree 7
// (|r| <= ln2/2, truncation error < 6e-9 relative).
__device__ __forceinline__ float det_exp(float y) {
  if (!(y >= -87.0f)) return 0.0f;
  const float n = rintf(__fmul_rn(y, 1.44269504088896341f));
  float r = __fmaf_rn(-n, 0.693145751953125f, y);
  r = __fmaf_rn(-n, 1.428606765330187045e-06f, r);
  float p = 1.0f / 5040.0f;
  p = __fmaf_rn(p, r, 1.0f / 720.0f);
  p = __fmaf_rn(p, r, 1.0f / 120.0f);
  p = __fmaf_rn(p, r, 1.0f / 24.0f);
  p = __fmaf_rn(p, r, 1.0f / 6.0f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const float scale = __int_as_float(((int)n + 127) << 23);
  return __fmul_rn(p, scale);
}

constexpr double kFixScale = 17592186044416.0;  // 2^44: row sums in 64-bit fixed point

// ---------------------------------------------------------------------------
// K3a: logits x[i][c] for the last LQ queries, rounded like the reference:
// round_dt(round_dt(dot) / sqrt_d); masked (c > S-LQ+i) entries are -inf.
// Stored as the input dtype's bits: x: [BH][LQ][S] uint16.
// Grid (ceil(S/128), H, B), 128 threads; one CTA = 64 query rows x 128 keys.
// Warp w owns rows [16w, 16w+16), lane l owns keys [4l, 4l+4): 64 independent
// fmaf chains per thread.  Each (row, key) dot product is still one chain
// over d = 0..D-1 in order, so the result is the oracle's bit for bit.  Q
// and the K tile are staged in shared memory as fp32, transposed ([d][row],
// [d][key]): one step over d reads one float4 of keys and four float4 of
// rows (the rows are the same for the whole warp: a broadcast).
// ---------------------------------------------------------------------------
constexpr int kLgRows = 64, kLgKeys = 128;

template <int D>
constexpr int vs_logits_smem_bytes() {
  return (kLgRows + kLgKeys) * D * 4;
}

template <typename DT, int D>
__global__ void __launch_bounds__(128) vs_logits_kernel(mi_tensor4 q, mi_tensor4 k, int H, int S,
                                                        int LQ, float sqrt_d, uint16_t* x) {
  extern __shared__ float4 lg_smem4[];
  float* qs = reinterpret_cast<float*>(lg_smem4);  // [D][64]
  float* ks = qs + D * kLgRows;                     // [D][128]
  const int h = blockIdx.y, b = blockIdx.z, bh = b * H + h;
  const int key0 = blockIdx.x * kLgKeys;
  const uint16_t* qb = reinterpret_cast<const uint16_t*>(q.ptr) + (long long)b * q.stride_b +
                       (long long)view_head(q, h) * q.stride_h;
  // Q tile: 16-byte loads (8 dims of one row), all issued before the
  // transposed fp32 stores; consecutive threads take consecutive rows, so
  // the stores are conflict-free.
  {
    constexpr int kUnits = kLgRows * D / 8;  // (row, 8-dim chunk) pairs
    constexpr int kPer = (kUnits + 127) / 128;
    uint4 raw[kPer];
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int e = threadIdx.x + r * 128;
      const int i = e % kLgRows, dc = e / kLgRows;
      raw[r] = make_uint4(0u, 0u, 0u, 0u);
      if (e < kUnits && i < LQ)
        raw[r] = *reinterpret_cast<const uint4*>(qb + (long long)(S - LQ + i) * q.stride_s + dc * 8);
    }
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int e = threadIdx.x + r * 128;
      if (e >= kUnits) break;
      const int i = e % kLgRows, dc = e / kLgRows;
      const uint16_t* hv = reinterpret_cast<const uint16_t*>(&raw[r]);
#pragma unroll
      for (int u = 0; u < 8; ++u) qs[(dc * 8 + u) * kLgRows + i] = DType<DT>::to_f(hv[u]);
    }
  }
  {
    const int c = key0 + threadIdx.x;
    const uint16_t* kr = reinterpret_cast<const uint16_t*>(k.ptr) + (long long)b * k.stride_b +
                         (long long)view_head(k, h) * k.stride_h + (long long)c * k.stride_s;
#pragma unroll
    for (int d = 0; d < D; d += 8) {
      uint4 raw = make_uint4(0u, 0u, 0u, 0u);
      if (c < S) raw = *reinterpret_cast<const uint4*>(kr + d);
      const uint16_t* hv = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
      for (int u = 0; u < 8; ++u) ks[(d + u) * kLgKeys + threadIdx.x] = DType<DT>::to_f(hv[u]);
    }
  }
  __syncthreads();

  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const float4* ks4 = reinterpret_cast<const float4*>(ks);
  const float4* qs4 = reinterpret_cast<const float4*>(qs);
  float acc[16][4];
#pragma unroll
  for (int r = 0; r < 16; ++r)
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[r][u] = 0.f;
#pragma unroll 2
  for (int d = 0; d < D; ++d) {
    const float4 kv = ks4[d * (kLgKeys / 4) + l];
#pragma unroll
    for (int r4 = 0; r4 < 4; ++r4) {
      const float4 qv = qs4[d * (kLgRows / 4) + w * 4 + r4];
      const float qr[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float* a = acc[r4 * 4 + u];
        a[0] = __fmaf_rn(qr[u], kv.x, a[0]);
        a[1] = __fmaf_rn(qr[u], kv.y, a[1]);
        a[2] = __fmaf_rn(qr[u], kv.z, a[2]);
        a[3] = __fmaf_rn(qr[u], kv.w, a[3]);
      }
    }
  }

  const uint16_t neg_inf = DType<DT>::kBF16 ? (uint16_t)0xFF80 : (uint16_t)0xFC00;
  const int c0 = key0 + 4 * l;
  const bool vec = (S % 4 == 0) && (c0 + 3 < S);
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    const int i = w * 16 + r;
    if (i >= LQ) break;
    uint16_t bits[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + u;
      if (c > S - LQ + i) {
        bits[u] = neg_inf;
      } else {
        const float r1 = DType<DT>::round(acc[r][u]);
        const float r2 = DType<DT>::round(__fdiv_rn(r1, sqrt_d));
        bits[u] = DType<DT>::kBF16 ? (uint16_t)(__float_as_uint(r2) >> 16)
                                   : __half_as_ushort(__float2half_rn(r2));
      }
    }
    uint16_t* xo = x + ((long long)bh * LQ + i) * S;
    if (vec) {
      *reinterpret_cast<uint2*>(xo + c0) =
          make_uint2((uint32_t)bits[0] | ((uint32_t)bits[1] << 16),
                     (uint32_t)bits[2] | ((uint32_t)bits[3] << 16));
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + u < S) xo[c0 + u] = bits[u];
    }
  }
}

// ---------------------------------------------------------------------------
// K3b: per-row max and sum of exp(x - max) (64-bit fixed point, so the sum is
// independent of the reduction order).  Grid (LQ, H, B), 1024 threads.
// stats: [BH][LQ] {m, 1/l}.  Rows up to kRowRegs * 8 * 1024 elements are read
// once with 16-byte loads and kept in registers for both passes (the max and
// the integer sum do not depend on the order); longer or unaligned rows take
// the two-pass scalar loop.
// ---------------------------------------------------------------------------
constexpr int kRowRegs = 8;  // uint4 per thread: 64 elements, rows up to 65536

template <typename DT>
__global__ void __launch_bounds__(1024) vs_rowstats_kernel(const uint16_t* x, int H, int S,
                                                           int LQ, float2* stats) {
  __shared__ float red_m[32];
  __shared__ unsigned long long red_s[32];
  const int i = blockIdx.x, h = blockIdx.y, b = blockIdx.z, bh = b * H + h;
  const uint16_t* xr = x + ((long long)bh * LQ + i) * S;
  const bool vec = S % 8 == 0 && S <= kRowRegs * 8 * 1024 &&
                   (reinterpret_cast<uintptr_t>(xr) & 15) == 0;
  uint4 v[kRowRegs];
  float m = -INFINITY;
  if (vec) {
    const int nv = S / 8;
#pragma unroll
    for (int r = 0; r < kRowRegs; ++r) {
      const int u = threadIdx.x + r * 1024;
      v[r] = u < nv ? reinterpret_cast<const uint4*>(xr)[u] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int r = 0; r < kRowRegs; ++r) {
      if (threadIdx.x + r * 1024 < nv) {
        const uint16_t* hv = reinterpret_cast<const uint16_t*>(&v[r]);
#pragma unroll
        for (int e = 0; e < 8; ++e) m = fmaxf(m, DType<DT>::to_f(hv[e]));
      }
    }
  } else {
    for (int c = threadIdx.x; c < S; c += blockDim.x) m = fmaxf(m, DType<DT>::to_f(xr[c]));
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red_m[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red_m[0];
  for (int w = 1; w < 32; ++w) m = fmaxf(m, red_m[w]);
  unsigned long long s = 0;
  auto add = [&](uint16_t bits) {
    const float e = det_exp(__fsub_rn(DType<DT>::to_f(bits), m));
    s += (unsigned long long)__float2ll_rz((float)(e * (float)kFixScale));
  };
  if (vec) {
    const int nv = S / 8;
#pragma unroll
    for (int r = 0; r < kRowRegs; ++r) {
      if (threadIdx.x + r * 1024 < nv) {
        const uint16_t* hv = reinterpret_cast<const uint16_t*>(&v[r]);
#pragma unroll
        for (int e = 0; e < 8; ++e) add(hv[e]);
      }
    }
  } else {
    for (int c = threadIdx.x; c < S; c += blockDim.x) add(xr[c]);
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long tot = 0;
    for (int w = 0; w < 32; ++w) tot += red_s[w];
    // {row max, 1 / row sum}: probabilities are exp(x - m) * (1 / l)
    const float l = (float)((double)tot / kFixScale);
    stats[(long long)bh * LQ + i] = make_float2(m, __fdiv_rn(1.0f, l));
  }
}

// ---------------------------------------------------------------------------
// K3c: p[i][c] = det_exp(x - m_i) * (1 / l_i);  vertical[c] = sum_i p[i][c];
// slash[t] = sum_i p[i][t + 1 + i - LQ] (columns outside [0,S) add nothing),
// both summed in row order.  Forced entries (c < 30, t >= S-100) get +inf.
// Output: order-preserving keys vkeys/skeys [BH][S].
// ---------------------------------------------------------------------------
template <typename DT>
__global__ void __launch_bounds__(256) vs_sums_kernel(const uint16_t* x, const float2* stats,
                                                      int H, int S, int LQ, uint32_t* vkeys,
                                                      uint32_t* skeys) {
  __shared__ float2 st[64];
  const int h = blockIdx.y, b = blockIdx.z, bh = b * H + h;
  if (threadIdx.x < LQ) st[threadIdx.x] = stats[(long long)bh * LQ + threadIdx.x];
  __syncthreads();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= S) return;
  const uint16_t* xb = x + (long long)bh * LQ * S;
  float vs = 0.f, ds = 0.f;
  for (int i = 0; i < LQ; ++i) {
    const float pv = __fmul_rn(det_exp(__fsub_rn(DType<DT>::to_f(xb[(long long)i * S + c]), st[i].x)), st[i].y);
    vs = __fadd_rn(vs, pv);
    const int col = c + 1 + i - LQ;
    if (col >= 0 && col < S) {
      const float pd = __fmul_rn(det_exp(__fsub_rn(DType<DT>::to_f(xb[(long long)i * S + col]), st[i].x)), st[i].y);
      ds = __fadd_rn(ds, pd);
    }
  }
  if (c < 30) vs = INFINITY;
  if (c >= S - 100) ds = INFINITY;
  vkeys[(long long)bh * S + c] = float_to_ordered(vs);
  skeys[(long long)bh * S + c] = float_to_ordered(ds);
}

// K3d: the two top-k selections.  One cluster of kVsSelCluster CTAs per
// (head, list): grid (H * kVsSelCluster, B, 2), 1024 threads per CTA.
constexpr int kVsSelThreads = 1024;
constexpr int kVsSelCluster = 8;
__global__ void __cluster_dims__(kVsSelCluster, 1, 1) __launch_bounds__(kVsSelThreads)
    vs_select_kernel(const uint32_t* vkeys, const uint32_t* skeys, int H, int S, int nv, int ns,
                     int32_t* v_idx, int32_t* s_idx) {
  __shared__ TopkSmem<kVsSelThreads> tsm;
  const int h = blockIdx.x / kVsSelCluster, b = blockIdx.y, bh = b * H + h;
  if (blockIdx.z == 0) {
    int32_t* dst = v_idx + (long long)bh * nv;
    cluster_topk<kVsSelThreads, kVsSelCluster>(vkeys + (long long)bh * S, S, nv, tsm,
                                               [&](int pos, int idx) { dst[pos] = idx; });
  } else {
    int32_t* dst = s_idx + (long long)bh * ns;
    cluster_topk<kVsSelThreads, kVsSelCluster>(skeys + (long long)bh * S, S, ns, tsm,
                                               [&](int pos, int idx) { dst[pos] = S - 1 - idx; });
  }
}

// ---------------------------------------------------------------------------
// K4a: per-head tables for the direct mask.
//   slashes   bitset of the selected slashes with per-word prefix counts
//             (SlashSet below; stored in the head's (S+1)-int P region)
//   vmask[kb] vertical columns of key block kb (64-bit)
//   smask[D]  for query block bq and key block kb = bq - D (not the ragged
//             last query block): key 64*kb + c is covered by a slash iff some
//             s lies in [D*64 - c, D*64 - c + 63]
//   clow[bq]  some slash s in (64*bq, 64*bq + 64) (range clamped to [0,64))
// Grid (H, B), 1024 threads.
// ---------------------------------------------------------------------------
// The selected slashes of a head as a bitset over [0, S) plus, per 32-bit
// word, the number of set bits in the words before it (nwords + 1 entries):
// the count of slashes in any range is two lookups and two popcounts.
struct SlashSet {
  const uint32_t* bits;
  const int* wpre;
};

__device__ __forceinline__ int vs_slash_words(int S) { return (S + 31) >> 5; }

// Number of selected slashes s < x, for 0 <= x <= S.
__device__ __forceinline__ int slash_rank(const SlashSet& ss, long long x) {
  const int w = (int)(x >> 5), r = (int)(x & 31);
  return ss.wpre[w] + (r ? __popc(ss.bits[w] & ((1u << r) - 1u)) : 0);
}

__device__ __forceinline__ bool any_slash(const SlashSet& ss, long long lo, long long hi, int S) {
  if (lo < 0) lo = 0;
  if (hi > S - 1) hi = S - 1;
  if (hi < lo) return false;
  return slash_rank(ss, hi + 1) - slash_rank(ss, lo) > 0;
}

__global__ void __launch_bounds__(1024) vs_tables_kernel(const int32_t* v_idx, int nv,
                                                         const int32_t* s_idx, int ns, int H,
                                                         int S, int nb, int* Pall,
                                                         unsigned long long* vmask_all,
                                                         uint32_t* smask_all, int* clow_all) {
  __shared__ int warp_tot[32];
  const int h = blockIdx.x, b = blockIdx.y, bh = b * H + h;
  const int nw = vs_slash_words(S);
  uint32_t* bits = reinterpret_cast<uint32_t*>(Pall + (long long)bh * (S + 1));
  int* wpre = reinterpret_cast<int*>(bits + nw);
  unsigned long long* vmask = vmask_all + (long long)bh * nb;
  uint32_t* smask = smask_all + (long long)bh * nb * 2;
  int* clow = clow_all + (long long)bh * nb;
  for (int i = threadIdx.x; i < nw; i += blockDim.x) bits[i] = 0u;
  for (int i = threadIdx.x; i < nb; i += blockDim.x) vmask[i] = 0ull;
  __syncthreads();
  for (int i = threadIdx.x; i < ns; i += blockDim.x) {
    const int sl = s_idx[(long long)bh * ns + i];
    if (sl >= 0 && sl < S) atomicOr(&bits[sl >> 5], 1u << (sl & 31));
  }
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    int c = v_idx[(long long)bh * nv + i];
    c = c < 0 ? 0 : (c > S - 1 ? S - 1 : c);
    atomicOr(&vmask[c >> 6], 1ull << (c & 63));
  }
  __syncthreads();
  // wpre: exclusive prefix of the word popcounts (contiguous word chunks per thread)
  const int ept = (nw + blockDim.x - 1) / blockDim.x;
  const int beg = min(nw, (int)threadIdx.x * ept), end = min(nw, beg + ept);
  int local = 0;
  for (int i = beg; i < end; ++i) local += __popc(bits[i]);
  int tot;
  int run = block_exclusive_scan<1024>(local, warp_tot, &tot);
  for (int i = beg; i < end; ++i) {
    wpre[i] = run;
    run += __popc(bits[i]);
  }
  if (threadIdx.x == 0) wpre[nw] = tot;
  __syncthreads();
  const SlashSet ss{bits, wpre};
  for (int base = 0; base < nb * 64; base += blockDim.x) {
    const int idx = base + threadIdx.x;
    bool bit = false;
    if (idx < nb * 64) {
      const long long Dl = idx >> 6, c = idx & 63;
      const long long d = Dl * 64 - c;
      bit = any_slash(ss, d, d + 63, S);
    }
    const unsigned bal = __ballot_sync(0xffffffffu, bit);
    if ((threadIdx.x & 31) == 0 && idx < nb * 64) smask[idx >> 5] = bal;
  }
  for (int bq = threadIdx.x; bq < nb; bq += blockDim.x)
    clow[bq] = any_slash(ss, (long long)bq * 64 + 1, (long long)bq * 64 + 63, S) ? 1 : 0;
}

// Slash coverage of key block kb for query block bq (the direct mask
// without the vertical columns).
__device__ __forceinline__ uint64_t vs_slash_mask(int bq, int kb, int S, int nb, const SlashSet& P,
                                                  const uint32_t* smask, const int* clow) {
  if (kb == 0 && clow[bq]) return ~0ull;
  uint64_t m = 0;
  const bool ragged_last = (bq == nb - 1) && (S % 64 != 0);
  if (!ragged_last) {
    const int Dl = bq - kb;
    m = (uint64_t)smask[2 * Dl] | ((uint64_t)smask[2 * Dl + 1] << 32);
  } else {
    const long long end_m = (long long)nb * 64;
    const long long lo_bound = end_m - S;  // slashes below this are clamped to [S-64, S)
    const bool high = any_slash(P, 0, lo_bound - 1, S);
    for (int c = 0; c < 64; ++c) {
      const long long j = (long long)kb * 64 + c;
      if (j >= S) break;
      const long long d = (long long)bq * 64 - j;
      long long lo = d > lo_bound ? d : lo_bound;
      bool bit = any_slash(P, lo, d + 63, S);
      if (high && j >= (long long)S - 64) bit = true;
      if (bit) m |= 1ull << c;
    }
  }
  return m;
}

// Gathered key groups of a tile (see AttnParams::gather).
struct VsGather {
  int gmax;              // groups per tile (0: gathering off)
  int32_t* gcols;        // [BH][T][gmax][64]
  unsigned long long* gmask;  // [BH][T][gmax][2], scratch for the masks
};

// K4b: plan.  One warp per 128-row query tile; entries in ascending kb.
// With gathering on, the vertical columns of a key block that no slash of
// either query block reaches (and that lies before both) are listed among
// the tile's gathered keys instead (with a visibility bit per query block),
// so a block touched only by scattered columns costs no 64-key step; blocks
// that are entries anyway keep their columns in their masks.  The groups
// follow the tile's block entries as entries with kb = -1 - g.  A group holds
// at least one column of each block it replaces and at most 64 columns, so
// groups never outnumber the blocks they replace and the tile's entries stay
// within its 2t + 2 plan slots.
__global__ void __launch_bounds__(128) vs_plan_kernel(int H, int S, int nb, int T,
                                                      const int* Pall,
                                                      const unsigned long long* vmask_all,
                                                      const uint32_t* smask_all,
                                                      const int* clow_all, long long cap,
                                                      long long head_stride, PlanEntry* plan,
                                                      int* plan_count, VsGather g) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + w;
  const int h = blockIdx.y, b = blockIdx.z, bh = b * H + h;
  if (t >= T) return;
  const uint32_t* pb = reinterpret_cast<const uint32_t*>(Pall + (long long)bh * (S + 1));
  const SlashSet P{pb, reinterpret_cast<const int*>(pb + vs_slash_words(S))};
  const unsigned long long* vmask = vmask_all + (long long)bh * nb;
  const uint32_t* smask = smask_all + (long long)bh * nb * 2;
  const int* clow = clow_all + (long long)bh * nb;
  const int bq0 = 2 * t, bq1 = 2 * t + 1;
  const int hi = min(bq1, nb - 1);
  PlanEntry* out = plan + (long long)bh * head_stride + plan_offset(t, cap);
  const long long gt = (long long)bh * T + t;
  int32_t* gcols = g.gmax ? g.gcols + gt * g.gmax * 64 : nullptr;
  unsigned long long* gmask = g.gmax ? g.gmask + gt * g.gmax * 2 : nullptr;
  if (g.gmax) {
    for (int i = lane; i < g.gmax * 64; i += 32) gcols[i] = -1;
    for (int i = lane; i < g.gmax * 2; i += 32) gmask[i] = 0ull;
    __syncwarp();
  }
  int count = 0, gtotal = 0;
  for (int base = 0; base <= hi; base += 32) {
    const int kb = base + lane;
    uint64_t m0 = 0, m1 = 0, u0 = 0, u1 = 0;
    if (kb <= hi) {
      const uint64_t vm = vmask[kb];
      const uint64_t v0 = (bq0 < nb && kb <= bq0) ? vm : 0ull;
      const uint64_t v1 = (bq1 < nb && kb <= bq1) ? vm : 0ull;
      if (bq0 < nb && kb <= bq0) m0 = vs_slash_mask(bq0, kb, S, nb, P, smask, clow);
      if (bq1 < nb && kb <= bq1) m1 = vs_slash_mask(bq1, kb, S, nb, P, smask, clow);
      if (g.gmax && (m0 | m1) == 0ull && kb < bq0) {
        // no slash reaches this block (which lies before both query blocks):
        // its columns are gathered instead of costing a 64-key step
        u0 = v0;
        u1 = v1;
      } else {
        m0 |= v0;
        m1 |= v1;
      }
    }
    const bool keep = (m0 | m1) != 0ull;
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    if (keep) {
      PlanEntry e;
      e.kb = kb;
      e.kb1 = kb;
      e.m0 = m0;
      e.m1 = m1;
      out[count + __popc(bal & ((1u << lane) - 1u))] = e;
    }
    count += __popc(bal);
    if (g.gmax) {
      // gathered keys in ascending order: this lane's block after the lower lanes'
      uint64_t un = u0 | u1;
      const int n = __popcll(un);
      int off = n;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, off, d);
        if (lane >= d) off += y;
      }
      const int tot = __shfl_sync(0xffffffffu, off, 31);
      int idx = gtotal + off - n;
      while (un) {
        const int c = __ffsll((long long)un) - 1;
        un &= un - 1;
        const int gi = idx >> 6, slot = idx & 63;
        if (gi < g.gmax) {
          gcols[gi * 64 + slot] = kb * 64 + c;
          if ((u0 >> c) & 1ull) atomicOr(&gmask[2 * gi], 1ull << slot);
          if ((u1 >> c) & 1ull) atomicOr(&gmask[2 * gi + 1], 1ull << slot);
        }
        ++idx;
      }
      gtotal += tot;
    }
  }
  if (g.gmax) {
    __syncwarp();
    __threadfence_block();
    const int ng = min((gtotal + 63) / 64, g.gmax);
    for (int gi = lane; gi < ng; gi += 32) {
      PlanEntry e;
      e.kb = -1 - gi;
      e.kb1 = e.kb;
      e.m0 = __ldcg(&gmask[2 * gi]);  // L2: the atomics above
      e.m1 = __ldcg(&gmask[2 * gi + 1]);
      out[count + gi] = e;
    }
    count += ng;
  }
  if (lane == 0) plan_count[gt] = count;
}


int launch_attention(const mi_tensor4& q, const mi_tensor4& k, const mi_tensor4& v,
                     const mi_tensor4& out, int64_t D, int dtype, AttnParams prm,
                     cudaStream_t stream);

}  // namespace mib200

using namespace mib200;

// ---------------------------------------------------------------------------
// Estimation entry point
// ---------------------------------------------------------------------------
extern "C" size_t mi_vs_estimate_workspace_size(int64_t B, int64_t H, int64_t S) {
  const int64_t LQ = S < 64 ? S : 64;
  return align_up(2ull * B * H * LQ * S) + align_up(sizeof(float2) * B * H * LQ) +
         2 * align_up(4ull * B * H * S);
}

template <typename DT, int D>
static void launch_vs_logits(const mi_tensor4& q, const mi_tensor4& k, int64_t B, int64_t H,
                             int64_t S, int LQ, float sqrt_d, uint16_t* x, cudaStream_t st) {
  dim3 g((unsigned)((S + kLgKeys - 1) / kLgKeys), (unsigned)H, (unsigned)B);
  constexpr int smem = vs_logits_smem_bytes<D>();
  cudaFuncSetAttribute(vs_logits_kernel<DT, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  vs_logits_kernel<DT, D><<<g, 128, smem, st>>>(q, k, (int)H, (int)S, LQ, sqrt_d, x);
}

extern "C" int mi_vs_estimate(mi_tensor4 q, mi_tensor4 k, int64_t B, int64_t H, int64_t S,
                              int64_t D, int dtype, int64_t vertical_size, int64_t slash_size,
                              float logit_scale, int32_t* v_idx, int32_t* s_idx, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (dtype != MI_F16 && dtype != MI_BF16) return MI_ERR_DTYPE;
  if (D != 64 && D != 96 && D != 128) return MI_ERR_SHAPE;
  if (B < 0 || H < 0 || S < 0 || S > (1 << 24)) return MI_ERR_SHAPE;
  if (vertical_size < 1 || vertical_size > S || slash_size < 1 || slash_size > S)
    return MI_ERR_SHAPE;
  // Rows of q and k are read with 16-byte loads: unit dim stride, 8-element
  // (16-byte) aligned batch / head / row strides and base pointers.
  auto rows16 = [](const mi_tensor4& t) {
    return t.stride_d == 1 && t.stride_s % 8 == 0 && t.stride_h % 8 == 0 && t.stride_b % 8 == 0 &&
           (reinterpret_cast<uintptr_t>(t.ptr) & 15) == 0;
  };
  if (!rows16(q) || !rows16(k)) return MI_ERR_ALIGN;
  if (B == 0 || H == 0 || S == 0) return MI_OK;
  if (!workspace || workspace_bytes < mi_vs_estimate_workspace_size(B, H, S)) return MI_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int LQ = (int)(S < 64 ? S : 64);
  char* w = reinterpret_cast<char*>(workspace);
  uint16_t* x = reinterpret_cast<uint16_t*>(w);
  w += align_up(2ull * B * H * LQ * S);
  float2* stats = reinterpret_cast<float2*>(w);
  w += align_up(sizeof(float2) * B * H * LQ);
  uint32_t* vkeys = reinterpret_cast<uint32_t*>(w);
  w += align_up(4ull * B * H * S);
  uint32_t* skeys = reinterpret_cast<uint32_t*>(w);
  // The reference divides by sqrt(D); logit_scale is 1/sqrt(D), so divide by its inverse.
  const float sqrt_d = 1.0f / logit_scale;
  const bool bf = dtype == MI_BF16;
#define VS_LOG(DD)                                                                              \
  if (D == DD) {                                                                                \
    if (bf) launch_vs_logits<__nv_bfloat16, DD>(q, k, B, H, S, LQ, sqrt_d, x, st);              \
    else launch_vs_logits<__half, DD>(q, k, B, H, S, LQ, sqrt_d, x, st);                        \
  }
  VS_LOG(64) VS_LOG(96) VS_LOG(128)
#undef VS_LOG
  dim3 g2((unsigned)LQ, (unsigned)H, (unsigned)B);
  dim3 g3((unsigned)((S + 255) / 256), (unsigned)H, (unsigned)B);
  if (bf) {
    vs_rowstats_kernel<__nv_bfloat16><<<g2, 1024, 0, st>>>(x, (int)H, (int)S, LQ, stats);
    vs_sums_kernel<__nv_bfloat16><<<g3, 256, 0, st>>>(x, stats, (int)H, (int)S, LQ, vkeys, skeys);
  } else {
    vs_rowstats_kernel<__half><<<g2, 1024, 0, st>>>(x, (int)H, (int)S, LQ, stats);
    vs_sums_kernel<__half><<<g3, 256, 0, st>>>(x, stats, (int)H, (int)S, LQ, vkeys, skeys);
  }
  dim3 g4((unsigned)(H * kVsSelCluster), (unsigned)B, 2);
  vs_select_kernel<<<g4, kVsSelThreads, 0, st>>>(vkeys, skeys, (int)H, (int)S, (int)vertical_size,
                                                 (int)slash_size, v_idx, s_idx);
  return cudaGetLastError() == cudaSuccess ? MI_OK : MI_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------
// Sparse attention entry point
// ---------------------------------------------------------------------------
struct VsWs {
  int* P;
  unsigned long long* vmask;
  uint32_t* smask;
  int* clow;
  PlanEntry* plan;
  int* count;
  int32_t* gcols;
  unsigned long long* gmask;
  size_t bytes;
};

// Gathered key groups per tile: vertical_size up to kVsGatherCols columns are
// gathered (kVsGatherMax groups of 64); larger vertical sets keep the columns
// in their blocks' masks.
constexpr int kVsGatherMax = 16;
constexpr int kVsGatherCols = kVsGatherMax * 64;

static VsWs vs_ws_layout(void* base, int64_t B, int64_t H, int64_t S) {
  const int64_t nb = (S + 63) / 64, T = (S + 127) / 128;
  const int64_t cap = 2 * T;
  VsWs w{};
  char* p = reinterpret_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t n) { char* r = p ? p + off : nullptr; off += align_up(n); return r; };
  w.P = reinterpret_cast<int*>(take(4ull * B * H * (S + 1)));
  w.vmask = reinterpret_cast<unsigned long long*>(take(8ull * B * H * nb));
  w.smask = reinterpret_cast<uint32_t*>(take(8ull * B * H * nb));
  w.clow = reinterpret_cast<int*>(take(4ull * B * H * nb));
  w.plan = reinterpret_cast<PlanEntry*>(take(sizeof(PlanEntry) * B * H * plan_offset(T, cap)));
  w.count = reinterpret_cast<int*>(take(4ull * B * H * T));
  w.gcols = reinterpret_cast<int32_t*>(take(4ull * B * H * T * kVsGatherMax * 64));
  w.gmask = reinterpret_cast<unsigned long long*>(take(16ull * B * H * T * kVsGatherMax));
  w.bytes = off;
  return w;
}

extern "C" size_t mi_vs_sparse_fwd_workspace_size(int64_t B, int64_t H, int64_t S) {
  return vs_ws_layout(nullptr, B, H, S).bytes;
}

extern "C" int mi_vs_sparse_fwd_rows(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out,
                                     int64_t B, int64_t H, int64_t S, int64_t D, int dtype,
                                     const int32_t* v_idx, int64_t nv, const int32_t* s_idx,
                                     int64_t ns, float softmax_scale, int64_t row_begin,
                                     int64_t row_end, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  if (dtype != MI_F16 && dtype != MI_BF16) return MI_ERR_DTYPE;
  if (D != 64 && D != 96 && D != 128) return MI_ERR_SHAPE;
  if (B < 0 || H < 0 || S < 0 || nv < 0 || ns < 0 || S > (1 << 24)) return MI_ERR_SHAPE;
  if (B > 65535 || H > 65535) return MI_ERR_SHAPE;
  if (!row_window_ok(row_begin, row_end, S)) return MI_ERR_SHAPE;
  if (B == 0 || H == 0 || S == 0 || row_begin == row_end) return MI_OK;
  const VsWs w = vs_ws_layout(workspace, B, H, S);
  if (!workspace || workspace_bytes < w.bytes) return MI_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t nb = (S + 63) / 64, T = (S + 127) / 128;
  const int64_t cap = 2 * T;
  const int64_t head_stride = plan_offset(T, cap);
  vs_tables_kernel<<<dim3((unsigned)H, (unsigned)B), 1024, 0, st>>>(
      v_idx, (int)nv, s_idx, (int)ns, (int)H, (int)S, (int)nb, w.P, w.vmask, w.smask, w.clow);
  // Gathered keys need K and V rows addressable as one 2-D row view: every
  // (b, h) starts a whole number of rows after the base pointer.
  static const bool gather_env = [] {
    const char* e = getenv("MI_VS_GATHER");
    return !(e && e[0] == '0');
  }();
  auto row_view = [](const mi_tensor4& t) {
    return t.stride_s > 0 && t.stride_h % t.stride_s == 0 && t.stride_b % t.stride_s == 0 &&
           t.stride_h >= 0 && t.stride_b >= 0;
  };
  const bool gather = gather_env && nv <= kVsGatherCols && row_view(k) && row_view(v) &&
                      k.stride_s == v.stride_s && k.stride_h == v.stride_h &&
                      k.stride_b == v.stride_b;
  VsGather vg{gather ? kVsGatherMax : 0, w.gcols, w.gmask};
  dim3 g((unsigned)((T + 3) / 4), (unsigned)H, (unsigned)B);
  vs_plan_kernel<<<g, 128, 0, st>>>((int)H, (int)S, (int)nb, (int)T, w.P, w.vmask, w.smask,
                                    w.clow, cap, head_stride, w.plan, w.count, vg);
  if (cudaGetLastError() != cudaSuccess) return MI_ERR_LAUNCH;
  AttnParams prm{};
  prm.B = (int)B;
  prm.H = (int)H;
  prm.Sq = (int)S;
  prm.Sk = (int)S;
  prm.q_off = 0;
  prm.T = (int)T;
  prm.mode = 1;
  prm.n_init = 0;
  prm.n_local = 1ll << 40;  // unbounded window (see AttnParams)
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  prm.plan = w.plan;
  prm.plan_count = w.count;
  prm.plan_cap = cap;
  prm.plan_head_stride = head_stride;
  if (gather) {
    prm.gather = 1;
    prm.gmax = kVsGatherMax;
    prm.gcols = w.gcols;
    prm.grow_b = k.stride_b / k.stride_s;
    prm.grow_h = k.stride_h / k.stride_s;
  }
  prm.t_lo = (int)(row_begin / 128);
  prm.t_n = (int)((row_end + 127) / 128) - prm.t_lo;
  return launch_attention(q, k, v, out, D, dtype, prm, st);
}

extern "C" int mi_vs_sparse_fwd(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out,
                                int64_t B, int64_t H, int64_t S, int64_t D, int dtype,
                                const int32_t* v_idx, int64_t nv, const int32_t* s_idx,
                                int64_t ns, float softmax_scale, void* workspace,
                                size_t workspace_bytes, void* stream) {
  return mi_vs_sparse_fwd_rows(q, k, v, out, B, H, S, D, dtype, v_idx, nv, s_idx, ns,
                               softmax_scale, 0, S, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// Legacy four-array VS index format (upstream MInference's
// convert_vertical_slash_indexes; the reference's CPU port is
// minference/backend_npu/cuda_shim.py:53-236).  One thread per
// (b, h, 64-row query block) runs the two-pointer merge of the ascending
// vertical list and the descending slash list:
//   * slashes s >= end_m are skipped;
//   * each slash gives a range ending at max(end_m - s, 64); a range that
//     starts more than one block after the current one is flushed as 64-key
//     blocks, a touching/overlapping one extends the current range by exactly
//     one block (the upstream "+= blk" rule, a superset of the exact union);
//   * vertical columns before the current range start are kept as columns;
//     columns inside a range are dropped; with no valid slash every vertical
//     column < end_m is kept.
// Rows past seqlens[b] get zero counts.  Entries beyond the counts are zero.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) vs_convert_kernel(
    const int32_t* seqlens, const int32_t* v_idx, int nv, const int32_t* s_idx, int ns, int H,
    int num_rows, int32_t* block_count, int32_t* block_offset, int32_t* column_count,
    int32_t* column_index) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  const int h = blockIdx.y, b = blockIdx.z, bh = b * H + h;
  if (row >= num_rows) return;
  const long long ro = (long long)bh * num_rows + row;
  int32_t* boff = block_offset + ro * ns;
  int32_t* cidx = column_index + ro * nv;
  const int32_t* vl = v_idx + (long long)bh * nv;
  const int32_t* sl = s_idx + (long long)bh * ns;
  const int blk = 64;
  const int start_m = row * blk;
  int nb = 0, nc = 0;
  if (start_m < seqlens[b]) {
    const int end_m = start_m + blk;
    int v = 0, s = 0;
    int v_val;
    if (nv == 0) {
      v_val = end_m + blk;
    } else {
      v_val = vl[0];
      v = 1;
    }
    int s_raw = 0;
    bool found = false;
    while (s < ns) {
      s_raw = sl[s++];
      if (s_raw < end_m) {
        found = true;
        break;
      }
    }
    if (!found) {
      while (true) {
        if (v_val <= end_m + blk && v_val < end_m) cidx[nc++] = v_val;
        if (v < nv) {
          v_val = vl[v++];
        } else {
          break;
        }
      }
    } else {
      int range_end = max(end_m - s_raw, blk);
      int range_start = range_end - blk;
      while (true) {
        if (v_val < range_end) {
          if (v_val < range_start) cidx[nc++] = v_val;
          if (v < nv) {
            v_val = vl[v++];
          } else {
            v_val = end_m + blk;
          }
        } else {
          int new_end;
          if (s < ns) {
            new_end = max(end_m - sl[s++], blk);
          } else {
            for (int x = range_start; x < range_end; x += blk) boff[nb++] = x;
            break;
          }
          if (new_end > range_end + blk) {
            for (int x = range_start; x < range_end; x += blk) boff[nb++] = x;
            range_start = new_end - blk;
            range_end = new_end;
          } else if (new_end > range_end) {
            range_end += blk;
          }
        }
      }
    }
  }
  block_count[ro] = nb;
  column_count[ro] = nc;
  for (int i = nb; i < ns; ++i) boff[i] = 0;
  for (int i = nc; i < nv; ++i) cidx[i] = 0;
}

extern "C" int mi_vs_convert_indexes(const int32_t* seqlens, const int32_t* v_idx, int64_t nv,
                                     const int32_t* s_idx, int64_t ns, int64_t B, int64_t H,
                                     int64_t context_size, int32_t* block_count,
                                     int32_t* block_offset, int32_t* column_count,
                                     int32_t* column_index, void* stream) {
  if (B < 0 || H < 0 || nv < 0 || ns < 0 || context_size < 0 || context_size > (1ll << 30))
    return MI_ERR_SHAPE;
  if (B > 65535 || H > 65535) return MI_ERR_SHAPE;
  const int64_t num_rows = (context_size + 63) / 64;
  if (B == 0 || H == 0 || num_rows == 0) return MI_OK;
  dim3 g((unsigned)((num_rows + 127) / 128), (unsigned)H, (unsigned)B);
  vs_convert_kernel<<<g, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      seqlens, v_idx, (int)nv, s_idx, (int)ns, (int)H, (int)num_rows, block_count, block_offset,
      column_count, column_index);
  return cudaGetLastError() == cudaSuccess ? MI_OK : MI_ERR_LAUNCH;
}
