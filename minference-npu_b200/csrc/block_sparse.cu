// block_sparse pattern: block mean-pooling, block scores + top-k selection,
// and the per-query-tile attention plan.
//
// Reference semantics (minference/ops/block_sparse_kernel_npu.py):
//   _select_block_sparse_topk_indices (:230-263): pad S to a multiple of 64,
//     mean-pool Q and K per 64-row block (in the input dtype, then fp32),
//     scores = q_pool @ k_pool^T * score_scale, key blocks after the query
//     block set to -inf, topk(min(k, n_bk)), indices sorted ascending.
//   _build_block_sparse_mask (:266-317): selected blocks expanded to tokens,
//     AND per-token causal.
#include "attention.cuh"
#include "host_util.h"
#include "topk.cuh"

namespace mib200 {

// ---------------------------------------------------------------------------
// K1: mean pooling.  Pooled value = round_to_input_dtype(sum_fp32 / 64) with
// the 64 rows added in row order (rows beyond S contribute the zero padding).
// q_pool: [BH][nbq][D] fp32, k_poolT: [BH][D][nbk] fp32 (transposed so the
// score kernel reads it coalesced).  Grid (max(nbq,nbk), H, B), 2*128 threads.
// ---------------------------------------------------------------------------
template <typename DT>
__global__ void __launch_bounds__(256) pool_kernel(mi_tensor4 q, mi_tensor4 k, int H, int Sq,
                                                   int Sk, int D, int nbq, int nbk,
                                                   float* q_pool, float* k_poolT) {
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int bh = b * H + h;
  const bool is_k = threadIdx.x >= 128;
  const int d = threadIdx.x & 127;
  if (d >= D) return;
  const int S = is_k ? Sk : Sq;
  const int nb = is_k ? nbk : nbq;
  if (blk >= nb) return;
  const mi_tensor4& t = is_k ? k : q;
  const uint16_t* base = reinterpret_cast<const uint16_t*>(t.ptr) + (long long)b * t.stride_b +
                         (long long)view_head(t, h) * t.stride_h + d;
  const int r0 = blk * 64;
  const int rn = min(64, S - r0);
  float vals[64];
#pragma unroll
  for (int r = 0; r < 64; ++r)
    vals[r] = (r < rn) ? DType<DT>::to_f(base[(long long)(r0 + r) * t.stride_s]) : 0.f;
  float acc = 0.f;
#pragma unroll
  for (int r = 0; r < 64; ++r) acc = __fadd_rn(acc, vals[r]);
  const float pooled = DType<DT>::round(__fdiv_rn(acc, 64.f));
  if (is_k)
    k_poolT[((long long)bh * D + d) * nbk + blk] = pooled;
  else
    q_pool[((long long)bh * nbq + blk) * D + d] = pooled;
}

// ---------------------------------------------------------------------------
// K1 (vectorised): same result as pool_kernel, 16-byte loads.  One thread
// owns 8 consecutive dims of one 64-row block and adds the 64 rows in row
// order.  Needs D % 8 == 0 and 16-byte aligned rows.  Grid
// (ceil(max(nbq,nbk)/8), H, 2B): z = 2b + (0: q, 1: k).  Block 8 * D/8 threads.
// ---------------------------------------------------------------------------
template <typename DT>
__global__ void __launch_bounds__(128) pool_kernel_v(mi_tensor4 q, mi_tensor4 k, int H, int Sq,
                                                     int Sk, int D, int nbq, int nbk,
                                                     float* q_pool, float* k_poolT) {
  const int chunks = D / 8;
  const int u = threadIdx.x / chunks, c = threadIdx.x % chunks;
  const int blk = blockIdx.x * 8 + u;
  const int h = blockIdx.y, b = blockIdx.z >> 1;
  const bool is_k = blockIdx.z & 1;
  const int bh = b * H + h;
  const int S = is_k ? Sk : Sq;
  const int nb = is_k ? nbk : nbq;
  if (u >= 8 || blk >= nb) return;
  const mi_tensor4& t = is_k ? k : q;
  const uint16_t* base = reinterpret_cast<const uint16_t*>(t.ptr) + (long long)b * t.stride_b +
                         (long long)view_head(t, h) * t.stride_h + (long long)blk * 64 * t.stride_s +
                         c * 8;
  const int rn = min(64, S - blk * 64);
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll 1
  for (int r0 = 0; r0 < 64; r0 += 16) {
    uint4 raw[16];
#pragma unroll
    for (int r = 0; r < 16; ++r)
      raw[r] = (r0 + r < rn) ? *reinterpret_cast<const uint4*>(base + (long long)(r0 + r) * t.stride_s)
                             : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const uint16_t* hv = reinterpret_cast<const uint16_t*>(&raw[r]);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], DType<DT>::to_f(hv[e]));
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float pooled = DType<DT>::round(__fdiv_rn(acc[e], 64.f));
    const int d = c * 8 + e;
    if (is_k)
      k_poolT[((long long)bh * D + d) * nbk + blk] = pooled;
    else
      q_pool[((long long)bh * nbq + blk) * D + d] = pooled;
  }
}

// ---------------------------------------------------------------------------
// K2: scores + top-k for kRows consecutive query blocks of one (b, h).
// score(bq, kb) = fmaf chain over d = 0..D-1 of q_pool[bq][d] * k_pool[kb][d],
// times score_scale; key blocks kb > bq score -inf; with force_sink_diag
// blocks 0 and bq rank above everything.  Every pooled-K value read from L2
// serves kRows query blocks.  Then warp w selects the top-k of row w.
// Dynamic shared memory: kRows * nbk keys + kRows * D floats.
// ---------------------------------------------------------------------------
constexpr int kSelThreads = 256;
constexpr int kSelRows = 8;        // query blocks per CTA (one selecting warp each)
constexpr int kMaxBlocks = 8192;   // S up to 512K tokens

__global__ void __launch_bounds__(kSelThreads) block_select_kernel(
    const float* q_pool, const float* k_poolT, int H, int D, int nbq, int nbk, int topk,
    int force_sink_diag, float score_scale, int64_t* out_idx) {
  extern __shared__ uint32_t sel_smem[];
  uint32_t* keys = sel_smem;                                          // [kSelRows][nbk]
  float* qv = reinterpret_cast<float*>(sel_smem + kSelRows * nbk);    // [kSelRows][D]
  __shared__ int hist[kSelRows][256];
  const int bq0 = blockIdx.x * kSelRows, h = blockIdx.y, b = blockIdx.z;
  const int bh = b * H + h;
  const int rows = min(kSelRows, nbq - bq0);
  for (int e = threadIdx.x; e < kSelRows * D; e += kSelThreads) {
    const int r = e / D, d = e % D;
    qv[e] = (r < rows) ? q_pool[((long long)bh * nbq + bq0 + r) * D + d] : 0.f;
  }
  __syncthreads();
  const float* kp = k_poolT + (long long)bh * D * nbk;
  const uint32_t kNegInf = float_to_ordered(-INFINITY);
  const int last_bq = bq0 + rows - 1;
  for (int kb = threadIdx.x; kb < nbk; kb += kSelThreads) {
    float acc[kSelRows];
#pragma unroll
    for (int r = 0; r < kSelRows; ++r) acc[r] = 0.f;
    if (kb <= last_bq) {
      // Unrolled so that several pooled-K loads (L2) are in flight ahead of
      // their fmaf steps; each row's chain still runs over d in order.
#pragma unroll 8
      for (int d = 0; d < D; ++d) {
        const float kv = kp[(long long)d * nbk + kb];
#pragma unroll
        for (int r = 0; r < kSelRows; ++r) acc[r] = __fmaf_rn(qv[r * D + d], kv, acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < kSelRows; ++r) {
      const int bq = bq0 + r;
      uint32_t key = (kb > bq) ? kNegInf : float_to_ordered(__fmul_rn(acc[r], score_scale));
      if (force_sink_diag && (kb == 0 || kb == bq)) key = 0xFFFFFFFFu;
      keys[r * nbk + kb] = key;
    }
  }
  __syncthreads();
  const int w = threadIdx.x >> 5;
  if (w < rows) {
    const int kk = min(topk, nbk);
    int64_t* dst = out_idx + ((long long)bh * nbq + bq0 + w) * kk;
    warp_topk(keys + w * nbk, nbk, kk, hist[w], [&](int pos, int idx) { dst[pos] = idx; });
  }
}

// ---------------------------------------------------------------------------
// Plan for the attention kernel: for query tile t (query blocks 2t, 2t+1),
// the ascending union of both blocks' key-block lists, restricted to
// kb <= bq (blocks after the query block are fully masked by causality).
// One warp per tile.  Mask m_h = all ones when block kb is selected by
// query block 2t+h, else 0.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) bs_plan_kernel(const int64_t* idx, int H, int nbq,
                                                      int nbk, int topk, int T, long long cap,
                                                      long long head_stride, PlanEntry* plan,
                                                      int* plan_count) {
  __shared__ uint32_t bits[4][2][kMaxBlocks / 32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + w;
  const int h = blockIdx.y, b = blockIdx.z;
  const int bh = b * H + h;
  if (t >= T) return;
  const int hi = min(2 * t + 1, nbk - 1);  // last key block any row of the tile can see
  const int nwords = hi / 32 + 1;
  for (int i = lane; i < nwords; i += 32) {
    bits[w][0][i] = 0;
    bits[w][1][i] = 0;
  }
  __syncwarp();
  for (int half = 0; half < 2; ++half) {
    const int bq = 2 * t + half;
    if (bq >= nbq) break;
    const int64_t* lst = idx + ((long long)bh * nbq + bq) * topk;
    for (int i = lane; i < topk; i += 32) {
      const long long kb = lst[i];
      if (kb >= 0 && kb <= bq && kb <= hi) atomicOr(&bits[w][half][kb >> 5], 1u << (kb & 31));
    }
  }
  __syncwarp();
  PlanEntry* out = plan + (long long)bh * head_stride + plan_offset(t, cap);
  int count = 0;
  for (int base = 0; base <= hi; base += 32) {
    const int kb = base + lane;
    const uint32_t w0 = bits[w][0][base >> 5], w1 = bits[w][1][base >> 5];
    const bool s0 = (kb <= hi) && ((w0 >> lane) & 1u);
    const bool s1 = (kb <= hi) && ((w1 >> lane) & 1u);
    const unsigned any = __ballot_sync(0xffffffffu, s0 || s1);
    if (s0 || s1) {
      const int pos = count + __popc(any & ((1u << lane) - 1u));
      PlanEntry e;
      e.kb = kb;
      e.kb1 = kb;
      e.m0 = s0 ? ~0ull : 0ull;
      e.m1 = s1 ? ~0ull : 0ull;
      out[pos] = e;
    }
    count += __popc(any);
  }
  if (lane == 0) plan_count[(long long)bh * T + t] = count;
}

// ---------------------------------------------------------------------------
// Split plan: entry i of tile t pairs the i-th selected key block of query
// block 2t (rows [0,64) of the tile) with the i-th of query block 2t+1 (rows
// [64,128)); each half's list is ascending, restricted to kb <= bq.  The
// tile has max(n0, n1) entries instead of |union|.  A half whose list is
// shorter gets key block 0 with mask 0 (a valid block, so V holds finite
// values where P is 0).  One warp per tile.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) bs_split_plan_kernel(const int64_t* idx, int H, int nbq,
                                                            int nbk, int topk, int T, long long cap,
                                                            long long head_stride,
                                                            PlanEntry* plan, int* plan_count) {
  __shared__ uint32_t bits[4][2][kMaxBlocks / 32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + w;
  const int h = blockIdx.y, b = blockIdx.z;
  const int bh = b * H + h;
  if (t >= T) return;
  const int hi = min(2 * t + 1, nbk - 1);
  const int nwords = hi / 32 + 1;
  for (int i = lane; i < nwords; i += 32) {
    bits[w][0][i] = 0;
    bits[w][1][i] = 0;
  }
  __syncwarp();
  for (int half = 0; half < 2; ++half) {
    const int bq = 2 * t + half;
    if (bq >= nbq) break;
    const int64_t* lst = idx + ((long long)bh * nbq + bq) * topk;
    for (int i = lane; i < topk; i += 32) {
      const long long kb = lst[i];
      if (kb >= 0 && kb <= bq && kb <= hi) atomicOr(&bits[w][half][kb >> 5], 1u << (kb & 31));
    }
  }
  __syncwarp();
  PlanEntry* out = plan + (long long)bh * head_stride + plan_offset(t, cap);
  int count[2] = {0, 0};
  for (int half = 0; half < 2; ++half) {
    for (int base = 0; base <= hi; base += 32) {
      const int kb = base + lane;
      const bool sel = (kb <= hi) && ((bits[w][half][base >> 5] >> lane) & 1u);
      const unsigned any = __ballot_sync(0xffffffffu, sel);
      if (sel) {
        PlanEntry* e = out + count[half] + __popc(any & ((1u << lane) - 1u));
        if (half == 0) {
          e->kb = kb;
          e->m0 = ~0ull;
        } else {
          e->kb1 = kb;
          e->m1 = ~0ull;
        }
      }
      count[half] += __popc(any);
    }
  }
  const int n = max(count[0], count[1]);
  for (int i = count[0] + lane; i < n; i += 32) {
    out[i].kb = 0;
    out[i].m0 = 0ull;
  }
  for (int i = count[1] + lane; i < n; i += 32) {
    out[i].kb1 = 0;
    out[i].m1 = 0ull;
  }
  if (lane == 0) plan_count[(long long)bh * T + t] = n;
}

// ---------------------------------------------------------------------------
// Host entry points
// ---------------------------------------------------------------------------

int launch_attention(const mi_tensor4& q, const mi_tensor4& k, const mi_tensor4& v,
                     const mi_tensor4& out, int64_t D, int dtype, AttnParams prm,
                     cudaStream_t stream);

}  // namespace mib200

using namespace mib200;

// Bytes of one pooled tensor (4-byte floats, B*H*nb*D of them), or SIZE_MAX
// when an argument is negative or the product does not fit in size_t.
static size_t pooled_bytes(int64_t B, int64_t H, int64_t nb, int64_t D) {
  if (B < 0 || H < 0 || nb < 0 || D < 0) return SIZE_MAX;
  unsigned __int128 n = (unsigned __int128)B * (uint64_t)H;
  n *= (uint64_t)nb;
  n *= (uint64_t)D;
  n *= sizeof(float);
  if (n > (unsigned __int128)(SIZE_MAX / 2)) return SIZE_MAX;
  return align_up((size_t)n);
}

extern "C" size_t mi_block_pool_topk_workspace_size(int64_t B, int64_t H, int64_t S_q,
                                                    int64_t S_k, int64_t D) {
  if (S_q < 0 || S_k < 0 || S_q > ((int64_t)1 << 40) || S_k > ((int64_t)1 << 40)) return SIZE_MAX;
  const int64_t nbq = (S_q + 63) / 64, nbk = (S_k + 63) / 64;
  const size_t a = pooled_bytes(B, H, nbq, D), b = pooled_bytes(B, H, nbk, D);
  if (a == SIZE_MAX || b == SIZE_MAX) return SIZE_MAX;
  return a + b;
}

extern "C" int mi_block_pool_topk(mi_tensor4 q, mi_tensor4 k, int64_t B, int64_t H, int64_t S_q,
                                  int64_t S_k, int64_t D, int dtype, int64_t topk,
                                  int force_sink_diag, float score_scale, int64_t* out_idx,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != MI_F16 && dtype != MI_BF16) return MI_ERR_DTYPE;
  if (B < 0 || H < 0 || S_q < 0 || S_k < 0 || D <= 0 || D > 128 || topk < 1) return MI_ERR_SHAPE;
  if (q.stride_d != 1 || k.stride_d != 1) return MI_ERR_SHAPE;
  const int64_t nbq = (S_q + 63) / 64, nbk = (S_k + 63) / 64;
  if (nbk > kMaxBlocks || nbq > 65535 * kSelRows) return MI_ERR_SHAPE;
  if (B == 0 || H == 0 || nbq == 0) return MI_OK;
  if (nbk == 0) return MI_ERR_SHAPE;
  if (workspace_bytes < mi_block_pool_topk_workspace_size(B, H, S_q, S_k, D) || !workspace)
    return MI_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* q_pool = reinterpret_cast<float*>(workspace);
  float* k_poolT = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                            align_up(sizeof(float) * B * H * nbq * D));
  const bool vec_ok = (D % 8 == 0) && !(reinterpret_cast<uintptr_t>(q.ptr) & 15) &&
                      !(reinterpret_cast<uintptr_t>(k.ptr) & 15) && !(q.stride_s % 8) &&
                      !(k.stride_s % 8) && !(q.stride_h % 8) && !(k.stride_h % 8) &&
                      !(q.stride_b % 8) && !(k.stride_b % 8);
  if (vec_ok) {
    dim3 g1((unsigned)((max(nbq, nbk) + 7) / 8), (unsigned)H, (unsigned)(2 * B));
    const int nthr = 8 * (int)(D / 8);
    if (dtype == MI_BF16)
      pool_kernel_v<__nv_bfloat16><<<g1, nthr, 0, st>>>(q, k, (int)H, (int)S_q, (int)S_k, (int)D,
                                                        (int)nbq, (int)nbk, q_pool, k_poolT);
    else
      pool_kernel_v<__half><<<g1, nthr, 0, st>>>(q, k, (int)H, (int)S_q, (int)S_k, (int)D,
                                                 (int)nbq, (int)nbk, q_pool, k_poolT);
  } else {
    dim3 g1((unsigned)max(nbq, nbk), (unsigned)H, (unsigned)B);
    if (dtype == MI_BF16)
      pool_kernel<__nv_bfloat16><<<g1, 256, 0, st>>>(q, k, (int)H, (int)S_q, (int)S_k, (int)D,
                                                     (int)nbq, (int)nbk, q_pool, k_poolT);
    else
      pool_kernel<__half><<<g1, 256, 0, st>>>(q, k, (int)H, (int)S_q, (int)S_k, (int)D,
                                              (int)nbq, (int)nbk, q_pool, k_poolT);
  }
  const size_t smem2 = (size_t)kSelRows * nbk * 4 + (size_t)kSelRows * D * 4;
  if (smem2 > 200 * 1024) return MI_ERR_SHAPE;  // ~S > 400K tokens
  if (cudaFuncSetAttribute(block_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem2) != cudaSuccess)
    return MI_ERR_LAUNCH;
  dim3 g2((unsigned)((nbq + kSelRows - 1) / kSelRows), (unsigned)H, (unsigned)B);
  block_select_kernel<<<g2, kSelThreads, smem2, st>>>(q_pool, k_poolT, (int)H, (int)D, (int)nbq,
                                                      (int)nbk, (int)topk, force_sink_diag,
                                                      score_scale, out_idx);
  return cudaGetLastError() == cudaSuccess ? MI_OK : MI_ERR_LAUNCH;
}

static inline int64_t bs_cap(int64_t topk) {
  int64_t cap = 2 * topk;
  return cap < 2 ? 2 : cap;
}

extern "C" size_t mi_block_sparse_fwd_workspace_size(int64_t B, int64_t H, int64_t S,
                                                     int64_t topk) {
  const int64_t nb = (S + 63) / 64, T = (S + 127) / 128;
  (void)nb;
  const int64_t per_head = plan_offset(T, bs_cap(topk));
  return align_up(sizeof(PlanEntry) * B * H * per_head) + align_up(sizeof(int) * B * H * T);
}

extern "C" int mi_block_sparse_fwd_rows(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v,
                                        mi_tensor4 out, int64_t B, int64_t H, int64_t S,
                                        int64_t D, int dtype, const int64_t* block_idx,
                                        int64_t topk, float softmax_scale, int64_t row_begin,
                                        int64_t row_end, void* workspace, size_t workspace_bytes,
                                        void* stream) {
  if (dtype != MI_F16 && dtype != MI_BF16) return MI_ERR_DTYPE;
  if (B < 0 || H < 0 || S < 0 || topk < 1) return MI_ERR_SHAPE;
  if (D != 64 && D != 96 && D != 128) return MI_ERR_SHAPE;
  const int64_t nb = (S + 63) / 64, T = (S + 127) / 128;
  if (nb > kMaxBlocks || B > 65535 || H > 65535) return MI_ERR_SHAPE;
  if (!row_window_ok(row_begin, row_end, S)) return MI_ERR_SHAPE;
  if (B == 0 || H == 0 || S == 0 || row_begin == row_end) return MI_OK;
  if (workspace_bytes < mi_block_sparse_fwd_workspace_size(B, H, S, topk) || !workspace)
    return MI_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t cap = bs_cap(topk);
  const int64_t head_stride = plan_offset(T, cap);
  PlanEntry* plan = reinterpret_cast<PlanEntry*>(workspace);
  int* count = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) +
                                      align_up(sizeof(PlanEntry) * B * H * head_stride));
  dim3 g((unsigned)((T + 3) / 4), (unsigned)H, (unsigned)B);
  // Split tiles (default): each 64-row query block walks its own list.
  // MI_BS_SPLIT=0 selects union tiles (both halves walk the union of the
  // two lists), kept for comparison.
  static const bool split = [] {
    const char* e = getenv("MI_BS_SPLIT");
    return !(e && e[0] == '0');
  }();
  if (split)
    bs_split_plan_kernel<<<g, 128, 0, st>>>(block_idx, (int)H, (int)nb, (int)nb, (int)topk,
                                            (int)T, cap, head_stride, plan, count);
  else
    bs_plan_kernel<<<g, 128, 0, st>>>(block_idx, (int)H, (int)nb, (int)nb, (int)topk, (int)T,
                                      cap, head_stride, plan, count);
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
  prm.plan = plan;
  prm.plan_count = count;
  prm.plan_cap = cap;
  prm.plan_head_stride = head_stride;
  prm.split = split ? 1 : 0;
  prm.t_lo = (int)(row_begin / 128);
  prm.t_n = (int)((row_end + 127) / 128) - prm.t_lo;
  return launch_attention(q, k, v, out, D, dtype, prm, st);
}

extern "C" int mi_block_sparse_fwd(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out,
                                   int64_t B, int64_t H, int64_t S, int64_t D, int dtype,
                                   const int64_t* block_idx, int64_t topk, float softmax_scale,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  return mi_block_sparse_fwd_rows(q, k, v, out, B, H, S, D, dtype, block_idx, topk, softmax_scale,
                                  0, S, workspace, workspace_bytes, stream);
}
