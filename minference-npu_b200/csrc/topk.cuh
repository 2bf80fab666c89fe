// Block-wide exact top-k selection with lowest-index tie-break.
//
// Keys are order-preserving uint32 images of fp32 scores (float_to_ordered).
// The k-th largest key T is found by a 4-pass 8-bit radix select; the result
// set is then {key > T} plus the first `need` elements equal to T in index
// order, emitted in ascending index order.
//
// Warp w owns the contiguous index segment [w*seg, (w+1)*seg) and walks it
// in rounds of 32 consecutive indices, so every load is coalesced and index
// order inside a round comes from ballots.  Rounds are loaded kTopkBatch at a
// time before they are processed (in order): the keys usually come from L2,
// and one dependent load per round would serialise on its latency.  Histograms are per warp, and
// lanes holding the same digit in a round are merged with __match_any_sync
// into one add: the scores' leading bytes are shared by most keys, so a
// block-wide histogram would serialise on one or two bins.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"

namespace mib200 {

// Exclusive block scan of one int per thread; returns the exclusive prefix,
// writes the block total to *total.
template <int NT>
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  int base = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) {
    const int wt = warp_tot[w];
    if (w < warp) base += wt;
    tot += wt;
  }
  __syncthreads();
  *total = tot;
  return base + x - v;
}

constexpr int kTopkBatch = 8;

// Walks [wbeg, wend) in rounds of 32 indices; f(i, key, valid) is called once
// per round per lane, rounds in ascending order.
template <typename F>
__device__ __forceinline__ void walk_rounds(const uint32_t* keys, int wbeg, int wend, F&& f) {
  const int lane = threadIdx.x & 31;
  for (int base = wbeg; base < wend; base += 32 * kTopkBatch) {
    uint32_t kk[kTopkBatch];
#pragma unroll
    for (int u = 0; u < kTopkBatch; ++u) {
      const int i = base + u * 32 + lane;
      kk[u] = i < wend ? keys[i] : 0u;
    }
#pragma unroll
    for (int u = 0; u < kTopkBatch; ++u) {
      const int i = base + u * 32 + lane;
      if (base + u * 32 < wend) f(i, kk[u], i < wend);
    }
  }
}

template <int NT>
struct TopkSmem {
  int hist[NT / 32][256];  // per-warp digit histograms
  int tot[256];            // this CTA's histogram
  int ctot[256];           // the cluster's histogram
  int warp_cnt[NT / 32];
  int cta_cnt;
  int sel_digit;
  int remaining;
};

// Sum of warp_cnt[0..w) for the calling warp (after a block barrier).
template <int NT>
__device__ __forceinline__ int warps_before(const int* warp_cnt, int w) {
  int s = 0;
  for (int x = 0; x < w; ++x) s += warp_cnt[x];
  return s;
}

// keys: n entries (shared or global memory).  Calls emit(pos, index) for the
// k selected indices with pos = 0..k-1 in ascending index order.
//
// CL > 1: the calling CTA is one of a cluster of CL CTAs that select
// together; CTA r owns the index segment [r*cseg, (r+1)*cseg).  Per radix
// pass each CTA builds its histogram, the cluster sums them through
// distributed shared memory, and every CTA picks the same digit; the
// tie-break and output positions use cluster-wide prefix counts.  All CTAs
// of the cluster must call it with the same arguments.
template <int NT, int CL, typename Emit>
__device__ void cluster_topk(const uint32_t* keys, int n, int k, TopkSmem<NT>& sm, Emit emit) {
  namespace cg = cooperative_groups;
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const unsigned lt = (1u << lane) - 1u;
  if (k <= 0) return;
  if (k > n) k = n;
  int crank = 0;
  if constexpr (CL > 1) crank = (int)cg::this_cluster().block_rank();
  auto cluster_sync = [&]() {
    if constexpr (CL > 1) cg::this_cluster().sync();
    else __syncthreads();
  };
  // Sum over the cluster's CTAs of a shared int (the caller's own included).
  auto cluster_sum = [&](int* local, int upto_rank) -> int {
    int s = 0;
    if constexpr (CL > 1) {
      for (int r = 0; r < upto_rank; ++r) s += *cg::this_cluster().map_shared_rank(local, r);
    } else {
      if (upto_rank > 0) s = *local;
    }
    return s;
  };
  const int cseg = (((n + CL - 1) / CL) + 31) & ~31;
  const int cbeg = min(n, crank * cseg);
  const int cend = min(n, cbeg + cseg);
  const int seg = ((((cend - cbeg) + NW - 1) / NW) + 31) & ~31;
  const int wbeg = min(cend, cbeg + warp * seg);
  const int wend = min(cend, wbeg + seg);

  uint32_t prefix = 0, pmask = 0;
  if (tid == 0) sm.remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
    for (int q = 0; q < 8; ++q) sm.hist[warp][lane * 8 + q] = 0;
    __syncwarp();
    walk_rounds(keys, wbeg, wend, [&](int, uint32_t key, bool valid) {
      const int d = (valid && (key & pmask) == prefix) ? (int)((key >> shift) & 255) : 256;
      const unsigned same = __match_any_sync(0xffffffffu, d);
      if (d != 256 && lane == __ffs(same) - 1) atomicAdd(&sm.hist[warp][d], __popc(same));
    });
    __syncthreads();
    for (int b = tid; b < 256; b += NT) {
      int c = 0;
#pragma unroll 8
      for (int w = 0; w < NW; ++w) c += sm.hist[w][b];
      sm.tot[b] = c;
    }
    cluster_sync();  // every CTA's histogram is complete
    for (int b = tid; b < 256; b += NT) sm.ctot[b] = cluster_sum(&sm.tot[b], CL);
    __syncthreads();
    if (warp == 0) {
      // lane l covers digits [255-8l-7, 255-8l], scanned from the top digit down.
      int c[8];
      int s = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        c[q] = sm.ctot[255 - 8 * lane - q];
        s += c[q];
      }
      int incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int excl = incl - s;
      const int rem = sm.remaining;
      const unsigned hit = __ballot_sync(0xffffffffu, incl >= rem);
      const int first = __ffs(hit) - 1;  // always exists: total count >= rem
      if (lane == first) {
        int cum = excl;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (cum + c[q] >= rem) {
            sm.sel_digit = 255 - 8 * lane - q;
            sm.remaining = rem - cum;
            break;
          }
          cum += c[q];
        }
      }
    }
    cluster_sync();  // no CTA still reads this CTA's tot when the next pass rewrites it
    prefix |= (uint32_t)sm.sel_digit << shift;
    pmask |= 255u << shift;
  }
  const uint32_t T = prefix;
  const int need_eq = sm.remaining;

  // Elements equal to T before this warp's segment (cluster-wide).
  int eq_w = 0;
  walk_rounds(keys, wbeg, wend, [&](int, uint32_t key, bool valid) {
    eq_w += __popc(__ballot_sync(0xffffffffu, valid && key == T));
  });
  if (lane == 0) sm.warp_cnt[warp] = eq_w;
  __syncthreads();
  if (tid == 0) sm.cta_cnt = warps_before<NT>(sm.warp_cnt, NW);
  const int eq_before_warp = warps_before<NT>(sm.warp_cnt, warp);
  cluster_sync();
  const int eq_before = eq_before_warp + cluster_sum(&sm.cta_cnt, crank);
  cluster_sync();
  // Walks the segment; calls f(i, rank among this warp's selected elements)
  // for selected i.  Returns the warp's selected count.
  auto walk = [&](auto&& f) -> int {
    int eq_seen = eq_before, cnt = 0;
    walk_rounds(keys, wbeg, wend, [&](int i, uint32_t key, bool valid) {
      const bool eq = valid && key == T;
      const unsigned eqb = __ballot_sync(0xffffffffu, eq);
      const bool sel = valid && (key > T || (eq && eq_seen + __popc(eqb & lt) < need_eq));
      const unsigned selb = __ballot_sync(0xffffffffu, sel);
      if (sel) f(i, cnt + __popc(selb & lt));
      cnt += __popc(selb);
      eq_seen += __popc(eqb);
    });
    return cnt;
  };
  const int sel_w = walk([](int, int) {});
  if (lane == 0) sm.warp_cnt[warp] = sel_w;
  __syncthreads();
  if (tid == 0) sm.cta_cnt = warps_before<NT>(sm.warp_cnt, NW);
  const int pos_warp = warps_before<NT>(sm.warp_cnt, warp);
  cluster_sync();
  const int pos_base = pos_warp + cluster_sum(&sm.cta_cnt, crank);
  walk([&](int i, int r) { emit(pos_base + r, i); });
  cluster_sync();  // no CTA reads another's shared memory after it exits
}

// Warp-scope variant: the calling warp selects k of n keys on its own (no
// block barriers), with `hist` a 256-int scratch private to the warp.  Lane l
// reads indices l, l+32, ... (conflict-free in shared memory); index order
// for the tie-break and the output comes from ballots over each group of 32
// consecutive indices.  Same result as cluster_topk.
template <typename Emit>
__device__ void warp_topk(const uint32_t* keys, int n, int k, int* hist, Emit emit) {
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  if (k <= 0) return;
  if (k > n) k = n;
  uint32_t prefix = 0, pmask = 0;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
    for (int q = 0; q < 8; ++q) hist[lane * 8 + q] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const uint32_t key = keys[i];
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1);
    }
    __syncwarp();
    int c[8];
    int s = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      c[q] = hist[255 - 8 * lane - q];
      s += c[q];
    }
    int incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int excl = incl - s;
    const unsigned hit = __ballot_sync(0xffffffffu, incl >= remaining);
    const int first = __ffs(hit) - 1;
    int digit = 0, rem_new = 0;
    if (lane == first) {
      int cum = excl;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (cum + c[q] >= remaining) {
          digit = 255 - 8 * lane - q;
          rem_new = remaining - cum;
          break;
        }
        cum += c[q];
      }
    }
    digit = __shfl_sync(0xffffffffu, digit, first);
    remaining = __shfl_sync(0xffffffffu, rem_new, first);
    prefix |= (uint32_t)digit << shift;
    pmask |= 255u << shift;
    __syncwarp();
  }
  const uint32_t T = prefix;
  int eq_seen = 0, pos = 0;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const bool valid = i < n;
    const uint32_t key = valid ? keys[i] : 0u;
    const bool eq = valid && key == T;
    const unsigned eqb = __ballot_sync(0xffffffffu, eq);
    const bool sel = valid && (key > T || (eq && eq_seen + __popc(eqb & lt) < remaining));
    const unsigned selb = __ballot_sync(0xffffffffu, sel);
    if (sel) emit(pos + __popc(selb & lt), i);
    pos += __popc(selb);
    eq_seen += __popc(eqb);
  }
}

}  // namespace mib200
