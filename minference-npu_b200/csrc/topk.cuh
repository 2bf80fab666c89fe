// Block-wide exact top-k selection with lowest-index tie-break.
//
// Keys are order-preserving uint32 images of fp32 scores (float_to_ordered).
// The k-th largest key is found by a 4-pass 8-bit radix select over
// shared-memory histograms; the result set is then {key > T} plus the first
// `need` elements equal to T in index order, emitted in ascending index order
// via two block-wide exclusive scans.  Each thread owns a contiguous chunk of
// indices, so "index order" is (thread, position in chunk).
#pragma once
#include "common.cuh"

namespace mib200 {

template <int NT>
struct TopkSmem {
  int hist[256];
  int warp_tot[NT / 32];
  int sel_digit;
  int remaining;
};

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

// keys: n entries (shared or global memory).  Calls emit(pos, index) for the
// k selected indices with pos = 0..k-1 in ascending index order.
template <int NT, typename Emit>
__device__ void block_topk(const uint32_t* keys, int n, int k, TopkSmem<NT>& sm, Emit emit) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int ept = (n + NT - 1) / NT;
  const int beg = min(n, tid * ept);
  const int end = min(n, beg + ept);
  if (k <= 0) return;
  if (k > n) k = n;

  uint32_t prefix = 0, pmask = 0;
  if (tid == 0) sm.remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += NT) sm.hist[i] = 0;
    __syncthreads();
    for (int i = beg; i < end; ++i) {
      const uint32_t key = keys[i];
      if ((key & pmask) == prefix) atomicAdd(&sm.hist[(key >> shift) & 255], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // lane l covers digits [255-8l-7, 255-8l], scanned from the top digit down.
      int c[8];
      int s = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        c[q] = sm.hist[255 - 8 * lane - q];
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
    __syncthreads();
    prefix |= (uint32_t)sm.sel_digit << shift;
    pmask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t T = prefix;
  const int need_eq = sm.remaining;

  int eq_local = 0;
  for (int i = beg; i < end; ++i) eq_local += (keys[i] == T);
  int tot;
  const int eq_before = block_exclusive_scan<NT>(eq_local, sm.warp_tot, &tot);
  int sel_local = 0;
  {
    int eq_seen = eq_before;
    for (int i = beg; i < end; ++i) {
      const uint32_t key = keys[i];
      if (key > T) {
        ++sel_local;
      } else if (key == T) {
        if (eq_seen < need_eq) ++sel_local;
        ++eq_seen;
      }
    }
  }
  const int pos0 = block_exclusive_scan<NT>(sel_local, sm.warp_tot, &tot);
  int pos = pos0;
  int eq_seen = eq_before;
  for (int i = beg; i < end; ++i) {
    const uint32_t key = keys[i];
    bool sel = false;
    if (key > T) {
      sel = true;
    } else if (key == T) {
      sel = eq_seen < need_eq;
      ++eq_seen;
    }
    if (sel) emit(pos++, i);
  }
  (void)lane;
}

// Warp-scope variant: the calling warp selects k of n keys on its own (no
// block barriers), with `hist` a 256-int scratch private to the warp.  Lane l
// reads indices l, l+32, ... (conflict-free in shared memory); index order
// for the tie-break and the output comes from ballots over each group of 32
// consecutive indices.  Same result as block_topk.
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
