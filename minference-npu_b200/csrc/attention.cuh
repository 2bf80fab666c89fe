// Sparse FlashAttention forward for sm_100a: one kernel serves all three
// MInference patterns plus dense causal attention.
//
// Work unit: one CTA = one (batch, head, 128-row query tile).  The tile walks
// a list of 64-key KV blocks ("entries"); each entry carries one 64-bit
// column mask per 64-row half of the query tile, so the kernel computes the
// exact token-level visible set of every pattern:
//   * stream_llm / dense (mode 0): entries are generated arithmetically
//     (sink blocks, then the band blocks that are not sink blocks); sink and
//     window predicates are evaluated per element, so the sink and local
//     partial softmaxes merge inside one online softmax (no LSE merge pass).
//   * block_sparse and vertical_and_slash (mode 1): entries come from a plan
//     written by the index kernels (block_sparse.cu / vs_index.cu).
//   * split tiles (block_sparse): each 64-row half of the tile walks its own
//     list; an entry names one key block per half, computed by two M=64 MMAs
//     that share the TMEM lanes (see attn_fwd_kernel).
// Causality (key <= absolute query position) is always applied per element.
//
// Warp roles (192 threads):
//   warps 0-3  softmax: each thread owns one query row of the tile; reads S
//              from TMEM, applies masks, online softmax in registers (exp2 on
//              the MUFU unit), writes P (bf16/fp16) back into the same TMEM
//              columns, rescales O in TMEM when the running max grows by more
//              than 2^8, final normalisation and TMA store of the tile.
//   warp 4     TMA producer: Q once, then K blocks and V blocks into rings
//              (K runs ahead because S = QK^T is issued one entry ahead of
//              O += PV).
//   warp 5     TMEM allocator and tcgen05.mma issuer (converged warp, one
//              elected lane issues): S = Q K^T (M=128, N=64, K=D, both
//              operands in shared memory) into a double-buffered TMEM tile;
//              O += P V (M=128, N=D+16, K=64) with P read from TMEM and V from
//              shared memory; V carries a ones column, so O column D is the
//              row sum of P.
#pragma once
#include "common.cuh"

namespace mib200 {

struct PlanEntry {
  int32_t kb;   // key block index (keys [64*kb, 64*kb+64)) of query rows [0,64)
  int32_t kb1;  // key block of query rows [64,128): equal to kb except in split tiles
  uint64_t m0;  // visible-column mask for query rows [0,64) of the tile
  uint64_t m1;  // visible-column mask for query rows [64,128) of the tile
};
static_assert(sizeof(PlanEntry) == 24, "PlanEntry layout");

// Entries of query tile t start at plan_offset(t, cap) inside a head's plan:
// tile t holds at most min(2t+2, cap) entries (cap even).
__host__ __device__ __forceinline__ int64_t plan_offset(int64_t t, int64_t cap) {
  const int64_t t0 = cap / 2;
  if (t <= t0) return t * (t + 1);
  return t0 * (t0 + 1) + (t - t0) * cap;
}

struct AttnParams {
  int B, H, Sq, Sk;
  int q_off;           // Sk - Sq: absolute position of query row 0
  int T;               // number of 128-row query tiles of the whole sequence
  int t_lo, t_n;       // this launch computes tiles [t_lo, t_lo + t_n) (the whole range by default)
  int mode;            // 0: stream/dense arithmetic entries, 1: plan entries
  long long n_init;    // sink length (mode 0; 0 in mode 1)
  long long n_local;   // window length (mode 0; 2^40, i.e. unbounded, in mode 1)
  float scale_log2;    // softmax_scale * log2(e)
  void* out;
  long long os_b, os_h, os_s;  // output element strides
  const PlanEntry* plan;       // mode 1
  const int* plan_count;       // mode 1: [B*H][T]
  long long plan_cap;          // mode 1
  long long plan_head_stride;  // mode 1: entries per (b,h)
  int split;                   // 1: split tiles (each half of the tile has its own key block)
  const int32_t* head_index;   // head table of the views, or null (see mi_tensor4)
  int n_replica;               // output replicas (see mi_tensor4), maps in ReplicaMaps
  // mode 1, gathered key groups (vertical_and_slash): a plan entry with
  // kb = kb1 = -1 - g is group g of its tile, up to 64 scattered keys loaded
  // row by row (TMA gather4 over a 2-D row view of K and V) whose positions
  // are gcols[((bh*T+t)*gmax+g)*64 ...] (-1 = empty slot); its masks are the
  // entry's m0 / m1 as for any entry.
  int gather;
  int gmax;
  const int32_t* gcols;
  long long grow_b, grow_h;    // row of key 0 of (b, h) in the 2-D row view: b*grow_b + h*grow_h
};

constexpr int kBM = 128;       // query rows per CTA
constexpr int kBN = 64;        // keys per KV block
#ifndef MI_KSTAGES
#define MI_KSTAGES 3
#endif
#ifndef MI_VSTAGES
#define MI_VSTAGES 3
#endif
constexpr int kKStages = MI_KSTAGES;  // K ring depth (K runs ahead of V)
constexpr int kVStages = MI_VSTAGES;  // V ring depth
constexpr int kThreads = 192;

// Ring depths.  A split tile stages two key blocks per entry (one per query
// half), so its rings are shallower where two CTAs share an SM (D <= 96; at
// D = 128 O needs more than half of TMEM and one CTA runs per SM).
#ifndef MI_SPLIT_KS
#define MI_SPLIT_KS 2
#endif
#ifndef MI_SPLIT_VS96
#define MI_SPLIT_VS96 1
#endif
template <int D, bool SPLIT>
struct RingDepth {
  static constexpr int K = SPLIT ? MI_SPLIT_KS : kKStages;
  static constexpr int V = SPLIT ? (D == 96 ? MI_SPLIT_VS96 : 2) : kVStages;
};

template <int D, bool SPLIT = false>
struct AttnSmem {
  static constexpr int NB = SPLIT ? 2 : 1;          // key blocks per entry
  static constexpr int KS = RingDepth<D, SPLIT>::K;
  static constexpr int VS = RingDepth<D, SPLIT>::V;
  static constexpr int NC = D / 32;                 // 64-byte chunks per row
  static constexpr int kQBytes = NC * kBM * 64;     // Q tile (reused for the output tile)
  static constexpr int kKVBytes = NC * kBN * 64;    // one K block (and the loaded part of V)
  // A V stage holds NC loaded chunks plus one constant chunk whose first column
  // is all ones: O += P V then also produces the row sums of P in O column D.
  static constexpr int kVBytes = (NC + 1) * kBN * 64;
  static constexpr int kKStage = NB * kKVBytes;     // one K ring stage
  static constexpr int kVStage = NB * kVBytes;      // one V ring stage
  static constexpr int kOCols = D + 16;             // O columns incl. the row-sum column
  // TMEM: S0 [0,64), S1 [64,128), O [128, 128+kOCols); P(j) aliases S(j&1)
  static constexpr uint32_t kTmemCols = (128 + kOCols <= 256) ? 256u : 512u;
  // The first KQ head dims of the Q tile are also staged in TMEM (columns
  // [kQCol, kQCol + KQ/2), two 16-bit elements per column): their QK K-steps
  // read A from TMEM, so they read only K from shared memory.  With both
  // operands in shared memory an M=128, N=64 MMA step is bound by
  // shared-memory bandwidth (~48 cycles for 32 cycles of tensor work);
  // with A in TMEM it runs at the tensor rate.
  static constexpr int kQCol = 128 + kOCols;
  static constexpr int KQ = ((int)kTmemCols - kQCol) / 8 * 16 < D
                                ? ((int)kTmemCols - kQCol) / 8 * 16 : D;
  static_assert(KQ % 32 == 0, "whole 32-dim chunks of Q in TMEM");
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + KS * kKStage;
  static constexpr int kBarOff = kVOff + VS * kVStage;
  // barriers: q_full, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
  //           s_full[2], p_full[2], pv_done[2], q_tmem
  static constexpr int kNumBars = 1 + 2 * KS + 2 * VS + 7;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kAbortOff = kTmemSlotOff + 4;
  static constexpr int kBytes = kAbortOff + 4;
  // +1 KiB to align the base; never less than ~80 KiB so at most two CTAs
  // share an SM (two CTAs use all 512 TMEM columns).
  static constexpr int kAlloc = (kBytes + 1024) > 80 * 1024 ? (kBytes + 1024) : 80 * 1024;
#ifndef MI_ONE_CTA_SPLIT
  static_assert(kTmemCols == 512 || kAlloc <= 113 * 1024, "two CTAs per SM");
#endif
};

// Tensor maps of the output replicas (kernel parameter).
struct ReplicaMaps {
  CUtensorMap m[MI_MAX_REPLICAS];
};

// Entry j of the current tile (identical result in every warp that asks).
struct EntrySource {
  int mode;
  // mode 0
  int nsb;         // number of sink blocks
  int band_start;  // first band block after the sink blocks
  // mode 1
  const PlanEntry* list;

  __device__ __forceinline__ void get(int j, int& kb, int& kb1, uint64_t& m0,
                                      uint64_t& m1) const {
    if (mode == 0) {
      kb = (j < nsb) ? j : band_start + (j - nsb);
      kb1 = kb;
      m0 = ~0ull;
      m1 = ~0ull;
    } else {
      const PlanEntry e = list[j];
      kb = e.kb;
      kb1 = e.kb1;
      m0 = e.m0;
      m1 = e.m1;
    }
  }
};

}  // namespace mib200
