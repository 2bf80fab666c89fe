// Block selector variant that allocates nothing: its scratch (the pooled Q
// and transposed pooled K of mi_block_pool_topk) lives in a fixed device
// array compiled into the library.
//
// Who needs this: code that must not call cudaMalloc on the hot path, e.g.
// work recorded into a CUDA graph (allocation is illegal during capture),
// engines that hand the whole device heap to their own pool up front and
// have nothing left for a second allocator, or latency-critical loops where
// an allocation's implicit synchronisation is not acceptable.  Such callers
// still provide q/k and the output buffer; only the scratch is built in.
//
// Cost and limits: every GPU that loads the library holds kNoAllocScratchBytes
// (32 MiB) of device memory until the process exits.  All calls share that one
// array, so calls that overlap on the GPU (different streams, or several host
// threads) race on it and must be serialised by the caller.  The array keeps
// whatever the previous call left in it; this selector overwrites every
// element it reads, so nothing needs clearing.
#include <mutex>

#include "host_util.h"

namespace mib200 {

constexpr size_t kNoAllocScratchBytes = 32ull << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch for the current device, resolved once
// per device (with that device current) and cached.  In host code the
// symbol itself is only a stand-in, never a device pointer.
static int noalloc_scratch_ptr(void** out) {
  static std::mutex mu;
  static void* cached[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return MI_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return MI_ERR_LAUNCH;
    cached[dev] = p;
  }
  *out = cached[dev];
  return MI_OK;
}

}  // namespace mib200

extern "C" size_t mi_block_pool_topk_noalloc_limit(void) { return mib200::kNoAllocScratchBytes; }

extern "C" int mi_block_pool_topk_noalloc(mi_tensor4 q, mi_tensor4 k, int64_t B, int64_t H,
                                          int64_t S_q, int64_t S_k, int64_t D, int dtype,
                                          int64_t topk, int force_sink_diag, float score_scale,
                                          int64_t* out_idx, void* stream) {
  // Argument checks first, so a bad shape reports MI_ERR_SHAPE / MI_ERR_DTYPE
  // rather than looking like a size beyond the scratch.
  if (dtype != MI_F16 && dtype != MI_BF16) return MI_ERR_DTYPE;
  if (B < 0 || H < 0 || S_q < 0 || S_k < 0 || D <= 0 || D > 128 || topk < 1) return MI_ERR_SHAPE;
  const size_t need = mi_block_pool_topk_workspace_size(B, H, S_q, S_k, D);
  if (need == SIZE_MAX) return MI_ERR_SHAPE;
  if (need > mib200::kNoAllocScratchBytes) return MI_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rc = mib200::noalloc_scratch_ptr(&scratch);
  if (rc != MI_OK) return rc;
  return mi_block_pool_topk(q, k, B, H, S_q, S_k, D, dtype, topk, force_sink_diag, score_scale,
                            out_idx, scratch, mib200::kNoAllocScratchBytes, stream);
}
