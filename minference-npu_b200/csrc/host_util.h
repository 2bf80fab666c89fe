// Host-side helpers: TMA tensor-map construction for BNSD views.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <cstdio>
#include <cstdlib>

#include "../../include/minference_b200.h"

namespace mib200 {

inline size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }

// A query-row window [row_begin, row_end) of an S-row sequence that the
// attention launch can restrict itself to: whole 128-row tiles, except that
// the window may end at S.
inline bool row_window_ok(int64_t row_begin, int64_t row_end, int64_t S) {
  if (row_begin < 0 || row_end < row_begin || row_end > S) return false;
  return row_begin % 128 == 0 && (row_end % 128 == 0 || row_end == S);
}

// cuTensorMapEncodeTiled is fetched through the runtime's driver entry point
// so the library does not link libcuda directly.
inline PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) ==
            cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 4-D map over a [B, H, S, D] view of 16-bit elements with a box of
// box_d x box_s elements (box_d * 2 == 64 bytes, 64-byte swizzle).
// Rows beyond S read as zeros.
inline int make_bnsd_map(CUtensorMap* map, const mi_tensor4& t, int64_t B, int64_t H, int64_t S,
                         int64_t D, int box_d, int box_s) {
  auto enc = get_encode_tiled();
  if (!enc) return MI_ERR_LAUNCH;
  if (t.stride_d != 1) return MI_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(t.ptr) & 15) return MI_ERR_ALIGN;
  const int64_t es = 2;
  if (t.head_index) {  // the map spans every head of the view; the kernel picks them
    if (t.head_extent < 1) return MI_ERR_SHAPE;
    H = t.head_extent;
  }
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  int64_t st[3] = {t.stride_s * es, t.stride_h * es, t.stride_b * es};
  cuuint64_t strides[3];
  int64_t span = D * es;  // bytes covered by the inner dimensions so far
  for (int i = 0; i < 3; ++i) {
    if (dims[i + 1] == 1) st[i] = ((span + 15) / 16) * 16;  // stride of a size-1 dim is unused
    if (st[i] <= 0 || st[i] % 16) return MI_ERR_ALIGN;
    strides[i] = (cuuint64_t)st[i];
    const int64_t ext = st[i] * (int64_t)dims[i + 1];
    if (ext > span) span = ext;
  }
  cuuint32_t box[4] = {(cuuint32_t)box_d, (cuuint32_t)box_s, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, t.ptr, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MI_OK : MI_ERR_ALIGN;
}

// 2-D map over `rows` rows of D 16-bit elements, `row_stride` elements apart,
// with a box of box_d x 1 (the shape tile::gather4 loads take); 64-byte
// swizzle like the 4-D maps.
inline int make_rows_map(CUtensorMap* map, void* ptr, int64_t rows, int64_t row_stride,
                         int64_t D, int box_d) {
  auto enc = get_encode_tiled();
  if (!enc) return MI_ERR_LAUNCH;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (row_stride * 2) % 16 || rows <= 0 ||
      rows >= (1ll << 31))
    return MI_ERR_ALIGN;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_d, 1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, ptr, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MI_OK : MI_ERR_ALIGN;
}

// With MI_DEBUG=1 in the environment, a failed kernel launch prints the CUDA
// error and the kernel's resource attributes to stderr (the C ABI itself only
// returns MI_ERR_LAUNCH).
inline void debug_launch_failure(const char* name, const void* func, cudaError_t err,
                                 int threads, int smem_bytes) {
  const char* dbg = getenv("MI_DEBUG");
  if (!dbg || dbg[0] != '1') return;
  cudaFuncAttributes fa{};
  cudaFuncGetAttributes(&fa, func);
  fprintf(stderr,
          "[minference_b200] %s launch failed: %s (threads %d, dynamic smem %d; kernel: %d regs, "
          "max threads %d, static smem %zu, local %zu)\n",
          name, cudaGetErrorString(err), threads, smem_bytes, fa.numRegs, fa.maxThreadsPerBlock,
          fa.sharedSizeBytes, fa.localSizeBytes);
}

}  // namespace mib200
