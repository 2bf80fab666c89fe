/*
 * minference_b200.h - C ABI of the B200 (sm_100a) dynamic sparse prefill
 * attention library (libminference_b200.so).
 *
 * Every entry point takes device pointers, int64 shapes and element strides,
 * a dtype enum, an explicit softmax scale, caller-owned workspace and a
 * cudaStream_t (passed as void*), and returns an int status (MI_OK = 0).
 * Work is enqueued on `stream`; nothing synchronises and nothing allocates.
 * Layout of q/k/v/out is BNSD ([B, H, S, D]) addressed through the strides,
 * so views produced by index_select / transpose can be passed directly.
 *
 * The functions replace the device work behind these reference entry points
 * (paths relative to the MInference-NPU project root):
 *   mi_stream_fwd         minference/ops/streaming_kernel_npu.py:349-397
 *                         (streaming_forward; band FA + sink FA + LSE merge
 *                          at :233-341 become one kernel)
 *   mi_dense_fwd          minference/backend_npu/attention.py:192-293
 *                         (dense_attention, prefill_dense, decode_dense)
 *   mi_block_pool_topk    minference/ops/block_sparse_kernel_npu.py:230-263
 *                         (_select_block_sparse_topk_indices)
 *   mi_block_sparse_fwd   minference/ops/block_sparse_kernel_npu.py:452-601
 *                         (_block_sparse_tilelang_npu_with_indices) with the
 *                         mask semantics of :266-348
 *   mi_vs_estimate        minference/modules/minference_forward.py:124-167
 *                         (sum_all_diagonal_matrix + _vertical_and_slash_kernel
 *                          index estimation)
 *   mi_vs_sparse_fwd      minference/ops/vertical_slash_kernel_npu.py:255-415
 *                         (_build_vs_mask_direct + _vertical_slash_pytorch_ref)
 *   mi_vs_convert_indexes minference/backend_npu/cuda_shim.py:147-236
 *                         (convert_vertical_slash_indexes, legacy format)
 */
#ifndef MINFERENCE_B200_H_
#define MINFERENCE_B200_H_

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MI_OK 0
#define MI_ERR_SHAPE 1       /* unsupported or inconsistent shape / argument */
#define MI_ERR_DTYPE 2       /* dtype not fp16/bf16 */
#define MI_ERR_WORKSPACE 3   /* workspace pointer null or too small */
#define MI_ERR_LAUNCH 4      /* CUDA launch / driver error */
#define MI_ERR_ALIGN 5       /* pointer or stride alignment not usable by TMA */
#define MI_ERR_DEVICE 6      /* not an sm_100 device */
#define MI_ERR_SCRATCH_LIMIT 7 /* problem needs more than the built-in scratch */

/* Element types of q/k/v/out. */
#define MI_F16 0
#define MI_BF16 1

/* A BNSD tensor view: device pointer plus element strides of B, H, S, D.
 * The D stride must be 1.
 *
 * Head tables: with head_index == NULL, head h of a call is head h of the
 * view.  Otherwise head_index is a device array of int32 with one entry per
 * head of the call, and head h of the call is head head_index[h] of the view
 * (0 <= head_index[h] < head_extent, the number of heads the view holds).
 * One launch then serves a non-contiguous set of heads -- the heads of one
 * pattern in a layer -- reading and writing them in place, where the
 * reference gathers them with index_select and scatters with index_copy_
 * (minference/modules/minference_forward.py:423-487).  All tensors of a call
 * (q, k, v and out) must use the same table. */
typedef struct mi_tensor4 {
  void* ptr;
  int64_t stride_b, stride_h, stride_s, stride_d;
  const int32_t* head_index;
  int64_t head_extent;
  /* Output replicas (for `out` of the attention entry points only; NULL / 0
   * otherwise): n_replica (at most MI_MAX_REPLICAS) more base pointers, in a
   * host array, of views with the same strides -- for instance the same
   * buffer of the other GPUs of a node, opened in this process through CUDA
   * IPC and reached over NVLink.  Every output tile is stored to `ptr` and to
   * each replica by the kernel that computes it, so a head-sharded layer's
   * output reaches every GPU without a separate all-gather.  The caller
   * orders the replicas' readers after the call (e.g. with any collective
   * on the stream after it). */
  void* const* replica;
  int64_t n_replica;
} mi_tensor4;

#define MI_MAX_REPLICAS 7

/* Library version string. */
const char* mi_version(void);

/* Reads the device-side error word (nonzero if a kernel gave up a bounded
 * wait) and clears it.  Synchronises the current device. */
int mi_get_device_error(int* code);

/* Self-test of the kernels' bounded waits (no counterpart in the reference):
 * a one-block kernel arms an mbarrier for a transaction that never arrives,
 * polls it at most spin_limit times, gives up, records device error code 120
 * (read and cleared by mi_get_device_error), writes 1 to *gave_up (a device
 * int) and returns.  Every wait in the attention kernels follows the same
 * pattern with a limit of 2^26 polls: a wait that runs out records its code
 * and the kernel unwinds instead of hanging.  Nothing faults or traps. */
int mi_selftest_wait_timeout(uint32_t spin_limit, int* gave_up, void* stream);

/* stream_llm: a query at absolute position i (= S_k - S_q + row) sees keys
 * j <= i with j < n_init or j > i - n_local.  Dense causal attention is the
 * special case n_init = 0, n_local >= S_k.  Sink and window are handled in one
 * online-softmax pass (no separate LSE merge).
 * Replaces streaming_forward (streaming_kernel_npu.py:349). */
int mi_stream_fwd(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out, int64_t B,
                  int64_t H, int64_t S_q, int64_t S_k, int64_t D, int dtype, int64_t n_init,
                  int64_t n_local, float softmax_scale, void* stream);

/* Dense attention, causal (bottom-right aligned when S_q < S_k: row r sees
 * keys j <= S_k - S_q + r) or not causal (every row sees all S_k keys).  The
 * caller passes the scale; the reference's default is 1/sqrt(D) of the
 * unpadded head dim.  Runs on the same kernel as mi_stream_fwd.
 * Replaces dense_attention / prefill_dense / decode_dense
 * (minference/backend_npu/attention.py:192-211, :243-255, :274-293). */
int mi_dense_fwd(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out, int64_t B, int64_t H,
                 int64_t S_q, int64_t S_k, int64_t D, int dtype, int causal, float softmax_scale,
                 void* stream);

/* block_sparse selector: mean-pools q and k over 64-row blocks (block_size
 * must be 64), scores q_pool . k_pool^T * score_scale with future blocks at
 * -inf, keeps the top `topk` key blocks per query block (ties -> lower block
 * index) and writes them in ascending order to out_idx, int64
 * [B, H, ceil(S_q/64), min(topk, ceil(S_k/64))], contiguous.
 * force_sink_diag != 0 additionally forces block 0 and the diagonal block in.
 * The workspace size is SIZE_MAX for negative or overflowing sizes.
 * Replaces _select_block_sparse_topk_indices (block_sparse_kernel_npu.py:230). */
size_t mi_block_pool_topk_workspace_size(int64_t B, int64_t H, int64_t S_q, int64_t S_k,
                                         int64_t D);
int mi_block_pool_topk(mi_tensor4 q, mi_tensor4 k, int64_t B, int64_t H, int64_t S_q,
                       int64_t S_k, int64_t D, int dtype, int64_t topk, int force_sink_diag,
                       float score_scale, int64_t* out_idx, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Allocation-free variant of mi_block_pool_topk.  No counterpart in the
 * reference.  It is meant for callers that cannot allocate device memory when
 * they call in -- code being captured into a CUDA graph, or engines that have
 * given the whole device heap to their own pool -- so instead of taking a
 * workspace it uses a fixed scratch array compiled into the library
 * (mi_block_pool_topk_noalloc_limit() bytes, 32 MiB, held on every GPU that
 * loads the library until the process exits).  Same arguments and results as
 * mi_block_pool_topk without the workspace; returns MI_ERR_SCRATCH_LIMIT when
 * mi_block_pool_topk_workspace_size(...) exceeds the limit.  The first call on
 * each device looks up the array's device address (cudaGetSymbolAddress), so
 * make that first call before any stream capture.  All calls share the one
 * array: calls that overlap on the GPU race and must be serialised by the
 * caller.  Allocates nothing (no cudaMalloc / cudaFree). */
size_t mi_block_pool_topk_noalloc_limit(void);
int mi_block_pool_topk_noalloc(mi_tensor4 q, mi_tensor4 k, int64_t B, int64_t H, int64_t S_q,
                               int64_t S_k, int64_t D, int dtype, int64_t topk,
                               int force_sink_diag, float score_scale, int64_t* out_idx,
                               void* stream);

/* block_sparse attention from per-query-block key-block lists:
 * block_idx int64 [B, H, ceil(S/64), topk] (any order, duplicates and
 * out-of-range entries ignored).  Causal, S_q == S_k.
 * Replaces the device path of block_sparse_attention
 * (block_sparse_kernel_npu.py:452-601, mask semantics :266-348). */
size_t mi_block_sparse_fwd_workspace_size(int64_t B, int64_t H, int64_t S, int64_t topk);
int mi_block_sparse_fwd(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out, int64_t B,
                        int64_t H, int64_t S, int64_t D, int dtype, const int64_t* block_idx,
                        int64_t topk, float softmax_scale, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Row-window variant of mi_block_sparse_fwd: computes (and writes) only
 * output rows [row_begin, row_end) -- whole 128-row tiles, except that the
 * window may end at S -- with the same visible sets as the full call; other
 * rows of `out` are left untouched.  q/k/v/out describe the whole sequence.
 * Used to split one head's query tiles over several GPUs; the full call is
 * the window [0, S).  No counterpart function in the reference (it serves
 * the same op, block_sparse_kernel_npu.py:452-601, over part of the rows). */
int mi_block_sparse_fwd_rows(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out, int64_t B,
                             int64_t H, int64_t S, int64_t D, int dtype, const int64_t* block_idx,
                             int64_t topk, float softmax_scale, int64_t row_begin,
                             int64_t row_end, void* workspace, size_t workspace_bytes,
                             void* stream);

/* vertical_and_slash index estimation from the last min(64, S) queries:
 * v_idx int32 [B, H, vertical_size] ascending, s_idx int32 [B, H, slash_size]
 * descending (s = S-1-diagonal).  Columns 0..29 and slashes 0..99 are forced
 * in.  `logit_scale` is applied as in the reference (1/sqrt(D)).
 * vertical_size / slash_size must already be clamped by the caller
 * (min(S, max(v, 30)), min(S, max(s, 50))).  q and k rows are read with
 * 16-byte loads: unit dim stride, batch/head/row strides multiples of 8
 * elements and 16-byte aligned base pointers, else MI_ERR_ALIGN.
 * Replaces _vertical_and_slash_kernel (minference_forward.py:140-167). */
size_t mi_vs_estimate_workspace_size(int64_t B, int64_t H, int64_t S);
int mi_vs_estimate(mi_tensor4 q, mi_tensor4 k, int64_t B, int64_t H, int64_t S, int64_t D,
                   int dtype, int64_t vertical_size, int64_t slash_size, float logit_scale,
                   int32_t* v_idx, int32_t* s_idx, void* workspace, size_t workspace_bytes,
                   void* stream);

/* vertical_and_slash attention (direct semantics): for query block bq
 * (64 rows, end_m = 64*(bq+1)) every slash s < end_m keeps the keys
 * [re-64, re) with re = min(max(end_m - s, 64), S); vertical columns are
 * visible to every row; everything AND causal.  v_idx / s_idx int32
 * [B, H, nv] / [B, H, ns] contiguous (any order).  S_q == S_k.
 * Replaces _build_vs_mask_direct + the masked attention
 * (vertical_slash_kernel_npu.py:255-415). */
size_t mi_vs_sparse_fwd_workspace_size(int64_t B, int64_t H, int64_t S);
int mi_vs_sparse_fwd(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out, int64_t B,
                     int64_t H, int64_t S, int64_t D, int dtype, const int32_t* v_idx,
                     int64_t nv, const int32_t* s_idx, int64_t ns, float softmax_scale,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Row-window variant of mi_vs_sparse_fwd (window rules as in
 * mi_block_sparse_fwd_rows).  No counterpart function in the reference (it
 * serves vertical_slash_kernel_npu.py:255-415 over part of the rows). */
int mi_vs_sparse_fwd_rows(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out, int64_t B,
                          int64_t H, int64_t S, int64_t D, int dtype, const int32_t* v_idx,
                          int64_t nv, const int32_t* s_idx, int64_t ns, float softmax_scale,
                          int64_t row_begin, int64_t row_end, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Legacy four-array VS index format of upstream MInference, as restated by
 * the reference's CPU port convert_vertical_slash_indexes
 * (minference/backend_npu/cuda_shim.py:147-236): per (b, h, 64-row query
 * block) the slash ranges as 64-key block offsets (merged with the upstream
 * one-block extension rule) and the vertical columns not covered by them.
 * seqlens int32 [B]; v_idx int32 [B,H,nv] ascending; s_idx int32 [B,H,ns]
 * descending.  Outputs (int32, fully written): block_count [B,H,R],
 * block_offset [B,H,R,ns], column_count [B,H,R], column_index [B,H,R,nv],
 * R = ceil(context_size/64). */
int mi_vs_convert_indexes(const int32_t* seqlens, const int32_t* v_idx, int64_t nv,
                          const int32_t* s_idx, int64_t ns, int64_t B, int64_t H,
                          int64_t context_size, int32_t* block_count, int32_t* block_offset,
                          int32_t* column_count, int32_t* column_index, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINFERENCE_B200_H_ */
