// C ABI entry points that are not tied to one pattern: version, device error
// word, and the stream_llm / dense causal attention.
#include "attention.cuh"
#include "host_util.h"

namespace mib200 {
int launch_attention(const mi_tensor4& q, const mi_tensor4& k, const mi_tensor4& v,
                     const mi_tensor4& out, int64_t D, int dtype, AttnParams prm,
                     cudaStream_t stream);
}  // namespace mib200

namespace mib200 {
// Self-test of the bounded wait: one thread arms an mbarrier for 16 bytes of
// transaction that nothing delivers, waits at most `limit` polls, records
// kSelftestWaitCode in the device error word and returns; the other threads
// of the block wait for it at __syncthreads and return too.
constexpr int kSelftestWaitCode = 120;
__global__ void selftest_wait_kernel(uint32_t limit, int* waited_out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&bar, 16);
    const bool done = mbar_wait_limit(&bar, 0, kSelftestWaitCode, limit);
    *waited_out = done ? 0 : 1;
  }
  __syncthreads();
}
}  // namespace mib200

using namespace mib200;

extern "C" const char* mi_version(void) { return "minference-b200 0.1.0 (sm_100a)"; }

extern "C" int mi_get_device_error(int* code) {
  if (!code) return MI_ERR_SHAPE;
  if (cudaDeviceSynchronize() != cudaSuccess) return MI_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return MI_ERR_LAUNCH;
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return MI_ERR_LAUNCH;
  *code = v;
  return MI_OK;
}

extern "C" int mi_stream_fwd(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out, int64_t B,
                             int64_t H, int64_t S_q, int64_t S_k, int64_t D, int dtype,
                             int64_t n_init, int64_t n_local, float softmax_scale, void* stream) {
  if (dtype != MI_F16 && dtype != MI_BF16) return MI_ERR_DTYPE;
  if (D != 64 && D != 96 && D != 128) return MI_ERR_SHAPE;
  if (B < 0 || H < 0 || S_q < 0 || S_k < 0 || S_q > S_k || S_k > (1 << 30)) return MI_ERR_SHAPE;
  if (B > 65535 || H > 65535) return MI_ERR_SHAPE;
  if (B == 0 || H == 0 || S_q == 0) return MI_OK;
  AttnParams prm{};
  prm.B = (int)B;
  prm.H = (int)H;
  prm.Sq = (int)S_q;
  prm.Sk = (int)S_k;
  prm.q_off = (int)(S_k - S_q);
  prm.T = (int)((S_q + 127) / 128);
  prm.mode = 0;
  prm.n_init = n_init < 0 ? 0 : (n_init > S_k ? S_k : n_init);
  prm.n_local = n_local < 0 ? 0 : (n_local > S_k + 1 ? S_k + 1 : n_local);
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  return launch_attention(q, k, v, out, D, dtype, prm, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mi_dense_fwd(mi_tensor4 q, mi_tensor4 k, mi_tensor4 v, mi_tensor4 out, int64_t B,
                            int64_t H, int64_t S_q, int64_t S_k, int64_t D, int dtype, int causal,
                            float softmax_scale, void* stream) {
  if (dtype != MI_F16 && dtype != MI_BF16) return MI_ERR_DTYPE;
  if (D != 64 && D != 96 && D != 128) return MI_ERR_SHAPE;
  if (B < 0 || H < 0 || S_q < 0 || S_k < 0 || S_k > (1 << 30)) return MI_ERR_SHAPE;
  if (causal && S_q > S_k) return MI_ERR_SHAPE;  // rows with no visible key
  if (B > 65535 || H > 65535) return MI_ERR_SHAPE;
  if (B == 0 || H == 0 || S_q == 0) return MI_OK;
  if (S_k == 0) return MI_ERR_SHAPE;
  AttnParams prm{};
  prm.B = (int)B;
  prm.H = (int)H;
  prm.Sq = (int)S_q;
  prm.Sk = (int)S_k;
  // Causal: bottom-right aligned, row r sits at absolute position S_k - S_q + r.
  // Not causal: every row is placed at or past the last key, so the causal
  // test j <= position passes for every key and only j < S_k bounds the walk.
  prm.q_off = causal ? (int)(S_k - S_q) : (int)(S_k - 1);
  prm.T = (int)((S_q + 127) / 128);
  prm.mode = 0;
  prm.n_init = 0;
  prm.n_local = S_k + 1 + (causal ? 0 : S_q);
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  return launch_attention(q, k, v, out, D, dtype, prm, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mi_selftest_wait_timeout(uint32_t spin_limit, int* gave_up, void* stream) {
  if (!gave_up) return MI_ERR_SHAPE;
  selftest_wait_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(spin_limit, gave_up);
  return cudaGetLastError() == cudaSuccess ? MI_OK : MI_ERR_LAUNCH;
}
