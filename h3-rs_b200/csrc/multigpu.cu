// multigpu.cu -- C ABI of the N-split linear across the GPUs of one node (one process per GPU): peer buffers shared
// through CUDA IPC, and the GEMM whose epilogue writes its column block straight into every rank's output over
// NVLink (GEMM and all-gather in one kernel).  The host-side exchange of IPC handles and the cross-rank barrier
// after the kernel belong to the caller's process group (h3q.parallel uses torch.distributed).
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <cuda_runtime.h>
#include "../../include/h3q.h"
#include "h3q_internal.h"

namespace h3q {
void set_last_error(const char* msg);
}

namespace {

h3q_status fail(h3q_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  h3q::set_last_error(buf);
  return s;
}

h3q_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return H3Q_OK;
  return fail(H3Q_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static_assert(sizeof(cudaIpcMemHandle_t) == H3Q_PEER_HANDLE_BYTES, "IPC handle size");

}  // namespace

extern "C" {

h3q_status h3q_peer_buffer_alloc(size_t bytes, void** ptr, void* handle) {
  const char* what = "h3q_peer_buffer_alloc";
  if (!ptr || !handle || bytes == 0) return fail(H3Q_ERR_ARG, "%s: null pointer or empty size", what);
  *ptr = nullptr;
  void* p = nullptr;
  if (h3q_status s = cuda_status(cudaMalloc(&p, bytes), what)) return s;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, what);
  }
  memcpy(handle, &h, sizeof h);
  *ptr = p;
  return H3Q_OK;
}

h3q_status h3q_peer_buffer_open(const void* handle, void** ptr) {
  const char* what = "h3q_peer_buffer_open";
  if (!ptr || !handle) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), what);
}

h3q_status h3q_peer_buffer_close(void* ptr) {
  if (!ptr) return H3Q_OK;
  return cuda_status(cudaIpcCloseMemHandle(ptr), "h3q_peer_buffer_close");
}

h3q_status h3q_peer_buffer_free(void* ptr) {
  if (!ptr) return H3Q_OK;
  return cuda_status(cudaFree(ptr), "h3q_peer_buffer_free");
}

h3q_status h3q_gemm_s8_allgather(const int8_t* a, const float* xs, const int8_t* w_local, const float* ws_local,
                                 int64_t ws_numel, const float* bias_local, void* const* outs, int n_ranks, int64_t m,
                                 int64_t n_total, int64_t n_offset, int64_t n_local, int64_t k, void* stream) {
  const char* what = "h3q_gemm_s8_allgather";
  if (m < 0 || k < 0 || n_local < 0 || n_offset < 0 || n_total < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (n_ranks < 1 || n_ranks > h3q::kMaxGatherRanks)
    return fail(H3Q_ERR_ARG, "%s: %d ranks (1..%d)", what, n_ranks, h3q::kMaxGatherRanks);
  if (n_offset + n_local > n_total)
    return fail(H3Q_ERR_ARG, "%s: columns [%lld, %lld) outside %lld", what, (long long)n_offset,
                (long long)(n_offset + n_local), (long long)n_total);
  if (m == 0 || n_local == 0) return H3Q_OK;
  if (!a || !xs || !w_local || !ws_local || !outs || ws_numel < 1) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (k == 0 || k % 16 != 0)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: this build needs k %% 16 == 0 and k > 0 (k = %lld)", what, (long long)k);
  if (n_offset % 8 != 0 || n_total % 8 != 0)
    return fail(H3Q_ERR_ARG, "%s: column offset and row width must be multiples of 8 (16 bytes)", what);
  if (!aligned16(a) || !aligned16(w_local)) return fail(H3Q_ERR_ARG, "%s: int8 operands must be 16-byte aligned", what);
  for (int r = 0; r < n_ranks; ++r)
    if (!outs[r] || !aligned16(outs[r])) return fail(H3Q_ERR_ARG, "%s: output %d null or not 16-byte aligned", what, r);
  h3q::GemmArgs g{};
  g.M = m;
  g.N = n_local;
  g.K = k;
  g.xs = xs;
  g.ws = ws_local;
  g.ws_per_row = (ws_numel == n_local && n_local > 1) ? 1 : 0;
  g.bias = bias_local;
  g.out = outs[0];
  g.out_kind = 2;
  g.epi = h3q::kEpiLinear;
  g.err = h3q::error_word_current();
  if (!g.err) return fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);
  return cuda_status(h3q::launch_gemm_i8_allgather(a, w_local, g, outs, n_ranks, n_total, n_offset,
                                                   static_cast<cudaStream_t>(stream)),
                     what);
}

}  // extern "C"
