// selftest.cu -- h3q_selftest_wait_timeout: runs the library's bounded-wait path on purpose.
//
// Every pipeline kernel of this library waits on mbarriers with a wall-clock limit (mbar_wait_bounded, ptx.cuh):
// a wait that gives up raises the CTA's abort flag, latches a code into an error word, lets the other roles of
// the CTA leave their own waits, frees TMEM and returns, so the context stays usable and the host reads the code
// (h3q_device_status).  In normal operation no wait runs out, so this entry point makes one run out: one CTA with
// the roles of a pipeline kernel (a producer lane, a TMEM-owning warp, two consumer warps) waits on a barrier
// that nothing ever completes.  The producer's wait has the caller's short limit; the consumers keep the
// kernels' default limit and leave because the producer raised the abort flag.  Then the CTA frees its TMEM and
// writes a completion marker.  Nothing faults, traps or spins without a limit.
#include <cstdint>
#include <cuda_runtime.h>
#include "../../include/h3q.h"
#include "ptx.cuh"
#include "h3q_internal.h"

namespace h3q {
void set_last_error(const char* msg);

namespace {

constexpr int kSelftestThreads = 128;
constexpr uint32_t kSelftestTmemCols = 32;

__global__ void __launch_bounds__(kSelftestThreads, 1)
    selftest_wait_kernel(int* err, uint64_t limit_ns, int* done) {
  __shared__ uint64_t never;  // a barrier no thread ever arrives at
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&never, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kSelftestTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  volatile int* abort_p = &abort_flag;
  bool gave_up = false;
  if (warp == 0) {
    if (elect_one()) gave_up = !mbar_wait_bounded(&never, 0, abort_p, err, kDevTimeoutSelftest, limit_ns);
  } else if (warp >= 2) {
    // consumers: the kernels' own limit; they leave as soon as the producer has raised the abort flag
    const bool ok = mbar_wait_bounded(&never, 0, abort_p, err, kDevTimeoutSelftest);
    gave_up = !__all_sync(0xffffffffu, ok);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kSelftestTmemCols);
  }
  if (threadIdx.x == 64 && done) *done = 1;   // the CTA reached its exit path
  if (warp == 0 && gave_up && done) atomicAdd(done, 2);  // the producer's own wait gave up
}

}  // namespace
}  // namespace h3q

extern "C" h3q_status h3q_selftest_wait_timeout(int target, uint64_t limit_ns, int* done, void* stream) {
  using namespace h3q;
  if (limit_ns == 0 || limit_ns > 1000000000ull) {
    set_last_error("h3q_selftest_wait_timeout: limit_ns must be in (0, 1e9]");
    return H3Q_ERR_ARG;
  }
  int* word = nullptr;
  if (target == 0) word = error_word_current();
  else if (target == 1) word = static_status_word_current();
  else {
    set_last_error("h3q_selftest_wait_timeout: target must be 0 (device error word) or 1 (static-scratch status)");
    return H3Q_ERR_ARG;
  }
  if (!word) {
    set_last_error("h3q_selftest_wait_timeout: could not resolve the error word");
    return H3Q_ERR_CUDA;
  }
  selftest_wait_kernel<<<1, kSelftestThreads, 0, static_cast<cudaStream_t>(stream)>>>(word, limit_ns, done);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return H3Q_ERR_CUDA;
  }
  return H3Q_OK;
}
