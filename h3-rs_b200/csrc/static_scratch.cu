// static_scratch.cu -- h3q_gemm_s8_static: the gemm_s8 linear for callers that cannot allocate device memory.
//
// h3q_gemm_s8 needs a workspace for the quantized activations (int8 codes + row scales) that the caller allocates.
// Some callers cannot allocate device memory at all: a plugin inside a host process that has already reserved
// the GPU's whole memory for its own pool, or code on a path where cudaMalloc's implicit device synchronisation
// and possible failure under memory pressure are not acceptable.  For them this file keeps that scratch in one
// fixed, file-scope device array of kStaticScratchBytes.  The CUDA runtime loads this file's module lazily, so
// the array is reserved on a device the first time its address is looked up there: by h3q_init(device) or by the
// first h3q_gemm_s8_static call on that device.  It is then held until the process exits.  The entry point
// itself calls no cudaMalloc, cudaFree or allocating library routine.
//
// Rules for callers:
//   * Call h3q_init(device) before taking the GPU's memory for another pool, so the array is reserved while
//     there is room for it.  Without it, the first h3q_gemm_s8_static call on a device reserves it.  Either
//     call looks the array's device address up (cudaGetSymbolAddress, once per device, with that device
//     current); make it before any stream capture.
//   * The looked-up address is kept for the life of the process: a device reset (cudaDeviceReset) after it is
//     not supported.
//   * Every call on a device shares the one array and leaves its contents behind; calls whose work overlaps
//     on the GPU (different streams without ordering between them) race on it.
//   * A problem whose codes and scales need more than the array holds is rejected with H3Q_ERR_ARG.
//   * A kernel that gives up a bounded wait latches its code into the array's own status word, not into the
//     word h3q_device_status reads.  The word is sticky: calls never clear it.
//     h3q_gemm_s8_static_status(device, &code) synchronises the device, reads it, clears it and returns
//     H3Q_ERR_TIMEOUT when it was set.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <cuda_runtime.h>
#include "../../include/h3q.h"
#include "h3q_internal.h"

namespace h3q {
void set_last_error(const char* msg);
}

namespace {

constexpr size_t kStaticScratchBytes = size_t(64) << 20;  // 64 MiB
constexpr size_t kStatusBytes = 256;                       // status word, padded to keep the codes aligned
__device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint8_t* g_scratch_dev[kMaxDevices] = {nullptr};

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

h3q_status fail(h3q_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  h3q::set_last_error(buf);
  return s;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device address of g_static_scratch on the current device; looked up once per device.  In host code the
// array's name is only a host-side stand-in, so kernels must be given this address instead.
h3q_status scratch_on_current_device(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(H3Q_ERR_CUDA, "h3q_gemm_s8_static: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(H3Q_ERR_UNSUPPORTED, "h3q_gemm_s8_static: device %d", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_dev[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return fail(H3Q_ERR_CUDA, "h3q_gemm_s8_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_dev[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch_dev[dev];
  return H3Q_OK;
}

}  // namespace

namespace h3q {
// The static-scratch status word on the current device (the array's first 4 bytes), reserving the array there if
// this is the first look-up; null when the look-up fails.
int* static_status_word_current() {
  uint8_t* base = nullptr;
  if (scratch_on_current_device(&base) != H3Q_OK) return nullptr;
  return reinterpret_cast<int*>(base);
}
}  // namespace h3q

extern "C" h3q_status h3q_gemm_s8_static_status(int device, int* code) {
  using namespace h3q;
  const char* what = "h3q_gemm_s8_static_status";
  if (code) *code = 0;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return fail(H3Q_ERR_CUDA, "%s: no device", what);
  if (cudaSetDevice(device) != cudaSuccess) return fail(H3Q_ERR_ARG, "%s: bad device %d", what, device);
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_static_scratch, sizeof(int), 0, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_static_scratch, &zero, sizeof(int), 0, cudaMemcpyHostToDevice);
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(H3Q_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  if (code) *code = v;
  if (v) return fail(H3Q_ERR_TIMEOUT, "a kernel of h3q_gemm_s8_static on device %d gave up waiting (code %d)", device, v);
  return H3Q_OK;
}

extern "C" h3q_status h3q_gemm_s8_static(const uint16_t* x, const int8_t* w, const float* ws, int64_t ws_numel,
                                         const float* bias, uint16_t* out, int64_t m, int64_t n, int64_t k,
                                         int swiglu, int rotate, void* stream) {
  using namespace h3q;
  const char* what = "h3q_gemm_s8_static";
  if (k % 64 != 0) return fail(H3Q_ERR_ARG, "gemm_s8: bf16 input with K %% 64 == 0 required (k = %lld)", (long long)k);
  if (m < 0 || n < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (swiglu && n % 2 != 0) return fail(H3Q_ERR_ARG, "%s: swiglu needs an even number of weight rows", what);
  if (rotate && k % 256 != 0) return fail(H3Q_ERR_ARG, "%s: ConvRot group 256 does not divide k = %lld", what, (long long)k);
  if (rotate && k / 256 > 64)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: the rotated quantizer handles k <= 16384 (k = %lld)", what, (long long)k);
  if (m == 0 || n == 0) return H3Q_OK;
  // m * k cannot wrap below: m is bounded by the array's size over k first
  if (k > 0 && m > (int64_t)(kStaticScratchBytes / (size_t)k))
    return fail(H3Q_ERR_ARG, "%s: m = %lld rows of k = %lld do not fit the fixed %zu-byte device scratch; use h3q_gemm_s8",
                what, (long long)m, (long long)k, kStaticScratchBytes);
  const size_t codes = align256((size_t)m * (size_t)k);
  const size_t need = kStatusBytes + codes + 4 * (size_t)m;
  if (need > kStaticScratchBytes)
    return fail(H3Q_ERR_ARG, "%s: m*k = %lld needs %zu bytes of the fixed %zu-byte device scratch; use h3q_gemm_s8",
                what, (long long)(m * k), need, kStaticScratchBytes);
  if (!x || !w || !ws || !out || ws_numel < 1) return fail(H3Q_ERR_ARG, "%s: null pointer or empty scale", what);
  if (!aligned16(x) || !aligned16(w) || !aligned16(out))
    return fail(H3Q_ERR_ARG, "%s: x, w and out must be 16-byte aligned", what);
  const int64_t nout = swiglu ? n / 2 : n;
  if ((nout * 2) % 16 != 0)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: this build needs output rows of a multiple of 16 bytes", what);

  uint8_t* base = nullptr;
  if (h3q_status s = scratch_on_current_device(&base)) return s;
  int* status = reinterpret_cast<int*>(base);
  int8_t* qa = reinterpret_cast<int8_t*>(base + kStatusBytes);
  float* xs = reinterpret_cast<float*>(base + kStatusBytes + codes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // The codes and scales are fully rewritten below.  The status word starts at zero (static storage) and only
  // h3q_gemm_s8_static_status clears it, so a time-out stays visible until the caller reads it.
  // The quantizer h3q_gemm_s8 selects (kernels.rs:1139): rot2 order for bf16 with k/256 <= 56, else rot order.
  const int order = !rotate ? 0 : (k % 256 == 0 && k / 256 <= 56 ? 2 : 1);
  cudaError_t e = launch_quant_rows(x, 2, qa, xs, m, k, order, status, st);
  if (e == cudaSuccess) {
    GemmArgs g{};
    g.M = m; g.N = n; g.K = k;
    g.xs = xs; g.ws = ws; g.ws_per_row = (ws_numel == n && n > 1) ? 1 : 0;
    g.bias = bias; g.out = out; g.out_kind = 2; g.epi = swiglu ? kEpiSwigluPairs : kEpiLinear;
    g.err = status;
    e = launch_gemm_i8(qa, w, g, st);
  }
  if (e != cudaSuccess) return fail(H3Q_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return H3Q_OK;
}
