// capi.cu -- the C ABI (include/h3q.h): argument checks mirroring the reference's host-side `bail!`s,
// workspace carving, per-device error word, and dispatch to the kernels.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <cuda_runtime.h>
#include "../../include/h3q.h"
#include "h3q_internal.h"

namespace h3q {
cudaError_t launch_dequant_i8(const int8_t* q, const float* scale, int per_row, void* out, int kind, int64_t rows,
                              int64_t cols, cudaStream_t st);
cudaError_t launch_dequant_nvfp4(const uint8_t* q, const uint8_t* bs, const float* g, void* out, int kind,
                                 int64_t rows, int64_t k, cudaStream_t st);
cudaError_t launch_gate_add(const void* x, const void* y, int kind, const float* gate, const uint32_t* idx, void* out,
                            int64_t S, int64_t C, cudaStream_t st);
}  // namespace h3q

using namespace h3q;

namespace {

thread_local std::string g_last_error;

h3q_status fail(h3q_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

h3q_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return H3Q_OK;
  return fail(H3Q_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
int* g_err_word[kMaxDevices] = {nullptr};

// The per-device error word kernels latch time-outs into; allocated once per device on first use.
int* error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_err_word[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_err_word[dev] = p;
  }
  return g_err_word[dev];
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// int8 codes [m,k] followed by f32 scales [m], the scale array 256-byte aligned
size_t quant_ws_bytes(int64_t m, int64_t k) { return align_up((size_t)m * (size_t)k, 256) + 4 * (size_t)m; }

h3q_status check_kind(int kind, const char* what) {
  if (kind < 0 || kind > 2) return fail(H3Q_ERR_ARG, "%s: unsupported kind %d (0 f32, 1 f16, 2 bf16)", what, kind);
  return H3Q_OK;
}

// The quantizer the reference picks (kernels.rs:1139): 2 = rot2 order, 1 = rot order, 0 = no rotation.
int rotation_order(int kind, int64_t k, int rotate) {
  if (!rotate) return 0;
  return (kind == 2 && k % 256 == 0 && k / 256 <= 56) ? 2 : 1;
}

h3q_status gemm_core(const int8_t* a, const float* xs, const int8_t* w, const float* ws, int64_t ws_numel,
                     const float* bias, void* out, int out_kind, int64_t m, int64_t n, int64_t k, int epi,
                     const float* gate, const uint32_t* gate_idx, const uint16_t* resid, cudaStream_t st,
                     const char* what) {
  if (m < 0 || n < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (m == 0 || n == 0) return H3Q_OK;
  if (!out || (epi != kEpiAccI32 && (!xs || !ws)) || (k > 0 && (!a || !w)))
    return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (epi != kEpiAccI32 && ws_numel < 1) return fail(H3Q_ERR_ARG, "%s: empty weight scale", what);
  if (k % 16 != 0) return fail(H3Q_ERR_UNSUPPORTED, "%s: this build needs k %% 16 == 0 (k = %lld)", what, (long long)k);
  if (k > 0 && (!aligned16(a) || !aligned16(w)))
    return fail(H3Q_ERR_ARG, "%s: int8 operands must be 16-byte aligned", what);
  if (!aligned16(out)) return fail(H3Q_ERR_ARG, "%s: output must be 16-byte aligned", what);
  if (epi == kEpiGateResid && (!gate || !resid || !aligned16(resid)))
    return fail(H3Q_ERR_ARG, "%s: gated residual epilogue needs gate and a 16-byte aligned residual", what);
  const int64_t nout = (epi == kEpiSwigluPairs || epi == kEpiSwigluHalves) ? n / 2 : n;
  const int oes = (epi == kEpiAccI32 || (epi == kEpiLinear && out_kind == 0) || (epi == kEpiSwigluHalves && out_kind == 0))
                      ? 4 : 2;
  if (((nout * oes) % 16) != 0)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: this build needs output rows of a multiple of 16 bytes (width %lld)", what,
                (long long)nout);
  GemmArgs g{};
  g.M = m; g.N = n; g.K = k;
  g.xs = xs; g.ws = ws; g.ws_per_row = (ws_numel == n && n > 1) ? 1 : 0;
  g.bias = bias; g.out = out; g.out_kind = out_kind; g.epi = epi;
  g.gate = gate; g.gate_idx = gate_idx; g.resid = resid;
  g.err = error_word();
  if (!g.err) return fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);
  return cuda_status(launch_gemm_i8(a, w, g, st), what);
}

}  // namespace

namespace h3q {
// Lets other translation units of the library report an error through h3q_last_error().
void set_last_error(const char* msg) { g_last_error = msg; }
int* error_word_current() { return error_word(); }
}  // namespace h3q

extern "C" {

const char* h3q_last_error(void) { return g_last_error.c_str(); }

const char* h3q_version(void) { return "h3q 0.1 (sm_100a, tcgen05 kind::i8)"; }

int h3q_available_arch(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return 0;
  return (major == 10 && minor == 0) ? 1 : 0;
}

int h3q_can_fuse_rotation(size_t k, size_t group) { return group == 256 && k % 256 == 0 && k / 256 <= 64; }

h3q_status h3q_init(int device) {
  const char* what = "h3q_init";
  if (!h3q_available_arch(device)) return fail(H3Q_ERR_UNSUPPORTED, "%s: device %d is not an sm_100 GPU", what, device);
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return fail(H3Q_ERR_CUDA, "%s: no device", what);
  if (cudaSetDevice(device) != cudaSuccess) return fail(H3Q_ERR_ARG, "%s: bad device %d", what, device);
  // the per-device state the entry points otherwise create on their first call: the device error word (a 4-byte
  // allocation), the SM count the persistent kernels size their grids by, and the fixed scratch array of
  // h3q_gemm_s8_static (its module loads lazily, so the array is reserved here rather than at that entry
  // point's first call, when the caller may already have taken the rest of the GPU's memory)
  h3q_status st = H3Q_OK;
  if (!h3q::error_word_current()) st = fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);
  h3q::sm_count(device);
  if (st == H3Q_OK && !h3q::static_status_word_current())
    st = fail(H3Q_ERR_CUDA, "%s: could not reserve the static scratch array on device %d", what, device);
  cudaSetDevice(prev);
  return st;
}

h3q_status h3q_device_status(int device, int* code) {
  if (code) *code = 0;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return fail(H3Q_ERR_CUDA, "h3q_device_status: no device");
  if (cudaSetDevice(device) != cudaSuccess) return fail(H3Q_ERR_ARG, "h3q_device_status: bad device %d", device);
  int* w = error_word();
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess && w) e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && w && v) e = cudaMemset(w, 0, sizeof(int));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_status(e, "h3q_device_status");
  if (code) *code = v;
  if (v) return fail(H3Q_ERR_TIMEOUT, "a kernel on device %d gave up waiting (code %d)", device, v);
  return H3Q_OK;
}

h3q_status h3q_quant_rows_i8(const void* x, int x_kind, int8_t* q, float* scale, int64_t m, int64_t k, int rotate,
                             void* stream) {
  const char* what = "h3q_quant_rows_i8";
  if (h3q_status s = check_kind(x_kind, what)) return s;
  if (m < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (rotate && k % 256 != 0) return fail(H3Q_ERR_ARG, "%s: ConvRot group 256 does not divide k = %lld", what, (long long)k);
  if (rotate && k / 256 > 64)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: the rotated quantizer handles k <= 16384 (k = %lld)", what, (long long)k);
  if (m == 0) return H3Q_OK;
  if (!x || !scale || (k > 0 && !q)) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  const int order = rotation_order(x_kind, k, rotate);
  if ((order != 0 || k % 256 == 0) && (!aligned16(x) || !aligned16(q)))
    return fail(H3Q_ERR_ARG, "%s: x and q must be 16-byte aligned", what);
  if (order == 0 && k % 256 == 0 && k / 256 > 64)  // wide unrotated rows take the generic kernel
    return cuda_status(launch_quant_rows(x, x_kind, q, scale, m, k, -1, error_word(), (cudaStream_t)stream), what);
  return cuda_status(launch_quant_rows(x, x_kind, q, scale, m, k, order, error_word(), (cudaStream_t)stream), what);
}

size_t h3q_gemm_s8_workspace_size(int64_t m, int64_t k) { return quant_ws_bytes(m, k); }

h3q_status h3q_gemm_s8(const uint16_t* x, const int8_t* w, const float* ws, int64_t ws_numel, const float* bias,
                       uint16_t* out, int64_t m, int64_t n, int64_t k, int swiglu, int rotate, void* workspace,
                       size_t workspace_bytes, void* stream) {
  const char* what = "h3q_gemm_s8";
  if (k % 64 != 0) return fail(H3Q_ERR_ARG, "gemm_s8: bf16 input with K %% 64 == 0 required (k = %lld)", (long long)k);
  if (m < 0 || n < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (swiglu && n % 2 != 0) return fail(H3Q_ERR_ARG, "%s: swiglu needs an even number of weight rows", what);
  if (m == 0 || n == 0) return H3Q_OK;
  if (workspace_bytes < quant_ws_bytes(m, k) || !workspace)
    return fail(H3Q_ERR_WORKSPACE, "%s: workspace of %zu bytes, need %zu", what, workspace_bytes, quant_ws_bytes(m, k));
  int8_t* qa = static_cast<int8_t*>(workspace);
  float* xs = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align_up((size_t)m * k, 256));
  if (h3q_status s = h3q_quant_rows_i8(x, 2, qa, xs, m, k, rotate, stream)) return s;
  return gemm_core(qa, xs, w, ws, ws_numel, bias, out, 2, m, n, k, swiglu ? kEpiSwigluPairs : kEpiLinear, nullptr,
                   nullptr, nullptr, (cudaStream_t)stream, what);
}

size_t h3q_int8_linear_workspace_size(int64_t m, int64_t k) { return quant_ws_bytes(m, k); }

h3q_status h3q_int8_linear_ex(const void* x, int x_kind, const int8_t* w, const float* scale, int64_t scale_numel,
                              const float* bias, void* out, int out_kind, int64_t m, int64_t n, int64_t k, int swiglu,
                              int rotate, void* workspace, size_t workspace_bytes, void* stream) {
  const char* what = "h3q_int8_linear_ex";
  if (h3q_status s = check_kind(x_kind, what)) return s;
  if (h3q_status s = check_kind(out_kind, what)) return s;
  if (m < 0 || n < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (k % 4 != 0) return fail(H3Q_ERR_ARG, "int8_linear: bad shapes %lldx%lld", (long long)m, (long long)k);
  const int64_t n_out = swiglu ? n / 2 : n;
  if (n_out % 4 != 0) return fail(H3Q_ERR_ARG, "int8_linear: output width must be a multiple of 4");
  if (m == 0 || n == 0) return H3Q_OK;
  if (workspace_bytes < quant_ws_bytes(m, k) || !workspace)
    return fail(H3Q_ERR_WORKSPACE, "%s: workspace of %zu bytes, need %zu", what, workspace_bytes, quant_ws_bytes(m, k));
  int8_t* qa = static_cast<int8_t*>(workspace);
  float* xs = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align_up((size_t)m * k, 256));
  // kernels.rs:981: the rotation applies only when k % 256 == 0 && k / 256 <= 64, through quant_rows_i8_rot
  const bool rot = rotate && k % 256 == 0 && k / 256 <= 64;
  if (!x || !xs) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (!aligned16(x)) return fail(H3Q_ERR_ARG, "%s: x must be 16-byte aligned", what);
  cudaError_t e = launch_quant_rows(x, x_kind, qa, xs, m, k, rot ? 1 : (k % 256 == 0 && k / 256 <= 64 ? 0 : -1),
                                    error_word(), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_status(e, what);
  return gemm_core(qa, xs, w, scale, scale_numel, bias, out, out_kind, m, n, k, swiglu ? kEpiSwigluHalves : kEpiLinear,
                   nullptr, nullptr, nullptr, (cudaStream_t)stream, what);
}

h3q_status h3q_gemm_s8_quantized(const int8_t* a, const float* xs, const int8_t* w, const float* ws,
                                 int64_t ws_numel, const float* bias, void* out, int out_kind, int64_t m, int64_t n,
                                 int64_t k, int epilogue, const float* gate, const uint32_t* gate_idx,
                                 const uint16_t* resid, void* stream) {
  const char* what = "h3q_gemm_s8_quantized";
  if (epilogue < 0 || epilogue > H3Q_EPI_ACC_I32) return fail(H3Q_ERR_ARG, "%s: unknown epilogue %d", what, epilogue);
  if (h3q_status s = check_kind(out_kind, what)) return s;
  if ((epilogue == H3Q_EPI_SWIGLU_PAIRS || epilogue == H3Q_EPI_SWIGLU_HALVES) && n % 2 != 0)
    return fail(H3Q_ERR_ARG, "%s: swiglu needs an even number of weight rows", what);
  const bool bf16_only = epilogue == H3Q_EPI_SWIGLU_PAIRS || epilogue == H3Q_EPI_GELU_TANH || epilogue == H3Q_EPI_GATE_RESID;
  return gemm_core(a, xs, w, ws, ws_numel, bias, out, bf16_only ? 2 : out_kind, m, n, k, epilogue, gate, gate_idx,
                   resid, (cudaStream_t)stream, what);
}

h3q_status h3q_gemm_s8_acc(const int8_t* a, const int8_t* w, int32_t* acc, int64_t m, int64_t n, int64_t k,
                           void* stream) {
  const char* what = "h3q_gemm_s8_acc";
  // the int32 epilogue reads no scales
  return gemm_core(a, nullptr, w, nullptr, 0, nullptr, acc, 0, m, n, k, kEpiAccI32, nullptr, nullptr, nullptr,
                   (cudaStream_t)stream, what);
}

h3q_status h3q_dequant_i8(const int8_t* q, const float* scale, int64_t scale_numel, void* out, int out_kind,
                          int64_t rows, int64_t cols, void* stream) {
  const char* what = "h3q_dequant_i8";
  if (h3q_status s = check_kind(out_kind, what)) return s;
  if (rows < 0 || cols < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (rows * cols == 0) return H3Q_OK;
  if (!q || !scale || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (scale_numel < 1) return fail(H3Q_ERR_ARG, "%s: empty scale", what);
  if (cols % 16 == 0 && (!aligned16(q) || !aligned16(out)))
    return fail(H3Q_ERR_ARG, "%s: q and out must be 16-byte aligned", what);
  const int per_row = (scale_numel == rows && rows > 1) ? 1 : 0;
  return cuda_status(launch_dequant_i8(q, scale, per_row, out, out_kind, rows, cols, (cudaStream_t)stream), what);
}

h3q_status h3q_dequant_nvfp4(const uint8_t* q, const uint8_t* block_scale, const float* global_scale, void* out,
                             int out_kind, int64_t rows, int64_t k, void* stream) {
  const char* what = "h3q_dequant_nvfp4";
  if (h3q_status s = check_kind(out_kind, what)) return s;
  if (rows < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (rows * k == 0) return H3Q_OK;
  if (!q || !block_scale || !global_scale || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (k % 16 != 0) return fail(H3Q_ERR_UNSUPPORTED, "%s: this build needs k %% 16 == 0 (k = %lld)", what, (long long)k);
  if ((reinterpret_cast<uintptr_t>(q) & 7u) || !aligned16(out))
    return fail(H3Q_ERR_ARG, "%s: q must be 8-byte and out 16-byte aligned", what);
  return cuda_status(launch_dequant_nvfp4(q, block_scale, global_scale, out, out_kind, rows, k, (cudaStream_t)stream),
                     what);
}

h3q_status h3q_gate_add(const void* x, const void* y, int kind, const float* gate, const uint32_t* idx, void* out,
                        int64_t s, int64_t c, void* stream) {
  const char* what = "h3q_gate_add";
  if (h3q_status st = check_kind(kind, what)) return st;
  if (s < 0 || c < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (s * c == 0) return H3Q_OK;
  if (!x || !y || !gate || !idx || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  return cuda_status(launch_gate_add(x, y, kind, gate, idx, out, s, c, (cudaStream_t)stream), what);
}

h3q_status h3q_rotate_activation(const uint16_t* x, uint16_t* y, int64_t m, int64_t k, void* stream) {
  const char* what = "h3q_rotate_activation";
  if (m < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (k % 256 != 0) return fail(H3Q_ERR_ARG, "ConvRot group 256 does not divide [%lld, %lld]", (long long)m, (long long)k);
  if (k / 256 > 64) return fail(H3Q_ERR_UNSUPPORTED, "%s: this build rotates rows of up to 16384 columns", what);
  if (m == 0 || k == 0) return H3Q_OK;
  if (!x || !y) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (!aligned16(x) || !aligned16(y)) return fail(H3Q_ERR_ARG, "%s: x and y must be 16-byte aligned", what);
  return cuda_status(launch_rotate_bf16(x, y, m, k, error_word(), (cudaStream_t)stream), what);
}

h3q_status h3q_swiglu(const void* y, void* out, int kind, int64_t rows, int64_t f, int interleaved, void* stream) {
  const char* what = "h3q_swiglu";
  if (h3q_status st = check_kind(kind, what)) return st;
  if (rows < 0 || f < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (rows * f == 0) return H3Q_OK;
  if (!y || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  return cuda_status(launch_swiglu(y, out, kind, rows, f, interleaved ? 1 : 0, (cudaStream_t)stream), what);
}

static h3q_status rms_modulate_checks(const uint16_t* x, const uint16_t* w, const float* scale, const float* shift,
                                      const uint32_t* idx, const void* out, int64_t S, int64_t C, const char* what) {
  if (S < 0 || C < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (S == 0 || C == 0) return H3Q_OK;
  if (!x || !w || !scale || !shift || !idx || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (C % 256 != 0 || C > 16384)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: this build needs C %% 256 == 0 and C <= 16384 (C = %lld)", what,
                (long long)C);
  if (!aligned16(x) || !aligned16(w) || !aligned16(scale) || !aligned16(shift) || !aligned16(out))
    return fail(H3Q_ERR_ARG, "%s: tensors must be 16-byte aligned", what);
  return H3Q_OK;
}

h3q_status h3q_rms_modulate(const uint16_t* x, const uint16_t* w, float eps, const float* scale, const float* shift,
                            const uint32_t* idx, uint16_t* out, int64_t S, int64_t C, void* stream) {
  const char* what = "h3q_rms_modulate";
  if (h3q_status st = rms_modulate_checks(x, w, scale, shift, idx, out, S, C, what)) return st;
  if (S == 0 || C == 0) return H3Q_OK;
  int* err = error_word();
  if (!err) return fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);
  return cuda_status(launch_rms_modulate(x, w, eps, scale, shift, idx, nullptr, nullptr, out, S, C, err,
                                         (cudaStream_t)stream),
                     what);
}

h3q_status h3q_rms_modulate_quant(const uint16_t* x, const uint16_t* w, float eps, const float* scale,
                                  const float* shift, const uint32_t* idx, int8_t* codes, float* row_scale, int64_t S,
                                  int64_t C, void* stream) {
  const char* what = "h3q_rms_modulate_quant";
  if (h3q_status st = rms_modulate_checks(x, w, scale, shift, idx, codes, S, C, what)) return st;
  if (S == 0 || C == 0) return H3Q_OK;
  if (!row_scale) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  int* err = error_word();
  if (!err) return fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);
  return cuda_status(launch_rms_modulate(x, w, eps, scale, shift, idx, codes, row_scale, nullptr, S, C, err,
                                         (cudaStream_t)stream),
                     what);
}

}  // extern "C"
