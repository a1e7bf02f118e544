// qlinear.cu -- host-side mirror of h3-rs's QLinear int8 dispatch (weights.rs:833-947) over the C ABI.
//
// The reference decides per call between the fused gemm_s8 (try_gemm_s8, weights.rs:889-909) and the
// cuBLASLt-style int8_linear_ex (apply_int8, weights.rs:911-947; run_swiglu, weights.rs:860-886), and between a
// rotation fused into the quantizer and a separate bf16 rotate_activation (weights.rs:482-489).  This file makes
// the same decisions from the same inputs (layer format, ConvRot group, interleaving, LoRA count, activation
// dtype and width, out_features, the four H3_* switches) and runs the chosen kernels.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>
#include "../../include/h3q.h"
#include "h3q_internal.h"

namespace h3q {
void set_last_error(const char* msg);
}

using h3q::launch_rotate_bf16;
using h3q::launch_swiglu;

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

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// try_gemm_s8's gate (weights.rs:892-895): the fused GEMM applies to bf16 activations with K % 64 == 0 and
// out_features % 128 == 0 on sm_80+ (every B200).
bool gemm_s8_applies(const h3q_qlinear* l, int x_kind, int64_t k, const h3q_switches* sw) {
  return sw->gemm_fused && x_kind == H3Q_KIND_BF16 && k % 64 == 0 && l->out_features % 128 == 0;
}

// The path for `swiglu` == 0 (QLinear::run) and 1 (QLinear::run_swiglu), or a negative status.
int plan(const h3q_qlinear* l, int x_kind, int64_t k, int swiglu, const h3q_switches* sw) {
  if (!l || !sw) return -H3Q_ERR_ARG;
  if (x_kind < 0 || x_kind > 2) return -H3Q_ERR_ARG;
  if (l->format != H3Q_FMT_INT8 || !sw->int8) return -H3Q_ERR_UNSUPPORTED;  // Prepared::Deq (weights.rs:838-841)
  if (l->n_loras > 0) return -H3Q_ERR_UNSUPPORTED;                         // LoRA deltas (weights.rs:937-940)
  if (k != l->in_features) return -H3Q_ERR_ARG;
  const int g = l->convrot;
  // run_swiglu on a non-interleaved layer goes straight to int8_linear_ex with the split-half SwiGLU
  // (weights.rs:868-883); everything else first tries the fused GEMM (weights.rs:850-853, :860-866).
  const bool direct_linear = swiglu && !l->interleaved;
  if (!direct_linear && gemm_s8_applies(l, x_kind, k, sw)) {
    const bool fused_rot = g == 256 && k / 256 <= 56 && sw->rot_fused;  // weights.rs:899
    int p = H3Q_PATH_GEMM_S8;
    if (g) p |= fused_rot ? H3Q_PATH_ROTATE_FUSED : H3Q_PATH_ROTATE_SEPARATE;
    if (swiglu) p |= H3Q_PATH_SWIGLU_FUSED;
    return p;
  }
  // int8_linear_ex: the rotation fuses only under H3_FUSED_ROT (can_fuse_rotation, kernels.rs:1081-1085)
  const bool fuse = g && sw->fused_rot_linear && g == 256 && k % 256 == 0 && k / 256 <= 64;
  int p = H3Q_PATH_INT8_LINEAR;
  if (g) p |= fuse ? H3Q_PATH_ROTATE_FUSED : H3Q_PATH_ROTATE_SEPARATE;
  if (swiglu) p |= direct_linear ? H3Q_PATH_SWIGLU_FUSED : H3Q_PATH_SWIGLU_AFTER;
  return p;
}

}  // namespace

extern "C" {

h3q_switches h3q_default_switches(void) {
  h3q_switches s;
  s.int8 = 1;
  s.gemm_fused = 1;
  s.rot_fused = 1;
  s.fused_rot_linear = 0;
  return s;
}

int h3q_qlinear_plan(const h3q_qlinear* layer, int x_kind, int64_t in_width, int swiglu, const h3q_switches* sw) {
  return plan(layer, x_kind, in_width, swiglu, sw);
}

size_t h3q_qlinear_workspace_size(const h3q_qlinear* layer, int x_kind, int64_t rows, int swiglu,
                                  const h3q_switches* sw) {
  const int p = plan(layer, x_kind, layer ? layer->in_features : 0, swiglu, sw);
  if (p < 0) return 0;
  const int64_t k = layer->in_features, n = layer->out_features;
  const size_t es = x_kind == H3Q_KIND_F32 ? 4 : 2;
  size_t bytes = h3q_gemm_s8_workspace_size(rows, k);
  if (p & H3Q_PATH_ROTATE_SEPARATE) bytes += align256((size_t)rows * k * es);
  if (p & H3Q_PATH_SWIGLU_AFTER) bytes += align256((size_t)rows * n * es);
  return bytes;
}

h3q_status h3q_qlinear_forward(const h3q_qlinear* l, const void* x, int x_kind, int64_t rows, int swiglu, void* out,
                               void* workspace, size_t workspace_bytes, const h3q_switches* sw, void* stream) {
  const char* what = "h3q_qlinear_forward";
  if (!l || !sw) return fail(H3Q_ERR_ARG, "%s: null layer or switches", what);
  const int p = plan(l, x_kind, l->in_features, swiglu, sw);
  if (p < 0) {
    if (p == -H3Q_ERR_UNSUPPORTED)
      return fail(H3Q_ERR_UNSUPPORTED, "%s: layer served by the dequantise-then-matmul path (format %d, int8 %d, "
                  "%d LoRA deltas)", what, l->format, sw->int8, l->n_loras);
    return fail(H3Q_ERR_ARG, "%s: invalid layer or activation kind", what);
  }
  if (rows < 0) return fail(H3Q_ERR_ARG, "%s: negative rows", what);
  if (rows == 0) return H3Q_OK;
  const size_t need = h3q_qlinear_workspace_size(l, x_kind, rows, swiglu, sw);
  if (!workspace || workspace_bytes < need)
    return fail(H3Q_ERR_WORKSPACE, "%s: workspace of %zu bytes, need %zu", what, workspace_bytes, need);
  const int64_t k = l->in_features, n = l->out_features;
  const size_t es = x_kind == H3Q_KIND_F32 ? 4 : 2;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* wsp = static_cast<uint8_t*>(workspace);
  const void* xr = x;
  if (p & H3Q_PATH_ROTATE_SEPARATE) {
    // rotate_activation(x, g) in the activation dtype (weights.rs:482-489)
    if (l->convrot != 256) return fail(H3Q_ERR_UNSUPPORTED, "%s: ConvRot group %d", what, l->convrot);
    if (x_kind != H3Q_KIND_BF16)
      return fail(H3Q_ERR_UNSUPPORTED, "%s: a separate rotation needs bf16 activations", what);
    if (k % 256 != 0) return fail(H3Q_ERR_ARG, "ConvRot group 256 does not divide %lld", (long long)k);
    if (k / 256 > 64) return fail(H3Q_ERR_UNSUPPORTED, "%s: rotation handles k <= 16384", what);
    uint16_t* xrot = reinterpret_cast<uint16_t*>(wsp);
    cudaError_t e = launch_rotate_bf16(static_cast<const uint16_t*>(x), xrot, rows, k, nullptr, st);
    if (e != cudaSuccess) return fail(H3Q_ERR_CUDA, "%s: rotation: %s", what, cudaGetErrorString(e));
    xr = xrot;
    wsp += align256((size_t)rows * k * es);
  }
  void* lin_out = out;
  if (p & H3Q_PATH_SWIGLU_AFTER) {
    lin_out = wsp;
    wsp += align256((size_t)rows * n * es);
  }
  const size_t qws = h3q_gemm_s8_workspace_size(rows, k);
  const int rot_fused = (p & H3Q_PATH_ROTATE_FUSED) ? 1 : 0;
  const int swiglu_fused = (p & H3Q_PATH_SWIGLU_FUSED) ? 1 : 0;
  h3q_status s;
  if (p & H3Q_PATH_GEMM_S8) {
    s = h3q_gemm_s8(static_cast<const uint16_t*>(xr), l->weight, l->scale, l->scale_numel, l->bias,
                    static_cast<uint16_t*>(lin_out), rows, n, k, swiglu_fused, rot_fused, wsp, qws, stream);
  } else {
    s = h3q_int8_linear_ex(xr, x_kind, l->weight, l->scale, l->scale_numel, l->bias, lin_out, x_kind, rows, n, k,
                           swiglu_fused, rot_fused, wsp, qws, stream);
  }
  if (s != H3Q_OK) return s;
  if (p & H3Q_PATH_SWIGLU_AFTER) {
    // swiglu_interleaved (weights.rs:806-816) or ops::swiglu (ops.rs:39-44) over the linear output
    cudaError_t e = launch_swiglu(lin_out, out, x_kind, rows, n / 2, l->interleaved, st);
    if (e != cudaSuccess) return fail(H3Q_ERR_CUDA, "%s: swiglu: %s", what, cudaGetErrorString(e));
  }
  return H3Q_OK;
}

}  // extern "C"
