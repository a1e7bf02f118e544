// attn_capi.cu -- C ABI of the int8 attention (include/h3q.h): argument checks, workspace carving and the
// stage sequence of attention_f16v (attn8.rs:617-627): K mean, Q and K quantisation, V relayout, attention.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>
#include "../../include/h3q.h"
#include "h3q_internal.h"

namespace h3q {
void set_last_error(const char* msg);
size_t kmean_workspace_bytes(int64_t S, int64_t H);
cudaError_t launch_kmean(const uint16_t* k, int64_t S, int64_t H, float* mean, float* part, cudaStream_t st);
cudaError_t launch_quant_heads(const uint16_t* x, const float* mean, int8_t* codes, float* scales, int64_t S,
                               int64_t H, bool block128, cudaStream_t st);
cudaError_t launch_v_layout(const uint16_t* x, int64_t rs, int64_t col, uint16_t* vt, int64_t S, int64_t H,
                            bool keep_bf16, cudaStream_t st);
cudaError_t launch_attention(const int8_t* q8, const float* qs, int64_t Sq, const int8_t* k8, const float* ks,
                             const uint16_t* vt, uint16_t* out, int64_t S, int64_t H, bool bf16pv,
                             int32_t* scores, int* err, cudaStream_t st);
cudaError_t launch_qk_norm_rope(const uint16_t* x, int64_t rs, int64_t col, int64_t hs, const uint16_t* w,
                                int do_norm, float eps, const float* cs, int rot, uint16_t* out, int64_t S, int64_t H,
                                int64_t D, cudaStream_t st);
cudaError_t launch_kmean_rope(const uint16_t* x, int64_t rs, int64_t col, const uint16_t* w, int do_norm, float eps,
                              const float* cs, int rot, int64_t S, int64_t H, float* mean, float* part,
                              cudaStream_t st);
cudaError_t launch_qk_rope_quant(const uint16_t* x, int64_t rs, int64_t col, const uint16_t* w, int do_norm,
                                 float eps, const float* cs, int rot, const float* mean, int8_t* codes, float* scales,
                                 int64_t S, int64_t H, bool block128, cudaStream_t st);
}  // namespace h3q

namespace {

constexpr int64_t HD = 128;

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
size_t a256(size_t v) { return (v + 255) / 256 * 256; }
int64_t padded(int64_t S) { return (S + 127) / 128 * 128; }

// Shapes the kernels index with 32-bit integers: tokens, heads, grid and TMA coordinates.
h3q_status check_shape(int64_t S, int64_t H, const char* what) {
  if (S < 0 || H < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (H == 0 && S > 0) return fail(H3Q_ERR_ARG, "%s: no heads", what);
  if (S > (int64_t)1 << 24 || H > 4096)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: this build handles S <= 2^24 tokens and H <= 4096 heads", what);
  return H3Q_OK;
}

h3q_status check_flags(int flags, const char* what) {
  if (flags & ~(H3Q_ATTN_SCALE_BLOCK128 | H3Q_ATTN_PV_BF16)) return fail(H3Q_ERR_ARG, "%s: unknown flags %d", what, flags);
  return H3Q_OK;
}

// Workspace carve-up (each piece 256-byte aligned): kmean [H*128] f32, kmean chunk sums, q codes, q scales,
// k codes, k scales, V^T.
struct AttnWs {
  float* kmean;
  float* part;
  int8_t* q8;
  float* qs;
  int8_t* k8;
  float* ks;
  uint16_t* vt;
  size_t bytes;
};

AttnWs carve(uint8_t* base, int64_t Sq, int64_t S, int64_t H) {
  AttnWs w{};
  const int64_t Sp = padded(S), Sqp = padded(Sq);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* p = base ? base + off : nullptr;
    off += a256(n);
    return p;
  };
  w.kmean = reinterpret_cast<float*>(take((size_t)H * HD * 4));
  w.part = reinterpret_cast<float*>(take(h3q::kmean_workspace_bytes(S, H)));
  w.q8 = reinterpret_cast<int8_t*>(take((size_t)Sq * H * HD));
  w.qs = reinterpret_cast<float*>(take((size_t)H * Sqp * 4));
  w.k8 = reinterpret_cast<int8_t*>(take((size_t)S * H * HD));
  w.ks = reinterpret_cast<float*>(take((size_t)H * Sp * 4));
  w.vt = reinterpret_cast<uint16_t*>(take((size_t)H * HD * Sp * 2));
  w.bytes = off;
  return w;
}

// attention_f16v (attn8.rs:617-627) for Sq query rows against S keys, V given as rows of [S, rs] at column `col`.
h3q_status run_attention(const uint16_t* q, int64_t Sq, const uint16_t* k, const uint16_t* vsrc, int64_t rs,
                         int64_t col, uint16_t* out, int64_t S, int64_t H, int flags, void* workspace,
                         size_t workspace_bytes, void* stream, const char* what) {
  if (h3q_status s = check_shape(S, H, what)) return s;
  if (h3q_status s = check_shape(Sq, H, what)) return s;
  if (h3q_status s = check_flags(flags, what)) return s;
  if (S == 0 || Sq == 0) return H3Q_OK;
  if (!q || !k || !vsrc || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (!aligned16(q) || !aligned16(k) || !aligned16(out))
    return fail(H3Q_ERR_ARG, "%s: q, k and out must be 16-byte aligned", what);
  const AttnWs need = carve(nullptr, Sq, S, H);
  if (!workspace || workspace_bytes < need.bytes)
    return fail(H3Q_ERR_WORKSPACE, "%s: workspace of %zu bytes, need %zu", what, workspace_bytes, need.bytes);
  if (!aligned16(workspace)) return fail(H3Q_ERR_ARG, "%s: workspace must be 16-byte aligned", what);
  const AttnWs w = carve(static_cast<uint8_t*>(workspace), Sq, S, H);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = h3q::error_word_current();
  if (!err) return fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);
  const bool block = (flags & H3Q_ATTN_SCALE_BLOCK128) != 0;
  const bool bf16pv = (flags & H3Q_ATTN_PV_BF16) != 0;
  // smoothing K by its mean over tokens shifts every score of a query by the same amount (attn8.rs:620-621)
  if (h3q_status s = cuda_status(h3q::launch_kmean(k, S, H, w.kmean, w.part, st), what)) return s;
  if (h3q_status s = cuda_status(h3q::launch_quant_heads(q, nullptr, w.q8, w.qs, Sq, H, block, st), what)) return s;
  if (h3q_status s = cuda_status(h3q::launch_quant_heads(k, w.kmean, w.k8, w.ks, S, H, block, st), what)) return s;
  if (h3q_status s = cuda_status(h3q::launch_v_layout(vsrc, rs, col, w.vt, S, H, bf16pv, st), what)) return s;
  return cuda_status(h3q::launch_attention(w.q8, w.qs, Sq, w.k8, w.ks, w.vt, out, S, H, bf16pv, nullptr, err, st),
                     what);
}

}  // namespace

extern "C" {

int h3q_attention_available(int64_t head_dim, int x_kind, int device) {
  return head_dim == HD && x_kind == H3Q_KIND_BF16 && h3q_available_arch(device) ? 1 : 0;
}

size_t h3q_attention_workspace_size(int64_t S, int64_t H, int flags) {
  (void)flags;
  if (S <= 0 || H <= 0) return 0;
  return carve(nullptr, S, S, H).bytes;
}

size_t h3q_attention_rows_workspace_size(int64_t Sq, int64_t S, int64_t H, int flags) {
  (void)flags;
  if (S <= 0 || Sq <= 0 || H <= 0) return 0;
  return carve(nullptr, Sq, S, H).bytes;
}

h3q_status h3q_attention_rows(const uint16_t* q, int64_t Sq, const uint16_t* k, const uint16_t* v_src,
                              int64_t v_row_stride, int64_t v_col, uint16_t* out, int64_t S, int64_t H, int flags,
                              void* workspace, size_t workspace_bytes, void* stream) {
  const char* what = "h3q_attention_rows";
  if (v_col < 0 || v_row_stride < v_col + H * HD)
    return fail(H3Q_ERR_ARG, "%s: V columns [%lld, %lld) outside a row of %lld elements", what, (long long)v_col,
                (long long)(v_col + H * HD), (long long)v_row_stride);
  return run_attention(q, Sq, k, v_src, v_row_stride, v_col, out, S, H, flags, workspace, workspace_bytes, stream,
                       what);
}

h3q_status h3q_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int64_t S,
                         int64_t H, int flags, void* workspace, size_t workspace_bytes, void* stream) {
  return run_attention(q, S, k, v, H * HD, 0, out, S, H, flags, workspace, workspace_bytes, stream, "h3q_attention");
}

h3q_status h3q_attention_qkv(const uint16_t* q, const uint16_t* k, const uint16_t* qkv, int64_t qkv_width,
                             int64_t v_col, uint16_t* out, int64_t S, int64_t H, int flags, void* workspace,
                             size_t workspace_bytes, void* stream) {
  const char* what = "h3q_attention_qkv";
  if (v_col < 0 || qkv_width < v_col + H * HD)
    return fail(H3Q_ERR_ARG, "%s: V columns [%lld, %lld) outside a qkv row of width %lld", what, (long long)v_col,
                (long long)(v_col + H * HD), (long long)qkv_width);
  return run_attention(q, S, k, qkv, qkv_width, v_col, out, S, H, flags, workspace, workspace_bytes, stream, what);
}

size_t h3q_attn_kmean_workspace_size(int64_t S, int64_t H) { return h3q::kmean_workspace_bytes(S, H); }

h3q_status h3q_attn_kmean(const uint16_t* k, int64_t S, int64_t H, float* kmean, void* workspace,
                          size_t workspace_bytes, void* stream) {
  const char* what = "h3q_attn_kmean";
  if (h3q_status s = check_shape(S, H, what)) return s;
  if (S == 0) return H3Q_OK;
  if (!k || !kmean) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (!aligned16(k) || !aligned16(kmean)) return fail(H3Q_ERR_ARG, "%s: k and kmean must be 16-byte aligned", what);
  const size_t need = h3q::kmean_workspace_bytes(S, H);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(H3Q_ERR_WORKSPACE, "%s: workspace of %zu bytes, need %zu (16-byte aligned)", what, workspace_bytes,
                need);
  return cuda_status(h3q::launch_kmean(k, S, H, kmean, static_cast<float*>(workspace), (cudaStream_t)stream), what);
}

h3q_status h3q_attn_quant_heads(const uint16_t* x, const float* mean, int8_t* codes, float* scales, int64_t S,
                                int64_t H, int flags, void* stream) {
  const char* what = "h3q_attn_quant_heads";
  if (h3q_status s = check_shape(S, H, what)) return s;
  if (h3q_status s = check_flags(flags, what)) return s;
  if (S == 0) return H3Q_OK;
  if (!x || !codes || !scales) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (!aligned16(x) || !aligned16(codes) || (mean && !aligned16(mean)) || !aligned16(scales))
    return fail(H3Q_ERR_ARG, "%s: tensors must be 16-byte aligned", what);
  return cuda_status(h3q::launch_quant_heads(x, mean, codes, scales, S, H, (flags & H3Q_ATTN_SCALE_BLOCK128) != 0,
                                             (cudaStream_t)stream),
                     what);
}

h3q_status h3q_attn_v_layout(const uint16_t* src, int64_t row_stride, int64_t col_off, uint16_t* vt, int64_t S,
                             int64_t H, int flags, void* stream) {
  const char* what = "h3q_attn_v_layout";
  if (h3q_status s = check_shape(S, H, what)) return s;
  if (h3q_status s = check_flags(flags, what)) return s;
  if (S == 0) return H3Q_OK;
  if (!src || !vt) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (col_off < 0 || row_stride < col_off + H * HD)
    return fail(H3Q_ERR_ARG, "%s: V columns [%lld, %lld) outside a row of %lld elements", what, (long long)col_off,
                (long long)(col_off + H * HD), (long long)row_stride);
  if (!aligned16(vt)) return fail(H3Q_ERR_ARG, "%s: vt must be 16-byte aligned", what);
  if ((reinterpret_cast<uintptr_t>(src) & 1u)) return fail(H3Q_ERR_ARG, "%s: src must be 2-byte aligned", what);
  return cuda_status(h3q::launch_v_layout(src, row_stride, col_off, vt, S, H, (flags & H3Q_ATTN_PV_BF16) != 0,
                                          (cudaStream_t)stream),
                     what);
}

h3q_status h3q_attention_core(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks,
                              const uint16_t* vt, uint16_t* out, int64_t S, int64_t H, int flags, int32_t* scores,
                              void* stream) {
  const char* what = "h3q_attention_core";
  if (h3q_status s = check_shape(S, H, what)) return s;
  if (h3q_status s = check_flags(flags, what)) return s;
  if (S == 0) return H3Q_OK;
  if (!q8 || !qs || !k8 || !ks || !vt || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (!aligned16(q8) || !aligned16(k8) || !aligned16(qs) || !aligned16(ks) || !aligned16(vt) || !aligned16(out))
    return fail(H3Q_ERR_ARG, "%s: tensors must be 16-byte aligned", what);
  if (scores && S > 8192) return fail(H3Q_ERR_ARG, "%s: the score dump is for S <= 8192", what);
  int* err = h3q::error_word_current();
  if (!err) return fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);
  return cuda_status(h3q::launch_attention(q8, qs, S, k8, ks, vt, out, S, H, (flags & H3Q_ATTN_PV_BF16) != 0, scores,
                                           err, (cudaStream_t)stream),
                     what);
}

h3q_status h3q_qk_norm_rope(const uint16_t* x, int64_t row_stride, int64_t col_off, int64_t head_stride,
                            const uint16_t* w, int do_norm, float eps, const float* rope, int rot, uint16_t* out,
                            int64_t S, int64_t H, int64_t D, void* stream) {
  const char* what = "h3q_qk_norm_rope";
  if (h3q_status s = check_shape(S, H, what)) return s;
  if (D < 1 || D > 256) return fail(H3Q_ERR_UNSUPPORTED, "%s: head_dim %lld (1..256)", what, (long long)D);
  if (S == 0) return H3Q_OK;
  if (!x || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (col_off < 0 || head_stride < 0 || row_stride < col_off + (H - 1) * head_stride + D)
    return fail(H3Q_ERR_ARG, "%s: heads at column %lld (stride %lld) outside a row of %lld elements", what,
                (long long)col_off, (long long)head_stride, (long long)row_stride);
  if (!rope) rot = 0;  // no table: no rotation (the reference's launch passes rot = 0)
  if (rot < 0 || rot % 2 != 0 || rot > D)
    return fail(H3Q_ERR_ARG, "%s: rot %d must be even and within head_dim %lld", what, rot, (long long)D);
  return cuda_status(h3q::launch_qk_norm_rope(x, row_stride, col_off, head_stride, do_norm ? w : nullptr,
                                              do_norm ? 1 : 0, eps, rope, rot, out, S, H, D, (cudaStream_t)stream),
                     what);
}

h3q_status h3q_attend_qkv(const uint16_t* qkv, int64_t qkv_width, int64_t q_col, int64_t k_col, int64_t v_col,
                          const uint16_t* q_norm, const uint16_t* k_norm, int do_norm, float eps, const float* rope,
                          int rot, uint16_t* out, int64_t S, int64_t H, int flags, void* workspace,
                          size_t workspace_bytes, void* stream) {
  const char* what = "h3q_attend_qkv";
  if (h3q_status s = check_shape(S, H, what)) return s;
  if (h3q_status s = check_flags(flags, what)) return s;
  if (S == 0) return H3Q_OK;
  if (!qkv || !out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  const int64_t cols[3] = {q_col, k_col, v_col};
  for (int i = 0; i < 3; ++i)
    if (cols[i] < 0 || qkv_width < cols[i] + H * HD)
      return fail(H3Q_ERR_ARG, "%s: columns [%lld, %lld) outside a qkv row of width %lld", what, (long long)cols[i],
                  (long long)(cols[i] + H * HD), (long long)qkv_width);
  if (!aligned16(qkv) || qkv_width % 8 || q_col % 8 || k_col % 8)
    return fail(H3Q_ERR_ARG, "%s: qkv must be 16-byte aligned with width and q / k columns multiples of 8", what);
  if (do_norm && ((q_norm && !aligned16(q_norm)) || (k_norm && !aligned16(k_norm))))
    return fail(H3Q_ERR_ARG, "%s: norm weights must be 16-byte aligned", what);
  if (!rope) rot = 0;
  if (rot < 0 || rot % 8 != 0 || rot > HD)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: this build rotates rot %% 8 == 0 dims, rot <= 128 (rot = %d); use "
                "h3q_qk_norm_rope + h3q_attention_qkv", what, rot);
  if (rot && !aligned16(rope)) return fail(H3Q_ERR_ARG, "%s: the rope table must be 16-byte aligned", what);
  if (!aligned16(out)) return fail(H3Q_ERR_ARG, "%s: out must be 16-byte aligned", what);
  const AttnWs need = carve(nullptr, S, S, H);
  if (!workspace || workspace_bytes < need.bytes)
    return fail(H3Q_ERR_WORKSPACE, "%s: workspace of %zu bytes, need %zu", what, workspace_bytes, need.bytes);
  if (!aligned16(workspace)) return fail(H3Q_ERR_ARG, "%s: workspace must be 16-byte aligned", what);
  const AttnWs w = carve(static_cast<uint8_t*>(workspace), S, S, H);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = h3q::error_word_current();
  if (!err) return fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);
  const bool block = (flags & H3Q_ATTN_SCALE_BLOCK128) != 0;
  const bool bf16pv = (flags & H3Q_ATTN_PV_BF16) != 0;
  const int dn = do_norm ? 1 : 0;
  const uint16_t* qw = dn ? q_norm : nullptr;
  const uint16_t* kw = dn ? k_norm : nullptr;
  // qk_norm_rope of q and k (dit.rs:748-749) fused into the K mean and the Q / K quantisation of attention_qkv
  if (h3q_status s = cuda_status(h3q::launch_kmean_rope(qkv, qkv_width, k_col, kw, dn, eps, rope, rot, S, H, w.kmean,
                                                        w.part, st), what))
    return s;
  if (h3q_status s = cuda_status(h3q::launch_qk_rope_quant(qkv, qkv_width, q_col, qw, dn, eps, rope, rot, nullptr,
                                                           w.q8, w.qs, S, H, block, st), what))
    return s;
  if (h3q_status s = cuda_status(h3q::launch_qk_rope_quant(qkv, qkv_width, k_col, kw, dn, eps, rope, rot, w.kmean,
                                                           w.k8, w.ks, S, H, block, st), what))
    return s;
  if (h3q_status s = cuda_status(h3q::launch_v_layout(qkv, qkv_width, v_col, w.vt, S, H, bf16pv, st), what)) return s;
  return cuda_status(h3q::launch_attention(w.q8, w.qs, S, w.k8, w.ks, w.vt, out, S, H, bf16pv, nullptr, err, st),
                     what);
}

}  // extern "C"
