// Host launchers for the reference's kernels.rs CUDA C (test infrastructure: GPU comparator only).
// The kernel text is extracted at build time into oracle/_ref/kernels_src.cu (see extract_cuda_src.py);
// launch shapes follow the reference's host code line by line.
#include <cuda_runtime.h>
#include "../_ref/kernels_src.cu"

extern "C" {

// quant_rows_raw selection and launch (kernels.rs:1133-1161): grid = rows, block = 256
int h3ref_quant_rows(const void* x, int kind, signed char* q, float* scale, int m, int k, int rotate, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  const bool rot2 = rotate && kind == 2 && k % 256 == 0 && k / 256 <= 56;
  if (m == 0) return 0;
  if (rot2) quant_rows_i8_rot2<<<m, 256, 0, s>>>((const u16*)x, q, scale, k);
  else if (rotate) quant_rows_i8_rot<<<m, 256, 0, s>>>(x, kind, q, scale, k);
  else quant_rows_i8<<<m, 256, 0, s>>>(x, kind, q, scale, k);
  return (int)cudaGetLastError();
}

// Int8Linear step 1 (kernels.rs:979-991): quant_rows_i8_rot when rotate && k % 256 == 0 && k / 256 <= 64
int h3ref_quant_rows_linear(const void* x, int kind, signed char* q, float* scale, int m, int k, int rotate,
                            void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  const bool rot = rotate && k % 256 == 0 && k / 256 <= 64;
  if (m == 0) return 0;
  if (rot) quant_rows_i8_rot<<<m, 256, 0, s>>>(x, kind, q, scale, k);
  else quant_rows_i8<<<m, 256, 0, s>>>(x, kind, q, scale, k);
  return (int)cudaGetLastError();
}

// int8_epilogue / int8_epilogue_swiglu launch (kernels.rs:1049-1066): grid (ceil(n_out/4/256), M)
int h3ref_int8_epilogue(const int* acc, const float* xs, const float* ws, int ws_per_row, const float* bias,
                        int has_bias, void* out, int okind, unsigned long long m, unsigned long long n_out, int swiglu,
                        void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid((unsigned)((n_out / 4 + 255) / 256), (unsigned)m);
  if (swiglu) int8_epilogue_swiglu<<<grid, 256, 0, s>>>(acc, xs, ws, ws_per_row, bias, has_bias, out, okind, m, n_out);
  else int8_epilogue<<<grid, 256, 0, s>>>(acc, xs, ws, ws_per_row, bias, has_bias, out, okind, m, n_out);
  return (int)cudaGetLastError();
}

static unsigned grid_for(unsigned long long n) {
  unsigned long long b = (n + 255) / 256;
  if (b < 1) b = 1;
  if (b > 65535ull * 8) b = 65535ull * 8;
  return (unsigned)b;
}

// dequant_i8 / dequant_nvfp4 / gate_add launches (kernels.rs:556-560 grid_for)
int h3ref_dequant_i8(const signed char* q, const float* scale, void* out, unsigned long long rows,
                     unsigned long long cols, int per_row, int okind, void* stream) {
  dequant_i8<<<grid_for(rows * cols), 256, 0, (cudaStream_t)stream>>>(q, scale, out, rows, cols, per_row, okind);
  return (int)cudaGetLastError();
}

int h3ref_dequant_nvfp4(const unsigned char* q, const unsigned char* bs, const float* g, void* out,
                        unsigned long long rows, unsigned long long k, int okind, void* stream) {
  dequant_nvfp4<<<grid_for(rows * k), 256, 0, (cudaStream_t)stream>>>(q, bs, g, out, rows, k, okind);
  return (int)cudaGetLastError();
}

int h3ref_gate_add(const void* x, const void* y, int kind, const float* gate, const unsigned* idx, void* out,
                   unsigned long long S, unsigned long long C, void* stream) {
  gate_add<<<grid_for(S * C), 256, 0, (cudaStream_t)stream>>>(x, y, kind, gate, idx, out, S, C);
  return (int)cudaGetLastError();
}

// RmsModulate::cuda_fwd launch (kernels.rs:1184-1196): one CTA of 512 threads per row
int h3ref_rms_modulate(const void* x, int kind, const void* w, float eps, const float* scale, const float* shift,
                       const unsigned* idx, void* out, int S, int C, void* stream) {
  if (S == 0) return 0;
  rms_modulate<<<S, 512, 0, (cudaStream_t)stream>>>(x, kind, w, eps, scale, shift, idx, out, C);
  return (int)cudaGetLastError();
}

// QkNormRope::cuda_fwd launch (kernels.rs:722-729): one CTA of roundup(D, 32) threads per (token, head) row
int h3ref_qk_norm_rope(const void* x, int xkind, unsigned long long row_stride, unsigned long long col_off,
                       unsigned long long head_stride, const void* w, int wkind, int has_w, int do_norm, float eps,
                       const float* cs, int rot, void* out, int okind, int S, int H, int D, void* stream) {
  if (S == 0 || H == 0) return 0;
  const unsigned threads = (unsigned)((D + 31) / 32 * 32);
  qk_norm_rope<<<(unsigned)(S * H), threads, 0, (cudaStream_t)stream>>>(x, xkind, row_stride, col_off, head_stride, w,
                                                                      wkind, has_w, do_norm, eps, cs, rot, out,
                                                                      okind, S, H, D);
  return (int)cudaGetLastError();
}

}  // extern "C"
