// Host launchers for the reference's attn8.rs CUDA C (test infrastructure: GPU comparator only).
// The kernel text is extracted at build time into oracle/_ref/attn8_src.cu (see extract_cuda_src.py).
#include <cuda_runtime.h>
#include "../_ref/attn8_src.cu"

extern "C" {

// Gemm::cuda_fwd launch (attn8.rs:543-563): 1-D grid of ceil(N/128)*ceil(M/128), 256 threads, 48 KiB smem
int h3ref_gemm_s8(const signed char* A, const signed char* B, const float* xs, const float* ws, int ws_per_row,
                  const float* bias, int has_bias, unsigned short* out, int M, int N, int K, int swiglu, void* stream) {
  const unsigned smem = 3 * (128 + 128) * 64;
  cudaFuncSetAttribute(gemm_s8, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const unsigned grid = (unsigned)(((N + 127) / 128) * ((M + 127) / 128));
  if (grid == 0) return 0;
  gemm_s8<<<grid, 256, smem, (cudaStream_t)stream>>>(A, B, xs, ws, ws_per_row, bias, has_bias, out, M, N, K, swiglu);
  return (int)cudaGetLastError();
}

// ColMean (attn8.rs:440-453): acc must be zeroed; grid (ceil(C/256), ceil(S/rows_per)), rows_per = ceil(S/min(128,S))
int h3ref_col_sum(const unsigned short* x, float* acc, int S, int C, void* stream) {
  const int parts = S < 128 ? S : 128;
  if (parts == 0) return 0;
  const int rows_per = (S + parts - 1) / parts;
  dim3 grid((C + 255) / 256, (S + rows_per - 1) / rows_per);
  col_sum<<<grid, 256, 0, (cudaStream_t)stream>>>(x, acc, S, C, rows_per);
  return (int)cudaGetLastError();
}

// QuantHeads (attn8.rs:406-425): out = int8 [H,S,128] then f32 scales [H,S]; grid ceil(S*H/8), 256 threads
int h3ref_quant_heads(const unsigned short* x, const float* mean, signed char* out, float* scale, int S, int H,
                      void* stream) {
  const unsigned rows = (unsigned)(S * H);
  if (rows == 0) return 0;
  quant_heads<<<(rows + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, mean, out, scale, S, H);
  return (int)cudaGetLastError();
}

// VToF16 (attn8.rs:474-485)
int h3ref_v_to_f16(const unsigned short* x, unsigned long long row_stride, unsigned long long col_off,
                   unsigned short* out, int S, int H, void* stream) {
  unsigned n = (unsigned)(S * H * 64);
  unsigned g = (n + 255) / 256;
  if (g > 65535u * 4) g = 65535u * 4;
  if (g == 0) return 0;
  v_to_f16<<<g, 256, 0, (cudaStream_t)stream>>>(x, row_stride, col_off, out, S, H);
  return (int)cudaGetLastError();
}

// Attn (attn8.rs:500-519): grid (ceil(S/64), H), 128 threads, 49,664 bytes of dynamic smem
int h3ref_attn_qk8(const signed char* q8, const float* qs, const signed char* k8, const float* ks,
                   const unsigned short* v, unsigned short* out, int S, int H, float scale_log2, void* stream) {
  const unsigned smem = 2 * 64 * 128 + 2 * 64 * 128 * 2 + 2 * 64 * 4;
  cudaFuncSetAttribute(attn_qk8, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((S + 63) / 64, H);
  if (S == 0 || H == 0) return 0;
  attn_qk8<<<grid, 128, smem, (cudaStream_t)stream>>>(q8, qs, k8, ks, v, out, S, H, scale_log2);
  return (int)cudaGetLastError();
}

}  // extern "C"
