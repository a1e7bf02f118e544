/*
 * gemm_s8_capi.c -- TEST PROGRAM: the C ABI of include/h3q.h used from plain C (C11, no C++, no Python, no torch),
 * the way a non-Python caller (a Rust, Go or C host behind an FFI) drives the library.
 *
 * It generates a linear layer's inputs with the CPU oracle (liboracle.so, test infrastructure), moves them to the
 * device with the CUDA runtime API, calls h3q_gemm_s8 (attn8::gemm_s8 with the ConvRot rotation), and checks every
 * bf16 output bit for bit against the oracle's quantizer -> int32 GEMM -> epilogue.  It also checks that a bad
 * shape is refused with H3Q_ERR_ARG and an error text.  Exit code 0 and "ok" on success.
 *
 * usage: gemm_s8_capi M K N
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <cuda_runtime_api.h>

#include "h3q.h"

/* the oracle's C entry points used here (oracle/h3q_oracle.c) */
void h3o_make_linear_inputs(uint64_t seed, int64_t M, int64_t K, int64_t N, int n_outliers, uint16_t* x, int8_t* w,
                            float* ws, float* bias);
int h3o_quant_rows(const void* x, int kind, int8_t* q, float* scale, int64_t M, int64_t K, int mode);
void h3o_gemm_s8_acc(const int8_t* A, const int8_t* B, int32_t* acc, int64_t M, int64_t N, int64_t K);
void h3o_gemm_s8_epilogue(const int32_t* acc, const float* xs, const float* ws, int ws_per_row, const float* bias,
                          uint16_t* out, int64_t M, int64_t N, int epi, const float* gate, const uint32_t* gate_idx,
                          const uint16_t* resid);

#define CHECK_CUDA(call)                                                                  \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess) {                                                              \
      fprintf(stderr, "%s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e_));        \
      return 2;                                                                           \
    }                                                                                     \
  } while (0)

int main(int argc, char** argv) {
  if (argc != 4) {
    fprintf(stderr, "usage: %s M K N\n", argv[0]);
    return 2;
  }
  const int64_t M = atoll(argv[1]), K = atoll(argv[2]), N = atoll(argv[3]);
  if (!h3q_available_arch(0)) {
    fprintf(stderr, "device 0 is not an sm_100 GPU\n");
    return 2;
  }
  if (h3q_init(0) != H3Q_OK) {
    fprintf(stderr, "h3q_init: %s\n", h3q_last_error());
    return 2;
  }
  uint16_t* x = malloc((size_t)M * K * 2);
  int8_t* w = malloc((size_t)N * K);
  float* ws = malloc((size_t)N * 4);
  float* bias = malloc((size_t)N * 4);
  int8_t* q = malloc((size_t)M * K);
  float* xs = malloc((size_t)M * 4);
  int32_t* acc = malloc((size_t)M * N * 4);
  uint16_t* want = malloc((size_t)M * N * 2);
  uint16_t* got = malloc((size_t)M * N * 2);
  if (!x || !w || !ws || !bias || !q || !xs || !acc || !want || !got) return 2;
  h3o_make_linear_inputs(7, M, K, N, 8, x, w, ws, bias);
  if (h3o_quant_rows(x, H3Q_KIND_BF16, q, xs, M, K, 2) != 0) return 2;
  h3o_gemm_s8_acc(q, w, acc, M, N, K);
  h3o_gemm_s8_epilogue(acc, xs, ws, 1, bias, want, M, N, H3Q_EPI_LINEAR, NULL, NULL, NULL);

  void *dx, *dw, *dws, *dbias, *dout, *dwork;
  const size_t work = h3q_gemm_s8_workspace_size(M, K);
  CHECK_CUDA(cudaMalloc(&dx, (size_t)M * K * 2));
  CHECK_CUDA(cudaMalloc(&dw, (size_t)N * K));
  CHECK_CUDA(cudaMalloc(&dws, (size_t)N * 4));
  CHECK_CUDA(cudaMalloc(&dbias, (size_t)N * 4));
  CHECK_CUDA(cudaMalloc(&dout, (size_t)M * N * 2));
  CHECK_CUDA(cudaMalloc(&dwork, work));
  cudaStream_t st;
  CHECK_CUDA(cudaStreamCreate(&st));
  CHECK_CUDA(cudaMemcpy(dx, x, (size_t)M * K * 2, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dw, w, (size_t)N * K, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dws, ws, (size_t)N * 4, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dbias, bias, (size_t)N * 4, cudaMemcpyHostToDevice));

  h3q_status s = h3q_gemm_s8((const uint16_t*)dx, (const int8_t*)dw, (const float*)dws, N, (const float*)dbias,
                             (uint16_t*)dout, M, N, K, 0, 1, dwork, work, (void*)st);
  if (s != H3Q_OK) {
    fprintf(stderr, "h3q_gemm_s8: %s\n", h3q_last_error());
    return 1;
  }
  CHECK_CUDA(cudaStreamSynchronize(st));
  int code = -1;
  if (h3q_device_status(0, &code) != H3Q_OK || code != 0) {
    fprintf(stderr, "device status %d: %s\n", code, h3q_last_error());
    return 1;
  }
  CHECK_CUDA(cudaMemcpy(got, dout, (size_t)M * N * 2, cudaMemcpyDeviceToHost));
  int64_t bad = 0;
  for (int64_t i = 0; i < M * N; ++i) bad += got[i] != want[i];
  if (bad) {
    fprintf(stderr, "%lld of %lld bf16 outputs differ from the oracle\n", (long long)bad, (long long)(M * N));
    return 1;
  }
  /* attn8.rs:571-573: K % 64 != 0 is refused before any launch, with the reference's message */
  s = h3q_gemm_s8((const uint16_t*)dx, (const int8_t*)dw, (const float*)dws, N, NULL, (uint16_t*)dout, M, N, 100, 0,
                  0, dwork, work, (void*)st);
  if (s != H3Q_ERR_ARG || strlen(h3q_last_error()) == 0) {
    fprintf(stderr, "a K of 100 was not refused (status %d)\n", (int)s);
    return 1;
  }
  cudaStreamDestroy(st);
  cudaFree(dx);
  cudaFree(dw);
  cudaFree(dws);
  cudaFree(dbias);
  cudaFree(dout);
  cudaFree(dwork);
  free(x); free(w); free(ws); free(bias); free(q); free(xs); free(acc); free(want); free(got);
  printf("ok: h3q_gemm_s8 M=%lld K=%lld N=%lld from C, bit-exact vs the oracle\n", (long long)M, (long long)K,
         (long long)N);
  return 0;
}
