// host_pipeline.cu -- the quantized linear on activations that live in host memory: row chunks are copied in on one
// copy stream, multiplied on the caller's stream, and copied out on a second copy stream, double-buffered, so the
// two PCIe directions and the GEMMs overlap (the link is full duplex).  The reference's public ops take device
// tensors; this is the path for a caller whose activations arrive from and return to the host.
//
// Per chunk c (buffers b = c mod 2):  in:  wait until the GEMM of chunk c-2 has read x[b]; copy x rows -> x[b]
//                                     compute: wait for x[b] and for the copy-out of chunk c-2 from o[b]; gemm_s8
//                                     out: wait for the GEMM; copy o[b] -> out rows
// A call starts after the work already on the caller's stream and the caller's stream waits for its last copy
// out, so calls chain like any stream-ordered operation (one call's host output may be the next call's input).
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>
#include "../../include/h3q.h"

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

}  // namespace

struct h3q_host_pipeline {
  int device = 0;
  int64_t chunk_rows = 0, max_k = 0, max_n = 0;
  cudaStream_t in = nullptr, out = nullptr;
  uint16_t* xbuf[2] = {nullptr, nullptr};
  uint16_t* obuf[2] = {nullptr, nullptr};
  void* ws = nullptr;
  size_t ws_bytes = 0;
  cudaEvent_t start = nullptr, done = nullptr;
  cudaEvent_t x_ready[2] = {}, x_free[2] = {}, o_ready[2] = {}, o_free[2] = {};
  ~h3q_host_pipeline() {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    if (in) cudaStreamSynchronize(in);
    if (out) cudaStreamSynchronize(out);
    cudaEvent_t* evs[] = {&start, &done, &x_ready[0], &x_ready[1], &x_free[0], &x_free[1],
                          &o_ready[0], &o_ready[1], &o_free[0], &o_free[1]};
    for (cudaEvent_t* e : evs) {
      if (*e) {
        cudaEventSynchronize(*e);
        cudaEventDestroy(*e);
      }
    }
    for (int b = 0; b < 2; ++b) {
      if (xbuf[b]) cudaFree(xbuf[b]);
      if (obuf[b]) cudaFree(obuf[b]);
    }
    if (ws) cudaFree(ws);
    if (in) cudaStreamDestroy(in);
    if (out) cudaStreamDestroy(out);
    cudaSetDevice(cur);
  }
};

extern "C" {

h3q_status h3q_host_pipeline_create(int64_t chunk_rows, int64_t max_k, int64_t max_n, h3q_host_pipeline** out) {
  const char* what = "h3q_host_pipeline_create";
  if (!out) return fail(H3Q_ERR_ARG, "%s: null output pointer", what);
  *out = nullptr;
  if (chunk_rows < 1 || max_k < 1 || max_n < 1)
    return fail(H3Q_ERR_ARG, "%s: chunk_rows, max_k and max_n must be positive", what);
  h3q_host_pipeline* p = new h3q_host_pipeline;
  cudaGetDevice(&p->device);
  p->chunk_rows = chunk_rows;
  p->max_k = max_k;
  p->max_n = max_n;
  p->ws_bytes = h3q_gemm_s8_workspace_size(chunk_rows, max_k);
  h3q_status st = H3Q_OK;
  auto chk = [&](cudaError_t e) {
    if (st == H3Q_OK) st = cuda_status(e, what);
  };
  chk(cudaStreamCreateWithFlags(&p->in, cudaStreamNonBlocking));
  chk(cudaStreamCreateWithFlags(&p->out, cudaStreamNonBlocking));
  for (int b = 0; b < 2 && st == H3Q_OK; ++b) {
    chk(cudaMalloc(&p->xbuf[b], (size_t)chunk_rows * max_k * 2));
    chk(cudaMalloc(&p->obuf[b], (size_t)chunk_rows * max_n * 2));
  }
  chk(cudaMalloc(&p->ws, p->ws_bytes));
  cudaEvent_t* evs[] = {&p->start, &p->done, &p->x_ready[0], &p->x_ready[1], &p->x_free[0], &p->x_free[1],
                        &p->o_ready[0], &p->o_ready[1], &p->o_free[0], &p->o_free[1]};
  for (cudaEvent_t* e : evs) chk(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  if (st != H3Q_OK) {
    delete p;
    return st;
  }
  *out = p;
  return H3Q_OK;
}

void h3q_host_pipeline_destroy(h3q_host_pipeline* p) { delete p; }

h3q_status h3q_host_pipeline_gemm_s8(h3q_host_pipeline* p, const uint16_t* x_host, const int8_t* w, const float* ws,
                                     int64_t ws_numel, const float* bias, uint16_t* out_host, int64_t m, int64_t n,
                                     int64_t k, int swiglu, int rotate, void* stream) {
  const char* what = "h3q_host_pipeline_gemm_s8";
  if (!p) return fail(H3Q_ERR_ARG, "%s: null pipeline", what);
  if (m < 0 || n < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  const int64_t n_out = swiglu ? n / 2 : n;
  if (k > p->max_k || n_out > p->max_n)
    return fail(H3Q_ERR_ARG, "%s: k = %lld and output width %lld exceed the pipeline's %lld and %lld", what,
                (long long)k, (long long)n_out, (long long)p->max_k, (long long)p->max_n);
  if (m == 0 || n == 0) return H3Q_OK;
  if (!x_host || !out_host) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  if (h3q_status s = cuda_status(cudaEventRecord(p->start, cs), what)) return s;
  if (h3q_status s = cuda_status(cudaStreamWaitEvent(p->in, p->start, 0), what)) return s;
  const int64_t chunks = (m + p->chunk_rows - 1) / p->chunk_rows;
  for (int64_t c = 0; c < chunks; ++c) {
    const int b = (int)(c & 1);
    const int64_t r0 = c * p->chunk_rows;
    const int64_t rows = (m - r0) < p->chunk_rows ? (m - r0) : p->chunk_rows;
    // copy in: the GEMM of chunk c-2 no longer reads x[b]
    if (c >= 2)
      if (h3q_status s = cuda_status(cudaStreamWaitEvent(p->in, p->x_free[b], 0), what)) return s;
    if (h3q_status s = cuda_status(cudaMemcpyAsync(p->xbuf[b], x_host + r0 * k, (size_t)rows * k * 2,
                                                   cudaMemcpyHostToDevice, p->in), what))
      return s;
    if (h3q_status s = cuda_status(cudaEventRecord(p->x_ready[b], p->in), what)) return s;
    // compute: x[b] has arrived and the copy-out of chunk c-2 has left o[b]
    if (h3q_status s = cuda_status(cudaStreamWaitEvent(cs, p->x_ready[b], 0), what)) return s;
    if (c >= 2)
      if (h3q_status s = cuda_status(cudaStreamWaitEvent(cs, p->o_free[b], 0), what)) return s;
    if (h3q_status s = h3q_gemm_s8(p->xbuf[b], w, ws, ws_numel, bias, p->obuf[b], rows, n, k, swiglu, rotate, p->ws,
                                   p->ws_bytes, stream))
      return s;
    if (h3q_status s = cuda_status(cudaEventRecord(p->x_free[b], cs), what)) return s;
    if (h3q_status s = cuda_status(cudaEventRecord(p->o_ready[b], cs), what)) return s;
    // copy out
    if (h3q_status s = cuda_status(cudaStreamWaitEvent(p->out, p->o_ready[b], 0), what)) return s;
    if (h3q_status s = cuda_status(cudaMemcpyAsync(out_host + r0 * n_out, p->obuf[b], (size_t)rows * n_out * 2,
                                                   cudaMemcpyDeviceToHost, p->out), what))
      return s;
    if (h3q_status s = cuda_status(cudaEventRecord(p->o_free[b], p->out), what)) return s;
  }
  if (h3q_status s = cuda_status(cudaEventRecord(p->done, p->out), what)) return s;
  return cuda_status(cudaStreamWaitEvent(cs, p->done, 0), what);
}

}  // extern "C"
