// host_pipeline.cu -- the quantized linear on activations that live in host memory: row chunks are copied in on one
// copy stream, multiplied on the caller's stream, and copied out on a second copy stream, double-buffered, so the
// two PCIe directions and the GEMMs overlap (the link is full duplex).  The reference's public ops take device
// tensors; this is the path for a caller whose activations arrive from and return to the host.
//
// Per chunk c, with nx input and no output chunk buffers (two each unless created with more):
//   in:      wait until the GEMM of chunk c-nx has read x[c mod nx]; copy x rows -> x[c mod nx]
//   compute: wait for x[c mod nx] and for the copy-out of chunk c-no from o[c mod no]; gemm_s8
//   out:     wait for the GEMM; copy o[c mod no] -> out rows
// More input buffers let the copies in run further ahead of the GEMMs: a batch whose later linears have wide
// inputs (fc2) then moves them while the earlier linears are still bound by their copies out.
// A call starts after the work already on the caller's stream and the caller's stream waits for its last copy
// out, so calls chain like any stream-ordered operation (one call's host output may be the next call's input).
// h3q_host_pipeline_run enqueues several linears as one sequence: the chunk numbering, and with it the buffer
// hand-over above, runs on across the linears, so linear i+1 copies in while linear i still computes and copies
// out.  A linear whose host input overlaps an earlier linear's host output waits for every copy out enqueued before
// it.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <vector>
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
  std::vector<uint16_t*> xbuf, obuf;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  cudaEvent_t start = nullptr, done = nullptr, outs_so_far = nullptr;
  std::vector<cudaEvent_t> x_ready, x_free, o_ready, o_free;
  ~h3q_host_pipeline() {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    if (in) cudaStreamSynchronize(in);
    if (out) cudaStreamSynchronize(out);
    std::vector<cudaEvent_t*> evs = {&start, &done, &outs_so_far};
    for (auto* v : {&x_ready, &x_free, &o_ready, &o_free})
      for (cudaEvent_t& e : *v) evs.push_back(&e);
    for (cudaEvent_t* e : evs) {
      if (*e) {
        cudaEventSynchronize(*e);
        cudaEventDestroy(*e);
      }
    }
    for (uint16_t* b : xbuf)
      if (b) cudaFree(b);
    for (uint16_t* b : obuf)
      if (b) cudaFree(b);
    if (ws) cudaFree(ws);
    if (in) cudaStreamDestroy(in);
    if (out) cudaStreamDestroy(out);
    cudaSetDevice(cur);
  }
};

extern "C" {

h3q_status h3q_host_pipeline_create_ex(int64_t chunk_rows, int64_t max_k, int64_t max_n, int in_slots, int out_slots,
                                       h3q_host_pipeline** out) {
  const char* what = "h3q_host_pipeline_create";
  if (!out) return fail(H3Q_ERR_ARG, "%s: null output pointer", what);
  *out = nullptr;
  if (chunk_rows < 1 || max_k < 1 || max_n < 1)
    return fail(H3Q_ERR_ARG, "%s: chunk_rows, max_k and max_n must be positive", what);
  if (in_slots < 2 || out_slots < 2 || in_slots > 4096 || out_slots > 4096)
    return fail(H3Q_ERR_ARG, "%s: in_slots and out_slots must be in [2, 4096]", what);
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
  p->xbuf.assign(in_slots, nullptr);
  p->obuf.assign(out_slots, nullptr);
  p->x_ready.assign(in_slots, nullptr);
  p->x_free.assign(in_slots, nullptr);
  p->o_ready.assign(out_slots, nullptr);
  p->o_free.assign(out_slots, nullptr);
  for (int b = 0; b < in_slots && st == H3Q_OK; ++b) chk(cudaMalloc(&p->xbuf[b], (size_t)chunk_rows * max_k * 2));
  for (int b = 0; b < out_slots && st == H3Q_OK; ++b) chk(cudaMalloc(&p->obuf[b], (size_t)chunk_rows * max_n * 2));
  chk(cudaMalloc(&p->ws, p->ws_bytes));
  std::vector<cudaEvent_t*> evs = {&p->start, &p->done, &p->outs_so_far};
  for (auto* v : {&p->x_ready, &p->x_free, &p->o_ready, &p->o_free})
    for (cudaEvent_t& e : *v) evs.push_back(&e);
  for (cudaEvent_t* e : evs) chk(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  if (st != H3Q_OK) {
    delete p;
    return st;
  }
  *out = p;
  return H3Q_OK;
}

h3q_status h3q_host_pipeline_create(int64_t chunk_rows, int64_t max_k, int64_t max_n, h3q_host_pipeline** out) {
  return h3q_host_pipeline_create_ex(chunk_rows, max_k, max_n, 2, 2, out);
}

void h3q_host_pipeline_destroy(h3q_host_pipeline* p) { delete p; }

h3q_status h3q_host_pipeline_run(h3q_host_pipeline* p, const h3q_host_linear* items, int count, void* stream) {
  const char* what = "h3q_host_pipeline_run";
  if (!p) return fail(H3Q_ERR_ARG, "%s: null pipeline", what);
  if (count < 0 || (count > 0 && !items)) return fail(H3Q_ERR_ARG, "%s: bad item list", what);
  // every item is checked before anything is enqueued
  for (int i = 0; i < count; ++i) {
    const h3q_host_linear& it = items[i];
    if (it.m < 0 || it.n < 0 || it.k < 0) return fail(H3Q_ERR_ARG, "%s: item %d: negative shape", what, i);
    const int64_t n_out = it.swiglu ? it.n / 2 : it.n;
    if (it.k > p->max_k || n_out > p->max_n)
      return fail(H3Q_ERR_ARG, "%s: item %d: k = %lld and output width %lld exceed the pipeline's %lld and %lld",
                  what, i, (long long)it.k, (long long)n_out, (long long)p->max_k, (long long)p->max_n);
    if (it.m > 0 && it.n > 0 && (!it.x_host || !it.out_host))
      return fail(H3Q_ERR_ARG, "%s: item %d: null pointer", what, i);
  }
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  if (h3q_status s = cuda_status(cudaEventRecord(p->start, cs), what)) return s;
  if (h3q_status s = cuda_status(cudaStreamWaitEvent(p->in, p->start, 0), what)) return s;
  int64_t gc = 0;  // chunk number across the whole sequence
  const int64_t nx = (int64_t)p->xbuf.size(), no = (int64_t)p->obuf.size();
  for (int i = 0; i < count; ++i) {
    const h3q_host_linear& it = items[i];
    if (it.m == 0 || it.n == 0) continue;
    const int64_t n_out = it.swiglu ? it.n / 2 : it.n;
    const uintptr_t x0 = (uintptr_t)it.x_host, x1 = x0 + (uintptr_t)(it.m * it.k * 2);
    bool reads_earlier_output = false;
    for (int e = 0; e < i; ++e) {
      const h3q_host_linear& pe = items[e];
      if (pe.m == 0 || pe.n == 0) continue;
      const uintptr_t o0 = (uintptr_t)pe.out_host;
      const uintptr_t o1 = o0 + (uintptr_t)(pe.m * (pe.swiglu ? pe.n / 2 : pe.n) * 2);
      if (x0 < o1 && o0 < x1) reads_earlier_output = true;
    }
    if (reads_earlier_output) {
      if (h3q_status s = cuda_status(cudaEventRecord(p->outs_so_far, p->out), what)) return s;
      if (h3q_status s = cuda_status(cudaStreamWaitEvent(p->in, p->outs_so_far, 0), what)) return s;
    }
    const int64_t chunks = (it.m + p->chunk_rows - 1) / p->chunk_rows;
    for (int64_t c = 0; c < chunks; ++c, ++gc) {
      const int bx = (int)(gc % nx), bo = (int)(gc % no);
      const int64_t r0 = c * p->chunk_rows;
      const int64_t rows = (it.m - r0) < p->chunk_rows ? (it.m - r0) : p->chunk_rows;
      // copy in: the GEMM nx chunks back no longer reads x[bx]
      if (gc >= nx)
        if (h3q_status s = cuda_status(cudaStreamWaitEvent(p->in, p->x_free[bx], 0), what)) return s;
      if (h3q_status s = cuda_status(cudaMemcpyAsync(p->xbuf[bx], it.x_host + r0 * it.k, (size_t)rows * it.k * 2,
                                                     cudaMemcpyHostToDevice, p->in), what))
        return s;
      if (h3q_status s = cuda_status(cudaEventRecord(p->x_ready[bx], p->in), what)) return s;
      // compute: x[bx] has arrived and the copy out no chunks back has left o[bo]
      if (h3q_status s = cuda_status(cudaStreamWaitEvent(cs, p->x_ready[bx], 0), what)) return s;
      if (gc >= no)
        if (h3q_status s = cuda_status(cudaStreamWaitEvent(cs, p->o_free[bo], 0), what)) return s;
      if (h3q_status s = h3q_gemm_s8(p->xbuf[bx], it.w, it.ws, it.ws_numel, it.bias, p->obuf[bo], rows, it.n, it.k,
                                     it.swiglu, it.rotate, p->ws, p->ws_bytes, stream))
        return s;
      if (h3q_status s = cuda_status(cudaEventRecord(p->x_free[bx], cs), what)) return s;
      if (h3q_status s = cuda_status(cudaEventRecord(p->o_ready[bo], cs), what)) return s;
      // copy out
      if (h3q_status s = cuda_status(cudaStreamWaitEvent(p->out, p->o_ready[bo], 0), what)) return s;
      if (h3q_status s = cuda_status(cudaMemcpyAsync(it.out_host + r0 * n_out, p->obuf[bo], (size_t)rows * n_out * 2,
                                                     cudaMemcpyDeviceToHost, p->out), what))
        return s;
      if (h3q_status s = cuda_status(cudaEventRecord(p->o_free[bo], p->out), what)) return s;
    }
  }
  if (h3q_status s = cuda_status(cudaEventRecord(p->done, p->out), what)) return s;
  return cuda_status(cudaStreamWaitEvent(cs, p->done, 0), what);
}

h3q_status h3q_host_pipeline_gemm_s8(h3q_host_pipeline* p, const uint16_t* x_host, const int8_t* w, const float* ws,
                                     int64_t ws_numel, const float* bias, uint16_t* out_host, int64_t m, int64_t n,
                                     int64_t k, int swiglu, int rotate, void* stream) {
  if (!p) return fail(H3Q_ERR_ARG, "h3q_host_pipeline_gemm_s8: null pipeline");
  const h3q_host_linear it{x_host, w, ws, ws_numel, bias, out_host, m, n, k, swiglu, rotate};
  return h3q_host_pipeline_run(p, &it, 1, stream);
}

}  // extern "C"
