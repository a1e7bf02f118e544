// streaming.cu -- weight streaming (weights.rs:185-273 upload_u8_async / copy_stream, dit.rs:1160-1186): layer
// weights held in host memory are copied into a ring of device slots on a dedicated copy stream while the
// compute stream runs the layers before them.
//
// Ordering is carried by events on the device, so the host never waits: a fetch into slot k makes the copy
// stream wait for the compute stream's release of slot k's previous contents, and makes the compute stream wait
// for the copy.  The reference bounds how far its uploads run ahead by waiting on a host marker each block; here
// the ring's slot count is the bound.
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

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

struct h3q_streamer {
  int device = 0;
  size_t slot_bytes = 0;
  int slots = 0;
  int next = 0;
  uint8_t* mem = nullptr;
  cudaStream_t copy = nullptr;
  std::vector<cudaEvent_t> ready;  // copy into the slot finished (recorded on the copy stream)
  std::vector<cudaEvent_t> freed;  // the compute stream is done with the slot (recorded at release)
  std::vector<char> held;          // fetched and not yet released
  ~h3q_streamer() {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    if (copy) cudaStreamSynchronize(copy);
    for (cudaEvent_t e : freed)
      if (e) cudaEventSynchronize(e);
    for (cudaEvent_t e : ready)
      if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : freed)
      if (e) cudaEventDestroy(e);
    if (copy) cudaStreamDestroy(copy);
    if (mem) cudaFree(mem);
    cudaSetDevice(cur);
  }
};

extern "C" {

h3q_status h3q_streamer_create(size_t slot_bytes, int slots, h3q_streamer** out) {
  const char* what = "h3q_streamer_create";
  if (!out) return fail(H3Q_ERR_ARG, "%s: null output pointer", what);
  *out = nullptr;
  if (slots < 1 || slots > 64 || slot_bytes == 0)
    return fail(H3Q_ERR_ARG, "%s: %d slots of %zu bytes (1..64 non-empty slots)", what, slots, slot_bytes);
  h3q_streamer* s = new h3q_streamer;
  cudaGetDevice(&s->device);
  s->slot_bytes = align256(slot_bytes);
  s->slots = slots;
  s->ready.assign(slots, nullptr);
  s->freed.assign(slots, nullptr);
  s->held.assign(slots, 0);
  h3q_status st = cuda_status(cudaMalloc(&s->mem, s->slot_bytes * (size_t)slots), what);
  if (st == H3Q_OK) st = cuda_status(cudaStreamCreateWithFlags(&s->copy, cudaStreamNonBlocking), what);
  for (int i = 0; i < slots && st == H3Q_OK; ++i) {
    st = cuda_status(cudaEventCreateWithFlags(&s->ready[i], cudaEventDisableTiming), what);
    if (st == H3Q_OK) st = cuda_status(cudaEventCreateWithFlags(&s->freed[i], cudaEventDisableTiming), what);
  }
  if (st != H3Q_OK) {
    delete s;
    return st;
  }
  *out = s;
  return H3Q_OK;
}

void h3q_streamer_destroy(h3q_streamer* s) { delete s; }

size_t h3q_streamer_slot_bytes(const h3q_streamer* s) { return s ? s->slot_bytes : 0; }

h3q_status h3q_streamer_fetch(h3q_streamer* s, const void* const* src, const size_t* bytes, int n,
                              void* compute_stream, int* slot, void** dst) {
  const char* what = "h3q_streamer_fetch";
  if (!s || !src || !bytes || !slot || !dst || n < 1) return fail(H3Q_ERR_ARG, "%s: null argument", what);
  size_t total = 0;
  for (int i = 0; i < n; ++i) {
    if (!src[i] && bytes[i]) return fail(H3Q_ERR_ARG, "%s: region %d has no source", what, i);
    total += align256(bytes[i]);
  }
  if (total > s->slot_bytes)
    return fail(H3Q_ERR_ARG, "%s: %zu bytes (256-byte aligned regions) exceed the slot size %zu", what, total,
                s->slot_bytes);
  const int k = s->next;
  if (s->held[k])
    return fail(H3Q_ERR_ARG, "%s: slot %d is still held (release it after enqueuing its last reader)", what, k);
  s->next = (s->next + 1) % s->slots;
  cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
  // the slot's previous contents are no longer read once the compute stream passes their release
  if (h3q_status e = cuda_status(cudaStreamWaitEvent(s->copy, s->freed[k], 0), what)) return e;
  uint8_t* base = s->mem + (size_t)k * s->slot_bytes;
  size_t off = 0;
  for (int i = 0; i < n; ++i) {
    dst[i] = base + off;
    if (bytes[i])
      if (h3q_status e = cuda_status(cudaMemcpyAsync(base + off, src[i], bytes[i], cudaMemcpyHostToDevice, s->copy),
                                     what))
        return e;
    off += align256(bytes[i]);
  }
  if (h3q_status e = cuda_status(cudaEventRecord(s->ready[k], s->copy), what)) return e;
  if (h3q_status e = cuda_status(cudaStreamWaitEvent(cs, s->ready[k], 0), what)) return e;
  s->held[k] = 1;
  *slot = k;
  return H3Q_OK;
}

h3q_status h3q_streamer_release(h3q_streamer* s, int slot, void* compute_stream) {
  const char* what = "h3q_streamer_release";
  if (!s || slot < 0 || slot >= s->slots || !s->held[slot])
    return fail(H3Q_ERR_ARG, "%s: slot %d is not held", what, slot);
  s->held[slot] = 0;
  return cuda_status(cudaEventRecord(s->freed[slot], static_cast<cudaStream_t>(compute_stream)), what);
}

}  // extern "C"
