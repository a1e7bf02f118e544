// comm.cu -- the multi-GPU data plane of the C ABI (one process per GPU): NCCL communicators, a byte all-gather, a
// cross-rank barrier, and the N-split linear step with its all-gather of output columns in four forms.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring a copy the process has already loaded, such as
// the one a framework brought in), so the library neither links nor pins an NCCL build; a process without NCCL
// gets H3Q_ERR_NCCL from these entry points and everything else keeps working.
//
// N-split (weight rows = output columns split over the ranks, activations replicated): rank r computes the columns
// h3q_nsplit_range(n_total, g, r) of every output row, and every rank ends up with the whole [m, n_total] output.
//   H3Q_NSPLIT_FUSED  one GEMM whose epilogue TMA-stores each output box into every rank's buffer (peer memory
//                     over NVLink): the transfer runs inside the GEMM, tile by tile;
//   H3Q_NSPLIT_PUSH   the GEMM in row chunks, each writing its column block into this rank's own buffer, and the
//                     copy engines pushing each finished chunk into every peer's buffer (2-D copies over NVLink,
//                     straight into the final column positions) while the next chunk computes;
//   H3Q_NSPLIT_NCCL   a local GEMM into a packed block, ncclAllGather of the blocks, and a relayout kernel
//                     (the library-collective baseline);
//   H3Q_NSPLIT_PEER   the GEMM into this rank's own buffer, then a kernel on every SM storing the column block
//                     into every peer's buffer, a warp per row, whole 512-byte stores, one peer per phase.
// FUSED, PUSH and PEER write into peers' buffers, so a barrier first makes sure every rank has finished with the
// previous contents of its output (stream-ordered), and a barrier last makes the complete output readable.
#include <dlfcn.h>
#include <nccl.h>
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

// ------------------------------------------------------------------------------------------------ NCCL at run time
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string why;  // empty when every symbol resolved
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // a copy already in the process
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (!h) {
      const char* e = dlerror();
      api.why = std::string("cannot load libnccl.so.2: ") + (e ? e : "?");
      return;
    }
    auto sym = [&](const char* name) -> void* {
      void* p = dlsym(h, name);
      if (!p && api.why.empty()) api.why = std::string("libnccl.so.2 lacks ") + name;
      return p;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
  });
  return api;
}

h3q_status nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return H3Q_OK;
  return fail(H3Q_ERR_NCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

h3q_status need_nccl(const char* what) {
  if (!nccl().why.empty()) return fail(H3Q_ERR_NCCL, "%s: %s", what, nccl().why.c_str());
  return H3Q_OK;
}

constexpr int kPushChunks = 4;     // row chunks of the PUSH form: chunk c's copies overlap chunk c+1's GEMM
constexpr int kMaxPeers = 15;      // copy streams of the PUSH form (one per peer)
constexpr int64_t kNsplitAlign = 256;  // the GEMM's tile width: every column block but the last is whole tiles

// Columns of rank r: whole 256-column tiles, spread as evenly as the tile count allows.
void range_of(int64_t n, int g, int r, int64_t* lo, int64_t* hi) {
  const int64_t tiles = (n + kNsplitAlign - 1) / kNsplitAlign;
  const int64_t t0 = tiles * r / g, t1 = tiles * (r + 1) / g;
  *lo = t0 * kNsplitAlign < n ? t0 * kNsplitAlign : n;
  *hi = t1 * kNsplitAlign < n ? t1 * kNsplitAlign : n;
}

int64_t widest_block(int64_t n, int g) {
  int64_t w = 0;
  for (int r = 0; r < g; ++r) {
    int64_t lo, hi;
    range_of(n, g, r, &lo, &hi);
    if (hi - lo > w) w = hi - lo;
  }
  return w;
}

// out[row, lo_r + c] = blocks[r][row][c] for c < width of rank r: the NCCL form's gathered [g][m][nmax] blocks into
// the [m, n] output.  One (rank, row) per block-iteration, 16 bytes per thread (every block offset and width is a
// multiple of 8 columns); the rank's column range is worked out once per row, not per element.
__global__ void __launch_bounds__(256) nsplit_relayout_kernel(const uint16_t* __restrict__ blocks,
                                                              uint16_t* __restrict__ out, int64_t m, int64_t n,
                                                              int64_t nmax, int g) {
  const int64_t tiles = (n + kNsplitAlign - 1) / kNsplitAlign;
  for (int64_t rr = blockIdx.x; rr < (int64_t)g * m; rr += gridDim.x) {
    const int r = (int)(rr / m);
    const int64_t row = rr - (int64_t)r * m;
    const int64_t t0 = tiles * r / g, t1 = tiles * (r + 1) / g;
    const int64_t lo = t0 * kNsplitAlign < n ? t0 * kNsplitAlign : n;
    const int64_t hi = t1 * kNsplitAlign < n ? t1 * kNsplitAlign : n;
    const uint4* src = reinterpret_cast<const uint4*>(blocks + rr * nmax);
    uint4* dst = reinterpret_cast<uint4*>(out + row * n + lo);
    for (int64_t v = threadIdx.x; v < (hi - lo) / 8; v += blockDim.x) dst[v] = __ldg(src + v);
  }
}

// The PEER form's exchange: this rank's column block [lo, lo + width) of rows [0, m) of its own output, read 16
// bytes at a time and stored to the same place in every peer's output (peer memory over NVLink), every SM taking
// part.  One warp per row: each store instruction writes 512 contiguous bytes of the row to ONE peer, so NVLink
// carries whole lines (a destination that changed from lane to lane split every warp store into 16-byte pieces
// bound for seven GPUs and ran 2.6x slower at 8 ranks).  The peers are served in phases: in phase d every warp
// stores to p[d] only, rank (r + 1 + d) mod g, so while the ranks run the same phase every GPU sends to one GPU
// and receives from one.  The block is re-read once per phase, mostly from L2.
constexpr int kMaxPeerDst = 8;
struct PeerDsts {
  uint16_t* p[kMaxPeerDst];  // peers' outputs in phase order (this rank's own excluded)
  int n;
};

__global__ void __launch_bounds__(512) nsplit_peer_store_kernel(const uint16_t* __restrict__ own, PeerDsts dsts,
                                                                int64_t m, int64_t n, int64_t lo, int64_t width) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t w0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int vpr = (int)(width / 8);  // 16-byte vectors per row
#pragma unroll 1
  for (int d = 0; d < dsts.n; ++d) {  // phase d: every warp stores to peer p[d] only
    uint16_t* out = dsts.p[d];
    for (int64_t row = w0; row < m; row += warps) {
      const int64_t base = row * n + lo;
      const uint4* src = reinterpret_cast<const uint4*>(own + base);
      uint4* dst = reinterpret_cast<uint4*>(out + base);
      for (int v = lane; v < vpr; v += 32) dst[v] = __ldg(src + v);
    }
  }
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

struct h3q_comm {
  ncclComm_t nc = nullptr;
  int rank = 0, nranks = 0, device = 0;
  float* flag = nullptr;                // one device float: the barrier's all-reduce operand
  // PUSH: one copy stream per peer (its copies run on their own copy engine, in parallel with the other peers'),
  // the chunk-done and call-start events every copy stream waits on, and one copies-done event per copy stream
  cudaStream_t copy[kMaxPeers] = {};
  cudaEvent_t ev[kPushChunks + 1] = {};
  cudaEvent_t done[kMaxPeers] = {};
};

extern "C" {

h3q_status h3q_comm_unique_id(void* id) {
  const char* what = "h3q_comm_unique_id";
  if (!id) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if (h3q_status s = need_nccl(what)) return s;
  ncclUniqueId u;
  if (h3q_status s = nccl_status(nccl().get_unique_id(&u), what)) return s;
  memcpy(id, &u, sizeof u);
  return H3Q_OK;
}

h3q_status h3q_comm_init(int nranks, int rank, const void* id, h3q_comm** comm) {
  const char* what = "h3q_comm_init";
  static_assert(sizeof(ncclUniqueId) == H3Q_COMM_ID_BYTES, "NCCL unique id size");
  if (!comm || !id) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  *comm = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(H3Q_ERR_ARG, "%s: rank %d of %d", what, rank, nranks);
  if (h3q_status s = need_nccl(what)) return s;
  h3q_comm* c = new h3q_comm();
  c->rank = rank;
  c->nranks = nranks;
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(&c->flag, sizeof(float));
  if (e == cudaSuccess) e = cudaMemset(c->flag, 0, sizeof(float));
  for (int i = 0; i + 1 < nranks && i < kMaxPeers && e == cudaSuccess; ++i) {
    e = cudaStreamCreateWithFlags(&c->copy[i], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->done[i], cudaEventDisableTiming);
  }
  for (int i = 0; i < kPushChunks + 1 && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&c->ev[i], cudaEventDisableTiming);
  h3q_status st = cuda_status(e, what);
  if (st == H3Q_OK) {
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    st = nccl_status(nccl().comm_init_rank(&c->nc, nranks, u, rank), what);
  }
  if (st != H3Q_OK) {
    h3q_comm_destroy(c);
    return st;
  }
  *comm = c;
  return H3Q_OK;
}

h3q_status h3q_comm_destroy(h3q_comm* c) {
  if (!c) return H3Q_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  h3q_status st = H3Q_OK;
  if (c->nc) st = nccl_status(nccl().comm_destroy(c->nc), "h3q_comm_destroy");
  for (cudaEvent_t& ev : c->ev)
    if (ev) cudaEventDestroy(ev);
  for (int i = 0; i < kMaxPeers; ++i) {
    if (c->done[i]) cudaEventDestroy(c->done[i]);
    if (c->copy[i]) cudaStreamDestroy(c->copy[i]);
  }
  if (c->flag) cudaFree(c->flag);
  cudaSetDevice(prev);
  delete c;
  return st;
}

int h3q_comm_rank(const h3q_comm* c) { return c ? c->rank : -1; }
int h3q_comm_size(const h3q_comm* c) { return c ? c->nranks : 0; }

h3q_status h3q_comm_allgather(h3q_comm* c, const void* send, void* recv, size_t bytes_per_rank, void* stream) {
  const char* what = "h3q_comm_allgather";
  if (!c) return fail(H3Q_ERR_ARG, "%s: null communicator", what);
  if (bytes_per_rank == 0) return H3Q_OK;
  if (!send || !recv) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  return nccl_status(nccl().all_gather(send, recv, bytes_per_rank, ncclUint8, c->nc, static_cast<cudaStream_t>(stream)),
                     what);
}

h3q_status h3q_comm_barrier(h3q_comm* c, void* stream) {
  const char* what = "h3q_comm_barrier";
  if (!c) return fail(H3Q_ERR_ARG, "%s: null communicator", what);
  return nccl_status(nccl().all_reduce(c->flag, c->flag, 1, ncclFloat32, ncclSum, c->nc,
                                       static_cast<cudaStream_t>(stream)),
                     what);
}

void h3q_nsplit_range(int64_t n, int nranks, int rank, int64_t* lo, int64_t* hi) {
  int64_t a = 0, b = 0;
  if (n > 0 && nranks > 0 && rank >= 0 && rank < nranks) range_of(n, nranks, rank, &a, &b);
  if (lo) *lo = a;
  if (hi) *hi = b;
}

size_t h3q_gemm_s8_nsplit_workspace_size(int64_t m, int64_t n_total, int nranks, int mode) {
  if (mode != H3Q_NSPLIT_NCCL || m <= 0 || n_total <= 0 || nranks < 1) return 0;
  const size_t block = (size_t)m * (size_t)widest_block(n_total, nranks) * 2;
  return align256(block) + (size_t)nranks * block;
}

h3q_status h3q_gemm_s8_nsplit(h3q_comm* c, int mode, const int8_t* a, const float* xs, const int8_t* w_local,
                              const float* ws_local, int64_t ws_numel, const float* bias_local, void* const* outs,
                              int64_t m, int64_t n_total, int64_t k, void* workspace, size_t workspace_bytes,
                              void* stream) {
  const char* what = "h3q_gemm_s8_nsplit";
  if (!c) return fail(H3Q_ERR_ARG, "%s: null communicator", what);
  if (mode != H3Q_NSPLIT_FUSED && mode != H3Q_NSPLIT_PUSH && mode != H3Q_NSPLIT_NCCL && mode != H3Q_NSPLIT_PEER)
    return fail(H3Q_ERR_ARG, "%s: unknown mode %d", what, mode);
  if (mode == H3Q_NSPLIT_PEER && c->nranks > kMaxPeerDst + 1)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: the peer form stores to at most %d peers", what, kMaxPeerDst);
  if (m < 0 || n_total < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  const int g = c->nranks, r = c->rank;
  if (mode == H3Q_NSPLIT_FUSED && g > h3q::kMaxGatherRanks)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: the fused form stores to at most %d ranks", what, h3q::kMaxGatherRanks);
  if (!outs) return fail(H3Q_ERR_ARG, "%s: null output list", what);
  if (n_total % 8 != 0) return fail(H3Q_ERR_ARG, "%s: n_total must be a multiple of 8 (16-byte rows)", what);
  if (k == 0 || k % 16 != 0)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: this build needs k %% 16 == 0 and k > 0 (k = %lld)", what, (long long)k);
  for (int d = 0; d < g; ++d) {
    if (mode == H3Q_NSPLIT_NCCL && d != r) continue;
    if (!outs[d] || (reinterpret_cast<uintptr_t>(outs[d]) & 15u))
      return fail(H3Q_ERR_ARG, "%s: output %d null or not 16-byte aligned", what, d);
  }
  int64_t lo, hi;
  range_of(n_total, g, r, &lo, &hi);
  const int64_t nl = hi - lo;
  const size_t need = h3q_gemm_s8_nsplit_workspace_size(m, n_total, g, mode);
  if (workspace_bytes < need)
    return fail(H3Q_ERR_WORKSPACE, "%s: workspace of %zu bytes, %zu needed", what, workspace_bytes, need);
  if (m == 0 || n_total == 0) return H3Q_OK;
  if (!a || !xs || !w_local || !ws_local || ws_numel < 1) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  h3q::GemmArgs ga{};
  ga.K = k;
  ga.ws = ws_local;
  ga.ws_per_row = (ws_numel == nl && nl > 1) ? 1 : 0;
  ga.bias = bias_local;
  ga.out_kind = 2;
  ga.epi = h3q::kEpiLinear;
  ga.err = h3q::error_word_current();
  if (!ga.err) return fail(H3Q_ERR_CUDA, "%s: could not set up the device error word", what);

  if (mode == H3Q_NSPLIT_NCCL) {
    const int64_t nmax = widest_block(n_total, g);
    uint16_t* send = static_cast<uint16_t*>(workspace);
    uint16_t* recv = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(workspace) + align256((size_t)m * nmax * 2));
    if (nl > 0) {
      ga.M = m;
      ga.N = nl;
      ga.xs = xs;
      ga.out = send;
      void* dst[1] = {send};
      if (h3q_status s = cuda_status(h3q::launch_gemm_i8_allgather(a, w_local, ga, dst, 1, nmax, 0, st), what)) return s;
    }
    if (h3q_status s = nccl_status(nccl().all_gather(send, recv, (size_t)m * nmax * 2, ncclUint8, c->nc, st), what))
      return s;
    const int64_t rows = (int64_t)g * m;
    nsplit_relayout_kernel<<<(unsigned)(rows < 16 * 148 ? rows : 16 * 148), 256, 0, st>>>(
        recv, static_cast<uint16_t*>(outs[r]), m, n_total, nmax, g);
    return cuda_status(cudaGetLastError(), what);
  }

  // FUSED and PUSH: every rank must be done with its output buffer's previous contents before peers write into it
  if (h3q_status s = h3q_comm_barrier(c, stream)) return s;
  if (mode == H3Q_NSPLIT_PEER) {
    // the GEMM writes this rank's columns into its own output, then every SM forwards them to the peers
    if (nl > 0) {
      ga.M = m;
      ga.N = nl;
      ga.xs = xs;
      ga.out = outs[r];
      void* dst[1] = {outs[r]};
      if (h3q_status s = cuda_status(h3q::launch_gemm_i8_allgather(a, w_local, ga, dst, 1, n_total, lo, st), what))
        return s;
      PeerDsts pd{};
      pd.n = 0;
      for (int d = 1; d < g; ++d) pd.p[pd.n++] = static_cast<uint16_t*>(outs[(r + d) % g]);
      if (pd.n > 0) {
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        nsplit_peer_store_kernel<<<(unsigned)(2 * sms), 512, 0, st>>>(static_cast<const uint16_t*>(outs[r]), pd, m,
                                                                      n_total, lo, nl);
        if (h3q_status s = cuda_status(cudaGetLastError(), what)) return s;
      }
    }
    return h3q_comm_barrier(c, stream);
  }
  if (mode == H3Q_NSPLIT_FUSED) {
    if (nl > 0) {
      ga.M = m;
      ga.N = nl;
      ga.xs = xs;
      ga.out = outs[0];
      if (h3q_status s = cuda_status(h3q::launch_gemm_i8_allgather(a, w_local, ga, outs, g, n_total, lo, st), what))
        return s;
    }
    return h3q_comm_barrier(c, stream);
  }

  // PUSH: row chunks of whole 256-row GEMM tiles; while the GEMM computes chunk j+1, the copy streams (one per peer,
  // so the peers' copies run on separate copy engines at once) forward chunk j
  if (nl > 0) {
    if (g - 1 > kMaxPeers) return fail(H3Q_ERR_UNSUPPORTED, "%s: the push form serves at most %d peers", what, kMaxPeers);
    const int64_t tile_rows = (m + 255) / 256;
    const int nch = (int)(tile_rows < kPushChunks ? tile_rows : kPushChunks);
    cudaError_t e = cudaEventRecord(c->ev[kPushChunks], st);
    for (int d = 1; d < g && e == cudaSuccess; ++d) e = cudaStreamWaitEvent(c->copy[d - 1], c->ev[kPushChunks], 0);
    uint16_t* own = static_cast<uint16_t*>(outs[r]);
    for (int j = 0; j < nch && e == cudaSuccess; ++j) {
      const int64_t r0 = tile_rows * j / nch * 256, r1 = tile_rows * (j + 1) / nch * 256;
      const int64_t rows = (r1 < m ? r1 : m) - r0;
      if (rows <= 0) continue;
      ga.M = rows;
      ga.N = nl;
      ga.xs = xs + r0;
      ga.out = own + r0 * n_total;
      void* dst[1] = {own + r0 * n_total};
      e = h3q::launch_gemm_i8_allgather(a + r0 * k, w_local, ga, dst, 1, n_total, lo, st);
      if (e == cudaSuccess) e = cudaEventRecord(c->ev[j], st);
      for (int d = 1; d < g && e == cudaSuccess; ++d) {
        const int p = (r + d) % g;  // peers in a rotating order, so no destination is everyone's first
        cudaStream_t cs = c->copy[d - 1];
        e = cudaStreamWaitEvent(cs, c->ev[j], 0);
        uint16_t* dstp = static_cast<uint16_t*>(outs[p]) + r0 * n_total + lo;
        if (e == cudaSuccess)
          e = cudaMemcpy2DAsync(dstp, (size_t)n_total * 2, own + r0 * n_total + lo, (size_t)n_total * 2,
                                (size_t)nl * 2, (size_t)rows, cudaMemcpyDeviceToDevice, cs);
      }
    }
    for (int d = 1; d < g && e == cudaSuccess; ++d) {
      e = cudaEventRecord(c->done[d - 1], c->copy[d - 1]);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(st, c->done[d - 1], 0);
    }
    if (h3q_status s = cuda_status(e, what)) return s;
  }
  return h3q_comm_barrier(c, stream);
}

}  // extern "C"
