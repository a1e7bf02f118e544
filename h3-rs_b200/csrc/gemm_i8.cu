// gemm_i8.cu -- W8A8 int8 GEMM on the 5th-generation tensor cores (tcgen05 kind::i8) with a fused epilogue.
//
// Computes acc[m,n] = sum_k A[m,k] * B[n,k] (A = quantized activations [M,K], B = int8 weight [N,K], both
// K-major) and applies the epilogue of the reference's fused GEMM gemm_s8 (attn8.rs:258-344) or of its
// cuBLASLt path (kernels.rs:955-1070 + int8_epilogue / int8_epilogue_swiglu, kernels.rs:333-373):
//   v = fmaf((float)acc * xs[m], ws[n], bias[n])      (the reference's `acc * x * w + b`, fmad-contracted)
//
// Structure (one persistent CTA per SM, 192 threads):
//   warp 0     one elected lane issues TMA tile loads (128-byte swizzle) into a STAGES-deep smem ring;
//   warp 1     allocates 512 TMEM columns; one elected lane issues tcgen05.mma (M=128, N=256, K=32) into a
//              double-buffered int32 accumulator (2 x 256 columns) and commits stage / accumulator barriers;
//   warps 2-5  epilogue: tcgen05.ld 32 lanes x 32 columns, scale / bias / activation, vector stores.
// Every barrier wait is bounded (ptx.cuh): on time-out the CTA records an error code, drains its own TMA
// loads, frees TMEM and returns.
#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "h3q_internal.h"
#include "gemm_common.cuh"

namespace h3q {

namespace {
constexpr int BK = 128;                       // K bytes per pipeline stage (one 128-byte swizzle row)
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;           // two 256-column int32 accumulators
}  // namespace

// Compile-time shape of the two kernel variants.  PAIR: a CTA pair (cluster of 2) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2, each CTA loading 128 rows of A and 128 rows of B; single: one CTA computes 128 x 256.
template <bool PAIR>
struct GemmCfg {
  static constexpr int kStages = PAIR ? 6 : 4;
  static constexpr int kBRows = PAIR ? 128 : 256;   // B rows held by one CTA
  static constexpr int kAStage = 128 * BK;          // 16 KiB
  static constexpr int kBStage = kBRows * BK;
  static constexpr int kStageBytes = kAStage + kBStage;
  static constexpr int kTileM = PAIR ? 256 : 128;   // output rows per tile
  static constexpr uint32_t kTxBytes = PAIR ? 2 * kStageBytes : kStageBytes;  // bytes landing per stage
  static constexpr uint32_t kIdesc = idesc_i8(PAIR ? 256 : 128, 256);
  static constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + EPI_SMEM + 256;
};

// candle's tanh GELU, 0.5 y (1 + tanh(z)) with z = sqrt(2/pi) (y + 0.044715 y^3), in its logistic form: since
// 1 + tanh(z) = 2 / (1 + e^(-2z)), it equals y / (1 + e^(-2z)), one exponential and one approximate reciprocal
// instead of a tanh.  Large negative y: e^(-2z) overflows, the reciprocal is 0 and the result -0, as the limit.
__device__ __forceinline__ float gelu_tanh(float y) {
  const float m2c = -2.f * 0.7978845608028654f;  // -2 sqrt(2/pi)
  const float z2 = m2c * __fmaf_rn(0.044715f * y, y * y, y);
  return __fdividef(y, 1.f + __expf(z2));
}

// Epilogue of one accumulator tile for the 32 output rows of this warp (TMEM lanes 32q..32q+31 of `tacc`).
// `row` is this lane's output row, `row0` the warp's first row, `nb` the tile column.
template <int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& p, EpiWarp& ew, uint32_t tacc, int64_t row,
                                              int64_t row0, int nb, bool kzero, bool ws_al, bool b_al) {
  const bool rv = row < p.M;
  const bool wv = row0 < p.M;  // any row of this warp's box inside the output
  const float xs = (EPI != kEpiAccI32 && rv) ? __ldg(p.xs + row) : 0.f;
  const float ws0 = (EPI == kEpiAccI32 || p.ws_per_row) ? 0.f : __ldg(p.ws);
  if (EPI == kEpiSwigluHalves) {
    const int64_t F = p.N / 2;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t rg[32], ru[32];
      __syncwarp();
      tmem_ld_32x32b_x32(tacc + 32 * c, rg);
      tmem_ld_32x32b_x32(tacc + 128 + 32 * c, ru);
      tmem_wait_ld();
      const int64_t j0 = (int64_t)nb * 128 + 32 * c;
      const int valid = clamp32(F - j0);
      float wg[32], wu[32], bg[32], bu[32];
      if (p.ws_per_row) {
        load_vec32(p.ws, j0, valid, ws_al, wg);
        load_vec32(p.ws, F + j0, valid, ws_al && (F % 4 == 0), wu);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) wg[i] = wu[i] = ws0;
      }
      if (p.bias) {
        load_vec32(p.bias, j0, valid, b_al, bg);
        load_vec32(p.bias, F + j0, valid, b_al && (F % 4 == 0), bu);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) bg[i] = bu[i] = 0.f;
      }
      float o[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float ag = kzero ? 0.f : (float)(int)rg[i], au = kzero ? 0.f : (float)(int)ru[i];
        float g = __fmaf_rn(__fmul_rn(ag, xs), wg[i], bg[i]);
        float u = __fmaf_rn(__fmul_rn(au, xs), wu[i], bu[i]);
        if (p.out_kind == 2) g = bf16r(g);
        float s = __fdiv_rn(g, __fadd_rn(1.f, __expf(-g)));
        if (p.out_kind == 2) { s = bf16r(s); u = bf16r(u); }
        o[i] = __fmul_rn(s, u);
      }
      uint32_t w[32];
      const int W = pack_out(o, p.out_kind, w);
      ew.store(w, W, (int32_t)j0, (int32_t)row0, wv && valid > 0);
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    uint32_t r[32];
    __syncwarp();
    tmem_ld_32x32b_x32(tacc + 32 * c, r);
    tmem_wait_ld();
    if (kzero) {
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = 0u;
    }
    const int64_t col0 = (int64_t)nb * 256 + 32 * c;
    const int valid = clamp32(p.N - col0);
    const bool st = wv && valid > 0;
    if (EPI == kEpiAccI32) {
      ew.store(r, 128, (int32_t)col0, (int32_t)row0, st);
      continue;
    }
    float w[32], b[32];
    if (p.ws_per_row) load_vec32(p.ws, col0, valid, ws_al, w);
    else {
#pragma unroll
      for (int i = 0; i < 32; ++i) w[i] = ws0;
    }
    if (p.bias) load_vec32(p.bias, col0, valid, b_al, b);
    else {
#pragma unroll
      for (int i = 0; i < 32; ++i) b[i] = 0.f;
    }
    // v = fma(acc * xs, ws, bias) two columns per instruction (paired f32 multiply and fma: each lane rounds
    // exactly as the scalar instruction, so the bits are the reference's `acc * x * w + b`)
    float v[32];
    const f2 xs2 = pk(xs, xs);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const f2 t = mul2(pk((float)(int)r[2 * i], (float)(int)r[2 * i + 1]), xs2);
      upk(fma2(t, pk(w[2 * i], w[2 * i + 1]), pk(b[2 * i], b[2 * i + 1])), v[2 * i], v[2 * i + 1]);
    }
    uint32_t o[32];
    if (EPI == kEpiSwigluPairs) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float h[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float gt = bf16r(v[4 * i + 2 * k]), up = bf16r(v[4 * i + 2 * k + 1]);
          const float sg = bf16r(__fdiv_rn(gt, __fadd_rn(1.f, __expf(-gt))));
          h[k] = __fmul_rn(sg, up);
        }
        o[i] = pack_bf2(h[0], h[1]);
      }
      ew.store(o, 32, (int32_t)(col0 / 2), (int32_t)row0, st);
    } else if (EPI == kEpiGelu) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(bf16r(v[i]));
      ew.store(o, pack_out(v, 2, o), (int32_t)col0, (int32_t)row0, st);
    } else if (EPI == kEpiGateResid) {
      float g[32];
      uint16_t rr[32];
      if (rv) {
        const uint32_t gi = p.gate_idx ? __ldg(p.gate_idx + row) : 0u;
        load_vec32(p.gate + (int64_t)gi * p.N, col0, valid, false, g);
        const uint16_t* rs = p.resid + row * p.N + col0;
        if (valid == 32) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<uint4*>(rr + 8 * i) = __ldg(reinterpret_cast<const uint4*>(rs) + i);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) rr[i] = i < valid ? rs[i] : (uint16_t)0;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) { g[i] = 0.f; rr[i] = 0; }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __fmaf_rn(bf16r(v[i]), bf16r(g[i]), bf2f(rr[i]));
      ew.store(o, pack_out(v, 2, o), (int32_t)col0, (int32_t)row0, st);
    } else {
      ew.store(o, pack_out(v, p.out_kind, o), (int32_t)col0, (int32_t)row0, st);
    }
  }
}

template <int EPI, bool PAIR, int NDST>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ OutMaps<NDST> tmO, const GemmArgs p, int num_m, int num_n, int nk,
                   int group_m) {
  using C = GemmCfg<PAIR>;
  extern __shared__ uint8_t smem_raw[];
  // align by offsetting the __shared__ array itself, so the compiler keeps shared-space (LDS/STS) accesses
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::kStages * C::kAStage;
  uint8_t* sE = sB + C::kStages * C::kBStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + EPI_SMEM);
  uint64_t* empty = full + C::kStages;
  uint64_t* accf = empty + C::kStages;
  uint64_t* acce = accf + 2;
  uint64_t* mma_done = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], PAIR ? 8 : 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0 && nk > 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int d = 0; d < (NDST == 1 ? 1 : tmO.n); ++d) tma_prefetch_desc(&tmO.m[d]);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (PAIR) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = num_m * num_n;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const bool halves = (EPI == kEpiSwigluHalves);
  const int64_t F = p.N / 2;

  if (warp == 0) {
    if (elect_one()) {
      // ------------------------------------------------------------------ TMA producer (both CTAs of a pair)
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_par = 0;
      for (int t = unit; t < num_tiles; t += units) {
        int mb, nb;
        tile_coords(t, num_m, num_n, group_m, mb, nb);
        const int32_t arow = mb * C::kTileM + (int32_t)rank * 128;
        int32_t b0, b1;
        if (PAIR) {
          b0 = halves ? (rank == 0 ? nb * 128 : (int32_t)(F + nb * 128)) : nb * 256 + (int32_t)rank * 128;
          b1 = b0;
        } else {
          b0 = halves ? nb * 128 : nb * 256;
          b1 = halves ? (int32_t)(F + nb * 128) : nb * 256 + 128;
        }
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&full[stage], C::kTxBytes);
          uint8_t* a_dst = sA + stage * C::kAStage;
          uint8_t* b_dst = sB + stage * C::kBStage;
          if (PAIR) {
            const uint32_t fb = mapa_shared(&full[stage], 0);
            tma_load_2d_pair(a_dst, &tmA, fb, kb * BK, arow);
            tma_load_2d_pair(b_dst, &tmB, fb, kb * BK, b0);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * BK, arow);
            tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, b0);
            tma_load_2d(b_dst + C::kBStage / 2, &tmB, &full[stage], kb * BK, b1);
          }
          issued_mask |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      // drain: the loads of every stage must land before the pair may exit (the leader's barriers count both
      // CTAs' bytes, so the leader's drain covers the peer's loads too; the final cluster barrier holds the peer)
      if (leader)
        for (int s = 0; s < C::kStages; ++s)
          if (issued_mask & (1u << s)) mbar_drain(&full[s], (issued_par >> s) & 1u, p.err, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      // ------------------------------------------------------------------ MMA issuer (pair leader only)
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = unit; t < num_tiles; t += units, ++it) {
        const int acc = it & 1;
        const uint32_t accph = (it >> 1) & 1;
        if (!mbar_wait_bounded(&acce[acc], accph ^ 1, abort_flag, p.err, kDevTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * 256;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, p.err, kDevTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = smem_desc_k128(smem_u32(sA + stage * C::kAStage));
          const uint64_t db = smem_desc_k128(smem_u32(sB + stage * C::kBStage));
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            if (PAIR) mma_i8_pair(d, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), C::kIdesc, (kb | k) != 0);
            else mma_i8(d, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), C::kIdesc, (kb | k) != 0);
          }
          if (PAIR) {
            mma_commit_pair(mapa_shared(&empty[stage], 0));
            mma_commit_pair(mapa_shared(&empty[stage], 1));
          } else {
            mma_commit(&empty[stage]);
          }
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (PAIR) {
          mma_commit_pair(mapa_shared(&accf[acc], 0));
          mma_commit_pair(mapa_shared(&accf[acc], 1));
        } else {
          mma_commit(&accf[acc]);
        }
      }
      // every MMA this thread issued must complete before TMEM is released
      if (PAIR) mma_commit_pair(mapa_shared(mma_done, 0));
      else mma_commit(mma_done);
      mbar_drain(mma_done, 0, p.err, kDevTimeoutDrain);
    }
  } else {
    // -------------------------------------------------------------------- epilogue warps 2..5 (both CTAs)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool ws_al = (reinterpret_cast<uintptr_t>(p.ws) & 15) == 0;
    const bool b_al = p.bias && (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0;
    EpiWarp ew{tmO.m, NDST == 1 ? 1 : tmO.n, sE + (warp - 2) * 2 * EPI_BUF, 0, lane};
    int it = 0;
    for (int t = unit; t < num_tiles; t += units, ++it) {
      const int acc = it & 1;
      const uint32_t accph = (it >> 1) & 1;
      int mb, nb;
      tile_coords(t, num_m, num_n, group_m, mb, nb);
      const bool ready = mbar_wait_bounded(&accf[acc], accph, abort_flag, p.err, kDevTimeoutAccFull);
      if (!__all_sync(0xffffffffu, ready)) break;  // the warp's TMEM loads need all 32 lanes
      tc_fence_after();
      const int64_t row0 = (int64_t)mb * C::kTileM + (int64_t)rank * 128 + 32 * q;
      const uint32_t tacc = tmem_base + ((uint32_t)(32 * q) << 16) + acc * 256;
      epilogue_tile<EPI>(p, ew, tacc, row0 + lane, row0, nb, nk == 0, ws_al, b_al);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_cluster(mapa_shared(&acce[acc], 0));
        else mbar_arrive(&acce[acc]);
      }
    }
    if (lane == 0) bulk_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  if (PAIR) cluster_sync(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------- host side

int sm_count(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (!cache[device]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    cache[device] = v > 0 ? v : 148;
  }
  return cache[device];
}

template <int EPI, bool PAIR, int NDST = 1>
static cudaError_t launch_epi(const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps<NDST>& to,
                              const GemmArgs& a, int num_m, int num_n, int nk, int group_m, cudaStream_t st) {
  using C = GemmCfg<PAIR>;
  auto kern = gemm_i8_kernel<EPI, PAIR, NDST>;
  static int grid_cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  if (PAIR) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!grid_cache[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
    if (e != cudaSuccess) return e;
    int units = sm_count(dev);
    if (PAIR) {
      // size the persistent grid by the clusters that can be co-resident, so no pair waits for another to finish
      int clusters = 0;
      cfg.gridDim = dim3(2 * (sm_count(dev) / 2), 1, 1);
      e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
      if (e != cudaSuccess) return e;
      units = clusters > 0 ? clusters : 1;
    }
    grid_cache[dev] = units;
  }
  const int64_t tiles = (int64_t)num_m * num_n;
  const int units = (int)(tiles < grid_cache[dev] ? tiles : grid_cache[dev]);
  cfg.gridDim = dim3(PAIR ? 2 * units : units, 1, 1);
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, to, a, num_m, num_n, nk, group_m);
}

// Row-chunk width (bytes) of the staged output and the output element size, by epilogue.
static void out_geometry(const GemmArgs& a, int& es, int& W, int64_t& nout) {
  const int kes = a.out_kind == 0 ? 4 : 2;
  switch (a.epi) {
    case kEpiSwigluPairs: es = 2; W = 32; nout = a.N / 2; break;
    case kEpiSwigluHalves: es = kes; W = 32 * kes; nout = a.N / 2; break;
    case kEpiGelu:
    case kEpiGateResid: es = 2; W = 64; nout = a.N; break;
    case kEpiAccI32: es = 4; W = 128; nout = a.N; break;
    default: es = kes; W = 32 * kes; nout = a.N; break;
  }
}

template <bool PAIR>
static cudaError_t launch_variant(const CUtensorMap& ta, const CUtensorMap& tb, const OutMaps<1>& to,
                                  const GemmArgs& a, int num_n, int nk, cudaStream_t st) {
  const int num_m = (int)((a.M + GemmCfg<PAIR>::kTileM - 1) / GemmCfg<PAIR>::kTileM);
  // L2 reuse (measured with ncu DRAM counters at the DiT shapes): a weight of up to ~32 MB stays resident while
  // tile-columns sweep fastest (group_m = 1), so both operands are read from DRAM about once.  A larger weight
  // does not stay resident; instead groups of tile-rows whose activation block is ~24 MB stay in L2 while the
  // weight streams past them (weight re-read num_m / group_m times, activations once).
  // For long K (the DiT's fc2, K = 13824) a ~40 MB activation block measured 2-3% faster than ~24 MB (group of 10-12
  // tile-rows instead of 6: 1.39-1.40 ms against 1.42-1.47 ms for the c1 fc2 at 32760 tokens); at K = 5120 24 MB
  // stays best.
  const double weight_bytes = (double)a.N * (double)a.K;
  int group_m = 1;
  if (weight_bytes > 32e6) {
    const double rows_bytes = (double)GemmCfg<PAIR>::kTileM * (double)(a.K > 0 ? a.K : 1);
    group_m = (int)((a.K > 8192 ? 40e6 : 24e6) / rows_bytes);
    if (group_m < 1) group_m = 1;
    if (group_m > num_m) group_m = num_m;
  }
  switch (a.epi) {
    case kEpiLinear: return launch_epi<kEpiLinear, PAIR>(ta, tb, to, a, num_m, num_n, nk, group_m, st);
    case kEpiSwigluPairs: return launch_epi<kEpiSwigluPairs, PAIR>(ta, tb, to, a, num_m, num_n, nk, group_m, st);
    case kEpiSwigluHalves: return launch_epi<kEpiSwigluHalves, PAIR>(ta, tb, to, a, num_m, num_n, nk, group_m, st);
    case kEpiGelu: return launch_epi<kEpiGelu, PAIR>(ta, tb, to, a, num_m, num_n, nk, group_m, st);
    case kEpiGateResid: return launch_epi<kEpiGateResid, PAIR>(ta, tb, to, a, num_m, num_n, nk, group_m, st);
    case kEpiAccI32: return launch_epi<kEpiAccI32, PAIR>(ta, tb, to, a, num_m, num_n, nk, group_m, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm_i8(const int8_t* A, const int8_t* B, const GemmArgs& a, cudaStream_t st) {
  if (a.M == 0) return cudaSuccess;
  const bool halves = a.epi == kEpiSwigluHalves;
  const int64_t ncols_tiles = halves ? (a.N / 2 + 127) / 128 : (a.N + 255) / 256;
  if (ncols_tiles == 0) return cudaSuccess;
  int es, W;
  int64_t nout;
  out_geometry(a, es, W, nout);
  CUtensorMap ta, tb;
  OutMaps<1> to;
  to.n = 1;
  if (!make_tmap_out(&to.m[0], a.out, (uint64_t)a.M, (uint64_t)nout, es, W)) return cudaErrorInvalidValue;
  if (a.K > 0) {
    if (!make_tmap_i8(&ta, A, (uint64_t)a.M, (uint64_t)a.K, 128)) return cudaErrorInvalidValue;
    if (!make_tmap_i8(&tb, B, (uint64_t)a.N, (uint64_t)a.K, 128)) return cudaErrorInvalidValue;
  } else {
    // K == 0: no tile is ever loaded (the epilogue sees zero accumulators); the maps only need to be valid
    if (!make_tmap_i8(&ta, a.out, 1, 16, 128)) return cudaErrorInvalidValue;
    tb = ta;
  }
  const int nk = (int)((a.K + BK - 1) / BK);
  // 256-row pair tiles when there are at least two 128-row tiles of work, else one CTA per 128 x 256 tile
  if (a.M > 128) return launch_variant<true>(ta, tb, to, a, (int)ncols_tiles, nk, st);
  return launch_variant<false>(ta, tb, to, a, (int)ncols_tiles, nk, st);
}


// The local weight rows' output columns stored into every destination buffer (the N-split all-gather): outs[d] is
// rank d's [M, n_total] bf16 output; this launch owns columns [n_offset, n_offset + a.N).  Each destination map
// starts at that column block and is a.N columns wide, so the TMA stores clip at the block's edge.
cudaError_t launch_gemm_i8_allgather(const int8_t* A, const int8_t* B, const GemmArgs& a, void* const* outs, int n_out,
                                     int64_t n_total, int64_t n_offset, cudaStream_t st) {
  if (a.M == 0 || a.N == 0) return cudaSuccess;
  if (a.epi != kEpiLinear || a.out_kind != 2 || n_out < 1 || n_out > kMaxGatherRanks || a.K <= 0)
    return cudaErrorInvalidValue;
  OutMaps<kMaxGatherRanks> to;
  to.n = n_out;
  for (int d = 0; d < n_out; ++d) {
    uint16_t* base = static_cast<uint16_t*>(outs[d]) + n_offset;
    if (!make_tmap_out(&to.m[d], base, (uint64_t)a.M, (uint64_t)a.N, 2, 64, (uint64_t)n_total))
      return cudaErrorInvalidValue;
  }
  CUtensorMap ta, tb;
  if (!make_tmap_i8(&ta, A, (uint64_t)a.M, (uint64_t)a.K, 128)) return cudaErrorInvalidValue;
  if (!make_tmap_i8(&tb, B, (uint64_t)a.N, (uint64_t)a.K, 128)) return cudaErrorInvalidValue;
  const int nk = (int)((a.K + BK - 1) / BK);
  const int num_n = (int)((a.N + 255) / 256);
  if (a.M > 128) {
    const int num_m = (int)((a.M + 255) / 256);
    return launch_epi<kEpiLinear, true, kMaxGatherRanks>(ta, tb, to, a, num_m, num_n, nk, 1, st);
  }
  const int num_m = (int)((a.M + 127) / 128);
  return launch_epi<kEpiLinear, false, kMaxGatherRanks>(ta, tb, to, a, num_m, num_n, nk, 1, st);
}

}  // namespace h3q
