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

namespace h3q {

namespace {
constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int A_STAGE = BM * BK;              // 16 KiB
constexpr int B_STAGE = BN * BK;              // 32 KiB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr int GROUP_M = 16;                   // tile-rows swept together across N (L2 reuse of B)
constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
constexpr uint32_t IDESC = idesc_i8(BM, BN);
}  // namespace

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = GROUP_M * num_n;
  const int group = t / per_group;
  const int first_m = group * GROUP_M;
  const int gsz = min(num_m - first_m, GROUP_M);
  const int local = t - group * per_group;
  mb = first_m + local % gsz;
  nb = local / gsz;
}

__device__ __forceinline__ int clamp32(int64_t v) { return v <= 0 ? 0 : (v >= 32 ? 32 : (int)v); }

// 32 consecutive f32 values starting at p[col0] (only `valid` of them exist); broadcast reads.
__device__ __forceinline__ void load_vec32(const float* p, int64_t col0, int valid, bool aligned, float (&o)[32]) {
  if (valid == 32 && aligned) {
    const float4* q = reinterpret_cast<const float4*>(p + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 f = __ldg(q + i);
      o[4 * i] = f.x; o[4 * i + 1] = f.y; o[4 * i + 2] = f.z; o[4 * i + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = i < valid ? __ldg(p + col0 + i) : 0.f;
  }
}

// Store n (<= 32) f32 values to row `dst` in the output kind; vector stores when all 32 fit.
__device__ __forceinline__ void store_row(void* out, int kind, int64_t off, const float (&v)[32], int n, int valid) {
  if (kind == 0) {
    float* d = reinterpret_cast<float*>(out) + off;
    if (valid == n) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        if (i < n) *reinterpret_cast<float4*>(d + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
      for (int i = 0; i < valid; ++i) d[i] = v[i];
    }
    return;
  }
  uint16_t* d = reinterpret_cast<uint16_t*>(out) + off;
  if (valid == n) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      if (i < n) {
        uint4 w;
        if (kind == 2) {
          w.x = pack_bf2(v[i], v[i + 1]); w.y = pack_bf2(v[i + 2], v[i + 3]);
          w.z = pack_bf2(v[i + 4], v[i + 5]); w.w = pack_bf2(v[i + 6], v[i + 7]);
        } else {
          w.x = (uint32_t)f2h(v[i]) | ((uint32_t)f2h(v[i + 1]) << 16);
          w.y = (uint32_t)f2h(v[i + 2]) | ((uint32_t)f2h(v[i + 3]) << 16);
          w.z = (uint32_t)f2h(v[i + 4]) | ((uint32_t)f2h(v[i + 5]) << 16);
          w.w = (uint32_t)f2h(v[i + 6]) | ((uint32_t)f2h(v[i + 7]) << 16);
        }
        *reinterpret_cast<uint4*>(d + i) = w;
      }
    }
  } else {
    for (int i = 0; i < valid; ++i) d[i] = kind == 2 ? (uint16_t)f2bf(v[i]) : f2h(v[i]);
  }
}

__device__ __forceinline__ float gelu_tanh(float y) {
  const float c = 0.7978845608028654f;  // sqrt(2/pi)
  return 0.5f * y * (1.f + tanhf(c * (y + 0.044715f * y * y * y)));
}

// Epilogue of one 128 x 256 accumulator tile; this thread owns tile row `lr` (TMEM lane) = output row `row`.
template <int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& p, uint32_t tacc, int64_t row, int nb, bool kzero,
                                              bool ws_al, bool b_al) {
  const bool rv = row < p.M;
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
      if (rv && valid > 0) store_row(p.out, p.out_kind, row * F + j0, o, 32, valid);
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
    const int64_t col0 = (int64_t)nb * BN + 32 * c;
    const int valid = clamp32(p.N - col0);
    if (EPI == kEpiAccI32) {
      if (rv && valid > 0) {
        int32_t* d = reinterpret_cast<int32_t*>(p.out) + row * p.N + col0;
        if (valid == 32) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<int4*>(d + i) = make_int4((int)r[i], (int)r[i + 1], (int)r[i + 2], (int)r[i + 3]);
        } else {
          for (int i = 0; i < valid; ++i) d[i] = (int)r[i];
        }
      }
    } else {
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
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __fmaf_rn(__fmul_rn((float)(int)r[i], xs), w[i], b[i]);
    if (!rv || valid <= 0) {
    } else if (EPI == kEpiSwigluPairs) {
      float o[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float gt = bf16r(v[2 * i]), up = bf16r(v[2 * i + 1]);
        const float sg = bf16r(__fdiv_rn(gt, __fadd_rn(1.f, __expf(-gt))));
        o[i] = __fmul_rn(sg, up);
      }
#pragma unroll
      for (int i = 16; i < 32; ++i) o[i] = 0.f;
      store_row(p.out, 2, row * (p.N / 2) + col0 / 2, o, 16, valid / 2);
    } else if (EPI == kEpiGelu) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(bf16r(v[i]));
      store_row(p.out, 2, row * p.N + col0, v, 32, valid);
    } else if (EPI == kEpiGateResid) {
      const uint32_t gi = p.gate_idx ? __ldg(p.gate_idx + row) : 0u;
      float g[32];
      load_vec32(p.gate + (int64_t)gi * p.N, col0, valid, false, g);
      const uint16_t* rs = p.resid + row * p.N + col0;
      uint16_t rr[32];
      if (valid == 32) {
#pragma unroll
        for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(rr + 8 * i) = __ldg(reinterpret_cast<const uint4*>(rs) + i);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) rr[i] = i < valid ? rs[i] : (uint16_t)0;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __fmaf_rn(bf16r(v[i]), bf16r(g[i]), bf2f(rr[i]));
      store_row(p.out, 2, row * p.N + col0, v, 32, valid);
    } else {
      store_row(p.out, p.out_kind, row * p.N + col0, v, 32, valid);
    }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs p, int num_m, int num_n, int nk) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* mma_done = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 128);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0 && nk > 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = num_m * num_n;
  const bool halves = (EPI == kEpiSwigluHalves);
  const int64_t F = p.N / 2;

  if (warp == 0) {
    if (elect_one()) {
      // ---------------------------------------------------------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_par = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        const int32_t b0 = halves ? nb * 128 : nb * BN;
        const int32_t b1 = halves ? (int32_t)(F + nb * 128) : nb * BN + 128;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sA + stage * A_STAGE, &tmA, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sB + stage * B_STAGE, &tmB, &full[stage], kb * BK, b0);
          tma_load_2d(sB + stage * B_STAGE + B_STAGE / 2, &tmB, &full[stage], kb * BK, b1);
          issued_mask |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      // drain: every load this thread issued must land before the CTA may exit
      for (int s = 0; s < STAGES; ++s) {
        if (!(issued_mask & (1u << s))) continue;
        int dummy = 0;
        mbar_wait_bounded(&full[s], (issued_par >> s) & 1u, &dummy, p.err, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      // ---------------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t accph = (it >> 1) & 1;
        if (!mbar_wait_bounded(&acce[acc], accph ^ 1, abort_flag, p.err, kDevTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, p.err, kDevTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = smem_desc_k128(smem_u32(sA + stage * A_STAGE));
          const uint64_t db = smem_desc_k128(smem_u32(sB + stage * B_STAGE));
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_i8(d, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), IDESC, (kb | k) != 0);
          mma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&accf[acc]);
      }
      // every MMA this thread issued must complete before TMEM is released
      mma_commit(mma_done);
      int dummy = 0;
      mbar_wait_bounded(mma_done, 0, &dummy, p.err, kDevTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------------ epilogue warps 2..5
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool ws_al = (reinterpret_cast<uintptr_t>(p.ws) & 15) == 0;
    const bool b_al = p.bias && (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t accph = (it >> 1) & 1;
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      if (!mbar_wait_bounded(&accf[acc], accph, abort_flag, p.err, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const int64_t row = (int64_t)mb * BM + 32 * q + lane;
      const uint32_t tacc = tmem_base + ((uint32_t)(32 * q) << 16) + acc * BN;
      epilogue_tile<EPI>(p, tacc, row, nb, nk == 0, ws_al, b_al);
      tc_fence_before();
      mbar_arrive(&acce[acc]);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------- host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// int8 [rows, cols] row-major, box = 128 bytes of K x box_rows rows, 128-byte swizzle, zero fill outside.
static bool make_tmap_i8(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {BK, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

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

template <int EPI>
static cudaError_t launch_epi(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int num_m, int num_n,
                              int nk, int grid, cudaStream_t st) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_i8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  gemm_i8_kernel<EPI><<<grid, THREADS, SMEM_BYTES, st>>>(ta, tb, a, num_m, num_n, nk);
  return cudaGetLastError();
}

cudaError_t launch_gemm_i8(const int8_t* A, const int8_t* B, const GemmArgs& a, cudaStream_t st) {
  if (a.M == 0) return cudaSuccess;
  const bool halves = a.epi == kEpiSwigluHalves;
  const int64_t ncols_tiles = halves ? (a.N / 2 + 127) / 128 : (a.N + BN - 1) / BN;
  if (ncols_tiles == 0) return cudaSuccess;
  CUtensorMap ta, tb;
  if (a.K > 0) {
    if (!make_tmap_i8(&ta, A, (uint64_t)a.M, (uint64_t)a.K, BM)) return cudaErrorInvalidValue;
    if (!make_tmap_i8(&tb, B, (uint64_t)a.N, (uint64_t)a.K, 128)) return cudaErrorInvalidValue;
  } else {
    // K == 0: no tile is ever loaded (the epilogue sees zero accumulators); the maps only need to be valid
    if (!make_tmap_i8(&ta, a.out, 1, 16, BM)) return cudaErrorInvalidValue;
    tb = ta;
  }
  const int num_m = (int)((a.M + BM - 1) / BM);
  const int num_n = (int)ncols_tiles;
  const int nk = (int)((a.K + BK - 1) / BK);
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t tiles = (int64_t)num_m * num_n;
  const int grid = (int)(tiles < sm_count(dev) ? tiles : sm_count(dev));
  switch (a.epi) {
    case kEpiLinear: return launch_epi<kEpiLinear>(ta, tb, a, num_m, num_n, nk, grid, st);
    case kEpiSwigluPairs: return launch_epi<kEpiSwigluPairs>(ta, tb, a, num_m, num_n, nk, grid, st);
    case kEpiSwigluHalves: return launch_epi<kEpiSwigluHalves>(ta, tb, a, num_m, num_n, nk, grid, st);
    case kEpiGelu: return launch_epi<kEpiGelu>(ta, tb, a, num_m, num_n, nk, grid, st);
    case kEpiGateResid: return launch_epi<kEpiGateResid>(ta, tb, a, num_m, num_n, nk, grid, st);
    case kEpiAccI32: return launch_epi<kEpiAccI32>(ta, tb, a, num_m, num_n, nk, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace h3q
