// nvfp4_gemm.cu -- the NVFP4 (+AWQ) linear of h3-rs's text encoder, fused: fp4 weights are decoded to bf16
// inside the GEMM and multiplied on the 5th-generation tensor cores (tcgen05 kind::f16, f32 accumulators).
//
// Reference (weights.rs:612-635 with dequant_nvfp4, kernels.rs:65-81):
//   x2 = bf16(x * bf16(pre_quant_scale))                    (AWQ, weights.rs:617-620)
//   W  = bf16(E2M1[nibble] * e4m3(block scale) * global)    (even column = high nibble, 128x4 swizzled scales)
//   y  = bf16(x2 @ W^T)  (+ bf16(bias), added in bf16)      (weights.rs:632-635)
// The reference materialises W in HBM (2 bytes per weight) for every call and runs a bf16 cuBLAS GEMM.  Here the
// packed weight (0.56 bytes per weight with its scales) is read once per tile and decoded in shared memory.
//
// One 2-CTA cluster computes a 256 x 256 output tile (tcgen05.mma.cta_group::2, M=256, N=256, K=16).  Per CTA:
//   warp 0      TMA: bf16 activation tile (128 rows x 64, 128-byte swizzle), packed weight tile (128 rows x
//               32 bytes) and the 512-byte block-scale atom of those 128 rows x 4 blocks, into a 5-stage ring;
//   warp 1      TMEM allocation; in the leader CTA, one thread issues the pair MMAs;
//   warps 2-5   epilogue (TMEM -> bf16 or f32 split-K partials -> TMA store);
//   warps 6-13  decoders: 256 threads, each turning half of one weight row (32 of the stage's 64 codes) into
//               bf16, written straight into the 128-byte-swizzled K-major layout the MMA reads; each decoder
//               warp then signals the leader's stage barrier itself (16 arrivals per stage), with no barrier
//               among the decoders.  Decode per pair of codes: cvt e2m1x2 -> f16x2, f16x2 multiply by the e4m3
//               scale (exact: at most 5 significant bits), widen to f32, multiply by the global scale, round to
//               bf16 -- the same rounding as the reference's dequant.
// Scheduling: when the 256 x 256 tiles fill the co-resident pairs in whole waves (>= 85%), pair p takes tiles p,
// p + P, ...  Otherwise (the text encoder's 40-tile down-proj on 74 pairs) the work is stream-K: the tiles' k-blocks
// in tile order, W = tiles x nk of them, are cut into P equal contiguous ranges, one per pair.  A pair's range is a
// run of segments: whole tiles, which it writes itself, and at most two partial ones (its first and last), which it
// writes as f32 to its two workspace slots; a fix-up kernel adds a split tile's slots in pair order (a fixed
// order) and writes it.  Every pair then does the same number of k-blocks, with no tail wave.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include "../../include/h3q.h"
#include "ptx.cuh"
#include "h3q_internal.h"
#include "gemm_common.cuh"

namespace h3q {
void set_last_error(const char* msg);

namespace {
constexpr int NF_STAGES = 5;
constexpr int NF_THREADS = 448;  // 14 warps: TMA, MMA, 4 epilogue, 8 decoders
constexpr int NF_A = 128 * 128;   // bf16 activation tile: 128 rows x 64 elements
constexpr int NF_BD = 128 * 128;  // decoded bf16 weight tile
constexpr int NF_BR = 128 * 32;   // packed fp4 weight tile: 128 rows x 64 codes
constexpr int NF_SC = 512;        // one 128-row x 4-block scale atom
constexpr uint32_t NF_TX = NF_A + NF_BR + NF_SC;
// the epilogue staging buffers must start on a 1024-byte boundary (the 128-byte swizzle atom of the f32 stores)
constexpr size_t NF_SC_REGION = ((size_t)NF_STAGES * NF_SC + 1023) / 1024 * 1024;
constexpr size_t NF_SMEM = 1024 + (size_t)NF_STAGES * (NF_A + NF_BD + NF_BR) + NF_SC_REGION + EPI_SMEM + 512;
constexpr uint32_t NF_IDESC = idesc_bf16(256, 256);
}  // namespace

struct Nvfp4Args {
  int64_t M, N, K;
  const uint8_t* bscale;  // swizzled e4m3 block scales
  const float* gscale;    // device scalar
  const float* bias;      // f32 [N] or null (added by whoever writes the finished tile)
  int streamk;            // 0: whole tiles round-robin over the pairs; 1: stream-K ranges of k-blocks
  int* err;
};

// four bytes of packed e2m1 pairs -> four f16x2 (per byte: low nibble -> low half, high nibble -> high half)
__device__ __forceinline__ void cvt_e2m1x8_f16x2(uint32_t w, uint32_t (&d)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(w));
}
__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint16_t two_bytes) {
  uint32_t d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(two_bytes));
  return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// bf16x2 word with `lo` in the low half (RNE, like f2bf for finite values)
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// Decode 8 packed bytes (16 codes of one 16-element block, even code in each byte's high nibble) with scale
// `sc2` (f16x2 of the block's e4m3 scale) and global scale g into 8 bf16x2 words in column order.
__device__ __forceinline__ void decode_block(uint32_t w0, uint32_t w1, uint32_t sc2, float g, uint32_t (&o)[8]) {
  const uint32_t w[2] = {w0, w1};
#pragma unroll
  for (int wi = 0; wi < 2; ++wi) {
    uint32_t d[4];
    cvt_e2m1x8_f16x2(w[wi], d);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t h = hmul2(d[b], sc2);  // exact: at most 5 significant bits, inside the f16 range
      const float odd = __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));   // low nibble
      const float even = __half2float(__ushort_as_half((unsigned short)(h >> 16)));     // high nibble
      float e2, o2;  // both products with the global scale in one paired multiply (each lane rounded as FMUL)
      upk(mul2(pk(even, odd), pk(g, g)), e2, o2);
      o[4 * wi + b] = cvt_bf16x2(e2, o2);
    }
  }
}

// One piece of a pair's work: k-blocks [a, b) of tile (mb, nb).  slot >= 0: a partial tile, written as f32 to
// workspace slot `slot` (2 p for the pair's first segment, 2 p + 1 for its last); slot < 0: a whole tile.
struct Seg {
  int mb, nb, a, b, slot;
};

// The segments of pair `pair` of `pairs`, in order (every role of the pair walks the same sequence).  `cur` starts at
// seg_begin(); next() fills `sg` and returns false past the last segment.
struct SegWalk {
  int64_t cur, end;
  int pair, pairs, num_m, num_n, nk, streamk;
  __device__ __forceinline__ SegWalk(int pair_, int pairs_, int num_m_, int num_n_, int nk_, int streamk_)
      : pair(pair_), pairs(pairs_), num_m(num_m_), num_n(num_n_), nk(nk_), streamk(streamk_) {
    const int64_t tiles = (int64_t)num_m * num_n;
    if (streamk) {
      const int64_t w = tiles * nk;
      cur = w * pair / pairs;
      end = w * (pair + 1) / pairs;
    } else {
      cur = pair;
      end = tiles;
    }
  }
  __device__ __forceinline__ bool next(Seg& sg) {
    if (cur >= end) return false;
    int tile;
    if (streamk) {
      const bool first = cur == (int64_t)((int64_t)num_m * num_n * nk) * pair / pairs;
      tile = (int)(cur / nk);
      sg.a = (int)(cur % nk);
      const int64_t left = end - cur;
      sg.b = left < nk - sg.a ? sg.a + (int)left : nk;
      cur += sg.b - sg.a;
      sg.slot = (sg.a == 0 && sg.b == nk) ? -1 : 2 * pair + (first ? 0 : 1);
    } else {
      tile = (int)cur;
      sg.a = 0;
      sg.b = nk;
      sg.slot = -1;
      cur += pairs;
    }
    tile_coords(tile, num_m, num_n, num_m, sg.mb, sg.nb);  // both tile-rows of an output column together
    return true;
  }
};

__global__ void __launch_bounds__(NF_THREADS, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmP,
                      const Nvfp4Args p, int num_m, int num_n, int nk) {
  extern __shared__ uint8_t smem_raw[];
  // align by offsetting the __shared__ array itself, so the compiler keeps shared-space (LDS/STS) accesses
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sBD = sA + NF_STAGES * NF_A;
  uint8_t* sBR = sBD + NF_STAGES * NF_BD;
  uint8_t* sSC = sBR + NF_STAGES * NF_BR;
  uint8_t* sE = sSC + NF_SC_REGION;
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + EPI_SMEM);
  uint64_t* decd = full + NF_STAGES;
  uint64_t* empty = decd + NF_STAGES;
  uint64_t* accf = empty + NF_STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* mma_done = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NF_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&decd[s], 16);  // every decoder warp of both CTAs
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 8);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int pair = (int)(blockIdx.x >> 1), pairs = (int)(gridDim.x >> 1);
  const int64_t ncb = (p.K / 16 + 3) / 4;  // scale atoms per 128-row group

  if (warp == 0) {
    if (elect_one()) {
      // ---------------------------------------------------------------- TMA producer (each CTA, own stages)
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_par = 0;
      SegWalk walk(pair, pairs, num_m, num_n, nk, p.streamk);
      Seg sg;
      while (walk.next(sg)) {
        const int32_t arow = sg.mb * 256 + (int32_t)rank * 128;
        const int32_t brow = sg.nb * 256 + (int32_t)rank * 128;
        bool ok = true;
        for (int kb = sg.a; kb < sg.b; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) { ok = false; break; }
          // weight rows past N (the second half of a last 256-wide tile): the codes arrive as zeros from the TMA's
          // out-of-bounds fill and no scale atom exists to copy; those accumulator columns are never stored
          const bool brows = brow < p.N;
          mbar_arrive_expect_tx(&full[stage], brows ? NF_TX : NF_TX - NF_SC);
          tma_load_2d(sA + stage * NF_A, &tmA, &full[stage], kb * 64, arow);
          tma_load_2d(sBR + stage * NF_BR, &tmB, &full[stage], kb * 32, brow);
          if (brows)
            bulk_load_1d(sSC + stage * NF_SC, p.bscale + ((int64_t)(brow / 128) * ncb + kb) * 512, NF_SC, &full[stage]);
          issued_mask |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (++stage == NF_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      for (int s = 0; s < NF_STAGES; ++s)
        if (issued_mask & (1u << s)) mbar_drain(&full[s], (issued_par >> s) & 1u, p.err, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      // ---------------------------------------------------------------- MMA issuer (pair leader)
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      SegWalk walk(pair, pairs, num_m, num_n, nk, p.streamk);
      Seg sg;
      for (; walk.next(sg); ++it) {
        const int acc = it & 1;
        const uint32_t accph = (it >> 1) & 1;
        if (!mbar_wait_bounded(&acce[acc], accph ^ 1, abort_flag, p.err, kDevTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * 256;
        bool ok = true;
        for (int kb = sg.a; kb < sg.b; ++kb) {
          // both CTAs' decoders have finished this stage: their activation and weight tiles are in place
          if (!mbar_wait_bounded(&decd[stage], phase, abort_flag, p.err, kDevTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = smem_desc_k128(smem_u32(sA + stage * NF_A));
          const uint64_t db = smem_desc_k128(smem_u32(sBD + stage * NF_BD));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16_pair(d, da + (uint64_t)(k * 2), db + (uint64_t)(k * 2), NF_IDESC, (kb > sg.a) || (k > 0));
          mma_commit_pair(mapa_shared(&empty[stage], 0));
          mma_commit_pair(mapa_shared(&empty[stage], 1));
          if (++stage == NF_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit_pair(mapa_shared(&accf[acc], 0));
        mma_commit_pair(mapa_shared(&accf[acc], 1));
      }
      mma_commit_pair(mapa_shared(mma_done, 0));
      mbar_drain(mma_done, 0, p.err, kDevTimeoutDrain);
    }
  } else if (warp >= 6) {
    // ------------------------------------------------------------------ decoders (both CTAs)
    const int d = threadIdx.x - 192;
    const int r = d & 127, h = d >> 7;  // weight row of the CTA's 128-row half; which 32 of its 64 codes
    const float g = __ldg(p.gscale);
    const uint32_t decd_leader0 = mapa_shared(&decd[0], 0);
    int stage = 0;
    uint32_t phase = 0;
    SegWalk walk(pair, pairs, num_m, num_n, nk, p.streamk);
    Seg sg;
    while (walk.next(sg)) {
      bool ok = true;
      for (int kb = sg.a; kb < sg.b; ++kb) {
        const bool landed = mbar_wait_bounded(&full[stage], phase, abort_flag, p.err, kDevTimeoutFull);
        if (!__all_sync(0xffffffffu, landed)) { ok = false; break; }
        const uint4 qv = *reinterpret_cast<const uint4*>(sBR + stage * NF_BR + r * 32 + 16 * h);
        const uint32_t sc2b =
            *reinterpret_cast<const uint16_t*>(sSC + stage * NF_SC + (r % 32) * 16 + (r / 32) * 4 + 2 * h);
        uint8_t* bd = sBD + stage * NF_BD + r * 128;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int blk = 2 * h + j;  // 16-code block of the row (4 per stage)
          const uint32_t sb = (sc2b >> (8 * j)) & 0xffu;
          const uint32_t sc2 = cvt_e4m3x2_f16x2((uint16_t)(sb | (sb << 8)));
          uint32_t o[8];
          decode_block(j ? qv.z : qv.x, j ? qv.w : qv.y, sc2, g, o);
          // 16 bf16 = chunks 2*blk and 2*blk+1 of the 128-byte row, 128-byte swizzle
          *reinterpret_cast<uint4*>(bd + (((2 * blk) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(bd + (((2 * blk + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {  // this warp's rows are in place: one arrival per decoder warp on the leader's barrier
          if (leader) mbar_arrive(&decd[stage]);
          else mbar_arrive_remote_own_data(decd_leader0 + (uint32_t)(stage * sizeof(uint64_t)));
        }
        if (++stage == NF_STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------------ epilogue warps 2..5 (both CTAs)
    const int q = warp & 3;
    EpiWarp ew{&tmO, 1, sE + (warp - 2) * 2 * EPI_BUF, 0, lane};
    EpiWarp ewp{&tmP, 1, sE + (warp - 2) * 2 * EPI_BUF, 0, lane};  // same staging buffers: one map per store
    int it = 0;
    SegWalk walk(pair, pairs, num_m, num_n, nk, p.streamk);
    Seg sg;
    for (; walk.next(sg); ++it) {
      const int mb = sg.mb, nb = sg.nb;
      const bool partial = sg.slot >= 0;
      const int acc = it & 1;
      const uint32_t accph = (it >> 1) & 1;
      const bool ready = mbar_wait_bounded(&accf[acc], accph, abort_flag, p.err, kDevTimeoutAccFull);
      if (!__all_sync(0xffffffffu, ready)) break;  // the warp's TMEM loads need all 32 lanes
      tc_fence_after();
      const int64_t row0 = (int64_t)mb * 256 + (int64_t)rank * 128 + 32 * q;
      const uint32_t tacc = tmem_base + ((uint32_t)(32 * q) << 16) + acc * 256;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t r32[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tacc + 32 * c, r32);
        tmem_wait_ld();
        const int64_t col0 = (int64_t)nb * 256 + 32 * c;
        const bool st = row0 < p.M && col0 < p.N;
        uint32_t o[32];
        if (partial) {
          // the tile's f32 partial into its workspace slot: [slot][256 rows][256 columns], every row and column
          ewp.sel = ew.sel;
          ewp.store(r32, 128, 32 * c, sg.slot * 256 + (int32_t)rank * 128 + 32 * q, true);
          ew.sel = ewp.sel;
        } else {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = bf16r(__uint_as_float(r32[i]));  // the bf16 GEMM output
          if (p.bias) {
            const int valid = clamp32(p.N - col0);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __fadd_rn(v[i], i < valid ? bf16r(__ldg(p.bias + col0 + i)) : 0.f);
          }
          ew.store(o, pack_out(v, 2, o), (int32_t)col0, (int32_t)row0, st);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(&acce[acc], 0));
    }
    if (lane == 0) bulk_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// x2 = bf16(x * bf16 pre_quant_scale), 8 elements per thread-iteration (weights.rs:617-620)
__global__ void awq_scale_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ pqs,
                                 uint16_t* __restrict__ x2, int64_t M, int64_t K) {
  const int64_t nv = M * K / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = (v * 8) % K;
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(x) + v);
    const uint4 s = __ldg(reinterpret_cast<const uint4*>(pqs + k));
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, sw[4] = {s.x, s.y, s.z, s.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = pack_bf2(__fmul_rn(__uint_as_float(aw[i] << 16), __uint_as_float(sw[i] << 16)),
                      __fmul_rn(__uint_as_float(aw[i] & 0xffff0000u), __uint_as_float(sw[i] & 0xffff0000u)));
    reinterpret_cast<uint4*>(x2)[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Pair whose stream-K range [W p / P, W (p + 1) / P) holds k-block position x.
__device__ __forceinline__ int pair_of(int64_t x, int64_t w, int pairs) {
  int p = (int)(x * pairs / w);
  while (p + 1 < pairs && w * (p + 1) / pairs <= x) ++p;
  while (p > 0 && w * p / pairs > x) --p;
  return p;
}

// The stream-K fix-up: for every tile that more than one pair worked on, out = bf16(bf16(sum of the pairs' f32
// slots, in pair order) + bf16(bias)), the finish the kernel's epilogue gives a whole tile.  One CTA per
// (tile, 32-row block), four columns per thread-iteration; tiles that one pair finished are skipped.
constexpr int kMaxFixupSlots = 64;  // pairs sharing one tile: the plan keeps every range >= nk / 62 k-blocks

__global__ void __launch_bounds__(256) streamk_fixup_kernel(const float* __restrict__ part,
                                                            const float* __restrict__ bias, uint16_t* __restrict__ out,
                                                            int64_t M, int64_t N, int num_m, int num_n, int nk,
                                                            int pairs) {
  __shared__ int slots[kMaxFixupSlots];
  __shared__ int nslots;
  const int tile = (int)(blockIdx.x >> 3), rb = (int)(blockIdx.x & 7);
  if (threadIdx.x == 0) {
    const int64_t w = (int64_t)num_m * num_n * nk;
    const int p0 = pair_of((int64_t)tile * nk, w, pairs), p1 = pair_of((int64_t)(tile + 1) * nk - 1, w, pairs);
    int n = 0;
    if (p1 > p0)  // more than one pair: every pair's piece of the tile is in its first (2q) or last (2q+1) slot
      for (int q = p0; q <= p1 && n < kMaxFixupSlots; ++q) slots[n++] = (w * q / pairs) / nk == tile ? 2 * q : 2 * q + 1;
    nslots = n;
  }
  __syncthreads();
  const int ns = nslots;
  if (ns == 0) return;
  int mb, nb;
  tile_coords(tile, num_m, num_n, num_m, mb, nb);
  for (int i = threadIdx.x; i < 32 * 64; i += blockDim.x) {
    const int r = rb * 32 + i / 64, c = 4 * (i % 64);
    const int64_t row = (int64_t)mb * 256 + r, col = (int64_t)nb * 256 + c;
    if (row >= M || col >= N) continue;  // N % 128 == 0: a 4-column group is inside or outside together
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < ns; ++j) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(part + ((int64_t)slots[j] * 256 + r) * 256 + c));
      acc.x = __fadd_rn(acc.x, v.x); acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z); acc.w = __fadd_rn(acc.w, v.w);
    }
    float o[4] = {bf16r(acc.x), bf16r(acc.y), bf16r(acc.z), bf16r(acc.w)};
    if (bias) {
      const float4 b = (reinterpret_cast<uintptr_t>(bias) & 15u) == 0
                           ? __ldg(reinterpret_cast<const float4*>(bias + col))
                           : make_float4(__ldg(bias + col), __ldg(bias + col + 1), __ldg(bias + col + 2),
                                         __ldg(bias + col + 3));
      o[0] = __fadd_rn(o[0], bf16r(b.x)); o[1] = __fadd_rn(o[1], bf16r(b.y));
      o[2] = __fadd_rn(o[2], bf16r(b.z)); o[3] = __fadd_rn(o[3], bf16r(b.w));
    }
    *reinterpret_cast<uint2*>(out + row * N + col) = make_uint2(pack_bf2(o[0], o[1]), pack_bf2(o[2], o[3]));
  }
}

static int nvfp4_pairs(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 1;
  if (!cache[dev]) {
    cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)NF_SMEM);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(NF_THREADS, 1, 1);
    cfg.dynamicSmemBytes = NF_SMEM;
    cfg.gridDim = dim3(2 * (sm_count(dev) / 2), 1, 1);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, nvfp4_gemm_kernel, &cfg) != cudaSuccess || clusters < 1) clusters = 1;
    cache[dev] = clusters;
  }
  return cache[dev];
}

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

struct Nvfp4Plan {
  int streamk;  // 1: stream-K ranges of k-blocks over `pairs` pairs
  int pairs;    // pairs launched
  size_t x2_bytes, part_bytes;
};

// Whole tiles round-robin when they fill the co-resident pairs in whole waves to 85% or more; stream-K otherwise,
// over as many pairs as keep every range at 8 k-blocks or more.
static Nvfp4Plan nvfp4_plan(int64_t m, int64_t n, int64_t k, bool awq) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t tiles = ((m + 255) / 256) * ((n + 255) / 256);
  const int64_t nk = k / 64;
  const int pairs = nvfp4_pairs(dev);
  Nvfp4Plan pl;
  const int64_t waves = (tiles + pairs - 1) / pairs;
  const double eff = (double)tiles / ((double)waves * pairs);
  // every stream-K range at least 8 k-blocks, and long enough that at most 64 pairs share a tile (the fix-up's
  // slot list)
  const int64_t min_range = nk / 62 > 8 ? nk / 62 : 8;
  const int64_t sk_pairs = (tiles * nk / min_range) < pairs ? tiles * nk / min_range : pairs;
  // measured on the text encoder's layers at M = 512: 200 tiles on 74 pairs (0.90 of whole waves) run faster
  // round-robin (0.131 ms against 0.141 stream-K, whose fix-up reads ~40 MB of partials), 40 tiles (0.54) faster
  // stream-K (0.134 ms against 0.163 with a 3-way split-K)
  pl.streamk = (eff < 0.85 && sk_pairs > 1) ? 1 : 0;
  pl.pairs = pl.streamk ? (int)sk_pairs : (int)(tiles < pairs ? tiles : pairs);
  pl.x2_bytes = awq ? align256((size_t)m * k * 2) : 0;
  pl.part_bytes = pl.streamk ? (size_t)2 * pl.pairs * 256 * 256 * 4 : 0;
  return pl;
}

}  // namespace h3q

using namespace h3q;

namespace {
h3q_status nf_fail(h3q_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  h3q::set_last_error(buf);
  return s;
}
int* nf_err_word() {
  // time-outs of this kernel are latched into the same per-device word as the int8 path's
  return h3q::error_word_current();
}
}  // namespace

extern "C" size_t h3q_nvfp4_linear_workspace_size(int64_t m, int64_t n, int64_t k, int has_pre_quant_scale) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const Nvfp4Plan pl = nvfp4_plan(m, n, k, has_pre_quant_scale != 0);
  return pl.x2_bytes + pl.part_bytes;
}

extern "C" h3q_status h3q_nvfp4_linear(const uint16_t* x, const uint16_t* pre_quant_scale, const uint8_t* q,
                                       const uint8_t* block_scale, const float* global_scale, const float* bias,
                                       uint16_t* out, int64_t m, int64_t n, int64_t k, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  const char* what = "h3q_nvfp4_linear";
  if (m < 0 || n < 0 || k < 0) return nf_fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (m == 0 || n == 0) return H3Q_OK;
  if (k % 64 != 0 || n % 128 != 0)
    return nf_fail(H3Q_ERR_UNSUPPORTED, "%s: this build needs k %% 64 == 0 and n %% 128 == 0 (k %lld, n %lld)", what,
                   (long long)k, (long long)n);
  if (!x || !q || !block_scale || !global_scale || !out) return nf_fail(H3Q_ERR_ARG, "%s: null pointer", what);
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(x) || !al16(q) || !al16(block_scale) || !al16(out) || (pre_quant_scale && !al16(pre_quant_scale)))
    return nf_fail(H3Q_ERR_ARG, "%s: tensors must be 16-byte aligned", what);
  const Nvfp4Plan pl = nvfp4_plan(m, n, k, pre_quant_scale != nullptr);
  if (workspace_bytes < pl.x2_bytes + pl.part_bytes || (pl.x2_bytes + pl.part_bytes > 0 && !workspace))
    return nf_fail(H3Q_ERR_WORKSPACE, "%s: workspace of %zu bytes, need %zu", what, workspace_bytes,
                   pl.x2_bytes + pl.part_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* wsp = static_cast<uint8_t*>(workspace);
  const uint16_t* xa = x;
  if (pre_quant_scale) {
    uint16_t* x2 = reinterpret_cast<uint16_t*>(wsp);
    const int64_t nv = m * k / 8;
    const int64_t blocks = (nv + 255) / 256;
    awq_scale_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, st>>>(x, pre_quant_scale, x2, m, k);
    xa = x2;
  }
  float* part = reinterpret_cast<float*>(wsp + pl.x2_bytes);
  CUtensorMap ta, tb, to;
  auto fn = encode_fn();
  if (!fn) return nf_fail(H3Q_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", what);
  {
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
    cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    if (fn(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(xa), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return nf_fail(H3Q_ERR_CUDA, "%s: activation tensor map", what);
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)(k / 2), (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)(k / 2)};
    cuuint32_t box[2] = {32, 128};
    cuuint32_t es[2] = {1, 1};
    if (fn(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return nf_fail(H3Q_ERR_CUDA, "%s: weight tensor map", what);
  }
  CUtensorMap tp;  // stream-K partial slots: [2 pairs x 256 rows, 256 columns] f32
  if (!make_tmap_out(&to, out, (uint64_t)m, (uint64_t)n, 2, 64) ||
      !make_tmap_out(&tp, pl.streamk ? (void*)part : (void*)out, pl.streamk ? (uint64_t)2 * pl.pairs * 256 : 1,
                     pl.streamk ? 256 : 32, 4, 128))
    return nf_fail(H3Q_ERR_CUDA, "%s: output tensor map", what);
  Nvfp4Args a{};
  a.M = m; a.N = n; a.K = k;
  a.bscale = block_scale; a.gscale = global_scale;
  a.bias = bias;
  a.streamk = pl.streamk;
  a.err = nf_err_word();
  const int num_m = (int)((m + 255) / 256), num_n = (int)((n + 255) / 256);
  const int nk = (int)(k / 64);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(NF_THREADS, 1, 1);
  cfg.dynamicSmemBytes = NF_SMEM;
  cfg.gridDim = dim3(2 * pl.pairs, 1, 1);
  cfg.stream = st;
  cudaError_t e = cudaLaunchKernelEx(&cfg, nvfp4_gemm_kernel, ta, tb, to, tp, a, num_m, num_n, nk);
  if (e == cudaSuccess && pl.streamk) {
    streamk_fixup_kernel<<<(unsigned)(num_m * num_n * 8), 256, 0, st>>>(part, bias, out, m, n, num_m, num_n, nk,
                                                                        pl.pairs);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return nf_fail(H3Q_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return H3Q_OK;
}
