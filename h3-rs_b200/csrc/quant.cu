// quant.cu -- fused ConvRot (block-diagonal Hadamard-256) rotation + per-row symmetric int8 quantization.
//
// Replaces kernels.rs's quant_rows_i8_rot2 (kernels.rs:220-293), quant_rows_i8_rot (kernels.rs:166-213) and
// quant_rows_i8 (kernels.rs:296-318).  Codes and scales are bit-identical to the kernel the reference would
// select for the same call (kernels.rs:1133-1161):
//   order 2 -- the warp-shuffle butterfly of quant_rows_i8_rot2: digit 0 sums ((a0+a1)+a2)+a3, digits 1-3 sum
//              (a0+a1)+(a2+a3), out_p = s - 2 a_{3-p}; codes clamp(__float2int_rn(v*inv)) (NaN -> 0);
//   order 1 -- the shared-memory butterfly of quant_rows_i8_rot: out_0 = ((a0+a1)+a2)-a3, out_1 =
//              ((a0+a1)-a2)+a3, out_2 = ((a0-a1)+a2)+a3, out_3 = ((-a0+a1)+a2)+a3; codes
//              min(max(rintf(v*inv), -128), 127) (NaN -> -128);
//   order 0 -- no rotation (quant_rows_i8), same code rule as order 1.
// Scale s = fmaxf(max|v| / 127, 1e-30), inv = 1 / s, both IEEE-rounded divisions.
//
// Layout (B200 design, not the reference's): one thread owns 64 contiguous elements of a 256-group, so base-4
// digits 0..2 of the in-group index are transformed in registers and only digit 3 crosses a lane quad (three
// shuffles per element, against about seven and a half in the reference's 8-elements-per-lane layout, which
// makes that kernel shuffle-bound well below HBM bandwidth on B200).  Rounding to the nearest-even integer
// uses the exact FADD trick (t + 1.5*2^23) instead of F2I conversions, which issue at a quarter of the FP32
// rate.  One warp-aligned thread team of roundup(4G, 32) threads per row; the row max is a warp reduction
// plus one shared-memory atomic per warp.
#include <climits>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "h3q_internal.h"

namespace h3q {

template <typename T> struct In;
template <> struct In<float> {
  static constexpr int kVec = 4;  // elements per 16-byte load
  __device__ static void cvt(const uint4& r, float* o) {
    o[0] = __uint_as_float(r.x); o[1] = __uint_as_float(r.y); o[2] = __uint_as_float(r.z); o[3] = __uint_as_float(r.w);
  }
};
template <> struct In<__half> {
  static constexpr int kVec = 8;
  __device__ static void cvt(const uint4& r, float* o) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = h2f((uint16_t)(w[i] & 0xffffu));
      o[2 * i + 1] = h2f((uint16_t)(w[i] >> 16));
    }
  }
};
template <> struct In<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ static void cvt(const uint4& r, float* o) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = __uint_as_float(w[i] << 16);
      o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};

// One in-register radix-4 stage over the 4 values a[b], a[b+st], a[b+2st], a[b+3st].  `s - 2a` is one FFMA:
// 2a is exact, so fma(-2, a, s) rounds the same real number once, as the reference's `s - 2.f * partner`.
template <int ORDER>
__device__ __forceinline__ void h4_inreg(float& a0, float& a1, float& a2, float& a3, bool first) {
  if (ORDER == 2) {
    float s = first ? __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3) : __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    float b0 = __fmaf_rn(-2.f, a3, s), b1 = __fmaf_rn(-2.f, a2, s);
    float b2 = __fmaf_rn(-2.f, a1, s), b3 = __fmaf_rn(-2.f, a0, s);
    a0 = b0; a1 = b1; a2 = b2; a3 = b3;
  } else {
    float b0 = __fsub_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
    float b1 = __fadd_rn(__fsub_rn(__fadd_rn(a0, a1), a2), a3);
    float b2 = __fadd_rn(__fadd_rn(__fsub_rn(a0, a1), a2), a3);
    float b3 = __fadd_rn(__fadd_rn(__fsub_rn(a1, a0), a2), a3);
    a0 = b0; a1 = b1; a2 = b2; a3 = b3;
  }
}

// Digit-3 butterfly of two columns at once: a_p holds (column c, column c+1) for digit-3 value p.
template <int ORDER>
__device__ __forceinline__ void h4_pair(f2& a0, f2& a1, f2& a2, f2& a3) {
  if (ORDER == 2) {
    const f2 s = add2(add2(a0, a1), add2(a2, a3));
    const f2 m2 = pk(-2.f, -2.f);
    const f2 b0 = fma2(m2, a3, s), b1 = fma2(m2, a2, s), b2 = fma2(m2, a1, s), b3 = fma2(m2, a0, s);
    a0 = b0; a1 = b1; a2 = b2; a3 = b3;
  } else {
    const f2 b0 = sub2(add2(add2(a0, a1), a2), a3);
    const f2 b1 = add2(sub2(add2(a0, a1), a2), a3);
    const f2 b2 = add2(add2(sub2(a0, a1), a2), a3);
    const f2 b3 = add2(add2(sub2(a1, a0), a2), a3);
    a0 = b0; a1 = b1; a2 = b2; a3 = b3;
  }
}

// Both halves rounded to bf16 (cvt.rn.bf16x2: nearest even, the reference's f2bf for finite values) and widened.
__device__ __forceinline__ f2 bf16r2(f2 v) {
  float lo, hi;
  upk(v, lo, hi);
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
  return pk(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
}

// Slot of a thread's 16-byte chunk c inside its exchange line: c ^ f(t).  With f(t) = (t & 7) ^ bit2(t), the
// 8 lanes of a shared-memory phase hit 8 different bank groups both when each writes its own line and when the
// lanes of two quads read chunks 2j, 2j+1 of one quad member's line.
__device__ __forceinline__ int xslot(int t) { return (t & 7) ^ ((t >> 2) & 1); }

// int8 code of t = v * inv as a byte: nearest-even integer through t + 1.5*2^23 (exact for |t| < 2^22; |t| <=
// 127 here by construction of inv).  NaN -> 0 (order 2, cvt.rni) or -128 (orders 0/1, fmaxf(rintf(t), -128)).
template <int ORDER>
__device__ __forceinline__ uint32_t code_of(float t) {
  if (ORDER != 2) t = fmaxf(t, -128.f);
  const uint32_t b = (uint32_t)__float_as_int(__fadd_rn(t, 12582912.0f)) & 0xffu;
  return (ORDER == 2 && t != t) ? 0u : b;
}

// Persistent row quantizer.  One CTA = one team of roundup(4G, 32) threads working through rows
// blockIdx.x, blockIdx.x + gridDim.x, ...; thread t < 4G owns elements [64t, 64t + 64) of the row.  Rows arrive
// by TMA (the row viewed as [K*es/128] x 128-byte lines, 128-byte swizzle) into a 3-stage ring, two rows ahead
// of the compute; with the swizzle each thread's 16-byte reads of its own line are bank-conflict free.
constexpr int kQStages = 3;
// MOD keeps two rows in flight: its shared-memory table slices (below) would otherwise cost a CTA per SM.
constexpr int kQStagesMod = 2;

// ROT_ONLY: write bf16(rotated row) to `ybf` instead of codes and scales (rotate_activation, weights.rs:482-489,
// for the paths that quantize a pre-rotated activation).
// MOD: apply RMSNorm + adaLN modulate to the row first (rms_modulate, kernels.rs:376-401; bf16 rows only):
//   inv = rsqrtf(sum(x^2) / K + eps), summed in that kernel's order (512 thread partials, thread t taking
//   elements t, t+512, ... with a fused multiply-add, then xor trees in 32-thread groups and over the 16 group sums);
//   n = bf16((x * inv) * w[c]); y = bf16(fma(n, 1 + bf16(scale[idx[r], c]), bf16(shift[idx[r], c]))).
// y is then rotated and quantized as the row would be after rms_modulate wrote it to memory: one pass instead of
// a bf16 round trip through HBM.  With ORDER 0 and ROT_ONLY the kernel writes y itself (rms_modulate).
struct ModArgs {
  const uint16_t* w;       // bf16 [K] norm weight
  const float* scale;      // f32 [R, K] adaLN scale table
  const float* shift;      // f32 [R, K] adaLN shift table
  const uint32_t* idx;     // [M] table row of each activation row
  float eps;
};

template <int ORDER, typename Tin, bool ROT_ONLY, bool MOD>
__device__ __forceinline__ void quant_rows_body(const CUtensorMap& tmx, int8_t* __restrict__ q,
                                                float* __restrict__ scale, int64_t M, int K, int box_rows,
                                                int boxes_per_row, int* err, uint16_t* __restrict__ ybf,
                                                const ModArgs& mod) {
  constexpr int NST = MOD ? kQStagesMod : kQStages;
  extern __shared__ uint8_t qsm_raw[];
  // align by offsetting the __shared__ array itself, so the compiler keeps shared-space (LDS/STS) accesses
  uint8_t* qsm = qsm_raw + ((1024u - (smem_u32(qsm_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full[NST];
  __shared__ unsigned s_max[3], s_max2[3];
  __shared__ float s_red[2][16];
  __shared__ int s_abort;
  constexpr int ES = sizeof(Tin);
  constexpr int LINES = 64 * ES / 128;  // 128-byte lines per thread: 1 (16-bit) or 2 (f32)
  const int G = K >> 8;
  const int t = threadIdx.x, j = t & 3;
  const bool owner = t < 4 * G;
  const uint32_t row_bytes = (uint32_t)K * ES;
  const uint32_t stage_bytes = (row_bytes + 1023u) & ~1023u;

  if (t == 0) {
    for (int s = 0; s < NST; ++s) mbar_init(&full[s], 1);
    s_max[0] = s_max[1] = s_max[2] = 0u;
    s_max2[0] = s_max2[1] = s_max2[2] = 0u;
    s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int64_t row, int stage) {
    mbar_arrive_expect_tx(&full[stage], row_bytes);
    for (int b = 0; b < boxes_per_row; ++b)
      tma_load_2d(qsm + (size_t)stage * stage_bytes + (size_t)b * box_rows * 128, &tmx, &full[stage], 0,
                  (int32_t)(row * box_rows * boxes_per_row + b * box_rows));
  };
  // Rows of this CTA: every gridDim.x-th row, or with MOD a contiguous block (neighbouring tokens share their
  // adaLN table row, which then stays in L1).
  const int64_t blk = (M + gridDim.x - 1) / gridDim.x;
  const int64_t rb0 = MOD ? (int64_t)blockIdx.x * blk : (int64_t)blockIdx.x;
  const int64_t rend = MOD ? (rb0 + blk < M ? rb0 + blk : M) : M;
  auto row_of = [&](int64_t i) -> int64_t { return MOD ? rb0 + i : rb0 + i * (int64_t)gridDim.x; };
  if (t == 0) {
    tma_prefetch_desc(&tmx);
    for (int s = 0; s < NST; ++s) {
      const int64_t r = row_of(s);
      if (r < rend) issue(r, s);
    }
  }
  uint32_t tab_idx = 0xffffffffu;  // MOD: table row held in this thread's shared-memory slice
  const int nown = 4 * G;           // owner threads (the table slices' stride)
  // MOD: rms_modulate's 16 group sums of squares of the landed row at `base` (128-byte-swizzled lines) -> dst[16].
  // The next row's sums are formed under the current row's max barrier, so a row costs one CTA barrier.
  auto partials = [&](const uint8_t* base, float* dst) {
    const int nw = blockDim.x >> 5, wp = t >> 5, ln = t & 31;
    if (blockDim.x >= 64) {
      // thread m < 64 holds the partials of reference threads 8m .. 8m+7 (one 16-byte piece per 512-element
      // stride, conflict-free); the reference's 32-thread xor trees are 4 neighbouring lanes here: levels 16 and
      // 8 cross lanes (xor 2, xor 1), levels 4, 2, 1 stay inside the thread
      float a[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = 0.f;
      if (t < 64) {
        for (int c0 = 8 * t; c0 < K; c0 += 512) {
          const int line = c0 >> 6, ch = (c0 >> 3) & 7;
          const uint4 r8 = *reinterpret_cast<const uint4*>(base + line * 128 + ((ch ^ (line & 7)) << 4));
          const uint32_t ww[4] = {r8.x, r8.y, r8.z, r8.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float x0 = __uint_as_float(ww[i] << 16), x1 = __uint_as_float(ww[i] & 0xffff0000u);
            a[2 * i] = __fmaf_rn(x0, x0, a[2 * i]);
            a[2 * i + 1] = __fmaf_rn(x1, x1, a[2 * i + 1]);
          }
        }
      }
#pragma unroll
      for (int lo = 2; lo >= 1; lo >>= 1) {  // tree levels 16 (lanes xor 2) and 8 (lanes xor 1)
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] = __fadd_rn(a[i], __shfl_xor_sync(0xffffffffu, a[i], lo));
      }
#pragma unroll
      for (int o = 4; o >= 1; o >>= 1) {  // tree levels 4, 2, 1
        float b[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) b[i] = __fadd_rn(a[i], a[i ^ o]);
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] = b[i];
      }
      if (t < 64 && (t & 3) == 0) dst[t >> 2] = a[0];
    } else {
      for (int rw = wp; rw < 16; rw += nw) {
        float sq = 0.f;
        for (int c = 32 * rw + ln; c < K; c += 512) {
          const int line = c >> 6, ch = (c >> 3) & 7;
          const float xv = bf2f(*reinterpret_cast<const uint16_t*>(base + line * 128 + ((ch ^ (line & 7)) << 4) +
                                                                   (c & 7) * 2));
          sq = __fmaf_rn(xv, xv, sq);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
        if (ln == 0) dst[rw] = sq;
      }
    }
  };
  bool stop = false;
  if (MOD && rb0 < rend) {
    const bool landed = mbar_wait_bounded(&full[0], 0u, &s_abort, err, kDevTimeoutFull);
    partials(qsm, s_red[0]);
    stop = !__syncthreads_and(landed);
  }
  int it = 0;
  for (int64_t row = row_of(0); row < rend; row = row_of(++it)) {
    const int stage = it % NST;
    if (MOD && owner) {
      // The thread's bf16 scale / shift values of the row's table row live in its slice of shared memory
      // (16-byte word i at tab + (i * 4G + t) * 16, columns 4i .. 4i+3 as scale pairs then shift pairs:
      // conflict-free), reloaded, before the row has landed, only when the table index changes.
      const uint32_t ridx = __ldg(mod.idx + row);
      if (ridx != tab_idx) {
        uint8_t* tab = qsm + (size_t)NST * stage_bytes;
        const float4* scv = reinterpret_cast<const float4*>(mod.scale + (int64_t)ridx * K + 64 * t);
        const float4* shv = reinterpret_cast<const float4*>(mod.shift + (int64_t)ridx * K + 64 * t);
#pragma unroll 4
        for (int q4 = 0; q4 < 16; ++q4) {
          const float4 a = __ldg(scv + q4), b = __ldg(shv + q4);
          uint32_t o[4];
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[0]) : "f"(a.y), "f"(a.x));
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[1]) : "f"(a.w), "f"(a.z));
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[2]) : "f"(b.y), "f"(b.x));
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[3]) : "f"(b.w), "f"(b.z));
          *reinterpret_cast<uint4*>(tab + ((size_t)q4 * nown + t) * 16) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        tab_idx = ridx;
      }
    }
    float inv_rms = 0.f;
    if (!MOD) {
      // one thread waits for the row's bytes (its mbarrier wait acquires them); the barrier then orders that wait
      // before every other thread's reads, and those threads sleep in the barrier instead of polling the mbarrier
      bool landed = true;
      if (t == 0) landed = mbar_wait_bounded(&full[stage], (uint32_t)(it / NST) & 1u, &s_abort, err, kDevTimeoutFull);
      if (!__syncthreads_and(landed)) break;  // the whole CTA gives up together (barriers follow)
    } else {
      if (stop) break;  // the row did not land (the CTA agreed under the previous barrier)
      // the reference's last xor tree over its 16 group sums, as lane 0 forms it (level 16 adds zeros)
      const float* g = s_red[it & 1];
      float a8[8], a4[4];
#pragma unroll
      for (int i = 0; i < 8; ++i) a8[i] = __fadd_rn(g[i], g[i + 8]);
#pragma unroll
      for (int i = 0; i < 4; ++i) a4[i] = __fadd_rn(a8[i], a8[i + 4]);
      const float tot = __fadd_rn(__fadd_rn(a4[0], a4[2]), __fadd_rn(a4[1], a4[3]));
      inv_rms = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), mod.eps));
    }
    // The thread's 64 values as 32 register pairs: v2[k] = elements (2k, 2k + 1).  Pairs of neighbouring elements
    // follow the same butterfly through digits 1..3, so those stages run as paired f32x2 operations.
    f2 v2[32];
    if (MOD && owner) {
      // y = bf16(fma(bf16((x * inv) * w), 1 + bf16(scale), bf16(shift))) for the thread's columns 64t .. 64t+63
      // (its own 128-byte line), two columns per instruction, written back in place as bf16 (y is a bf16 value);
      // the roundings are cvt.rn (nearest even, as the reference's f2bf for every finite value; a NaN stays a
      // NaN).  One 16-byte chunk at a time keeps the register footprint of the pass small.
      uint8_t* own = qsm + (size_t)stage * stage_bytes + (size_t)t * 128;
      const uint8_t* tab = qsm + (size_t)NST * stage_bytes;
      const f2 inv2 = pk(inv_rms, inv_rms), one2 = pk(1.f, 1.f);
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint4* px = reinterpret_cast<uint4*>(own + ((c ^ (t & 7)) << 4));
        const uint4 raw = *px;
        const uint4 w8 = __ldg(reinterpret_cast<const uint4*>(mod.w + 64 * t) + c);
        const uint4 tb0 = *reinterpret_cast<const uint4*>(tab + ((size_t)(2 * c) * nown + t) * 16);
        const uint4 tb1 = *reinterpret_cast<const uint4*>(tab + ((size_t)(2 * c + 1) * nown + t) * 16);
        const uint32_t xx[4] = {raw.x, raw.y, raw.z, raw.w}, ww[4] = {w8.x, w8.y, w8.z, w8.w};
        const uint32_t sp[4] = {tb0.x, tb0.y, tb1.x, tb1.y}, hp[4] = {tb0.z, tb0.w, tb1.z, tb1.w};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // columns 8c + 2i, +1
          const f2 x2 = pk(__uint_as_float(xx[i] << 16), __uint_as_float(xx[i] & 0xffff0000u));
          const f2 w2 = pk(__uint_as_float(ww[i] << 16), __uint_as_float(ww[i] & 0xffff0000u));
          const f2 sc2 = pk(__uint_as_float(sp[i] << 16), __uint_as_float(sp[i] & 0xffff0000u));
          const f2 sh2 = pk(__uint_as_float(hp[i] << 16), __uint_as_float(hp[i] & 0xffff0000u));
          const f2 n = bf16r2(mul2(mul2(x2, inv2), w2));
          float y0, y1;
          upk(fma2(n, add2(one2, sc2), sh2), y0, y1);
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[i]) : "f"(y1), "f"(y0));
        }
        *px = make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();  // these generic writes precede a later TMA refill of the stage
    }
    if (owner) {
      const uint8_t* base = qsm + (size_t)stage * stage_bytes;
#pragma unroll
      for (int l = 0; l < LINES; ++l) {
        const int line = t * LINES + l;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 raw = *reinterpret_cast<const uint4*>(base + line * 128 + ((c ^ (line & 7)) << 4));
          float tmp[In<Tin>::kVec];
          In<Tin>::cvt(raw, tmp);
#pragma unroll
          for (int i = 0; i < In<Tin>::kVec / 2; ++i)
            v2[((l * 8 + c) * In<Tin>::kVec) / 2 + i] = pk(tmp[2 * i], tmp[2 * i + 1]);
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) v2[k] = pk(0.f, 0.f);
    }
    // Digit 3 crosses the quad.  Transpose through shared memory in two passes of 32 columns, each thread
    // writing into its own (already consumed) 128-byte line of this stage: afterwards thread j holds, for all
    // four digit-3 values, columns 8j..8j+7 (pass 0) and 32+8j..32+8j+7 (pass 1) of its group.
    f2 u2[4][8];  // u2[d3][i] = columns (2i, 2i + 1) of the thread's two 8-column slices, in pass order
    if (ORDER != 0) {
      // digit 0 (element offsets 1): within a pair, so scalar, with the reference's first-stage sum order
#pragma unroll
      for (int b4 = 0; b4 < 16; ++b4) {
        float a0, a1, a2, a3;
        upk(v2[2 * b4], a0, a1);
        upk(v2[2 * b4 + 1], a2, a3);
        h4_inreg<ORDER>(a0, a1, a2, a3, true);
        v2[2 * b4] = pk(a0, a1);
        v2[2 * b4 + 1] = pk(a2, a3);
      }
      // digit 1 (element offsets 4 = pair offsets 2) and digit 2 (offsets 16 = pair offsets 8), paired
#pragma unroll
      for (int blk = 0; blk < 4; ++blk)
#pragma unroll
        for (int k = 0; k < 2; ++k)
          h4_pair<ORDER>(v2[8 * blk + k], v2[8 * blk + k + 2], v2[8 * blk + k + 4], v2[8 * blk + k + 6]);
#pragma unroll
      for (int k = 0; k < 8; ++k) h4_pair<ORDER>(v2[k], v2[k + 8], v2[k + 16], v2[k + 24]);
      uint8_t* xb = qsm + (size_t)stage * stage_bytes;
      uint8_t* own = xb + (size_t)t * LINES * 128;
      const int fo = xslot(t);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        if (owner) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float x0, x1, x2, x3;
            upk(v2[16 * r + 2 * c], x0, x1);
            upk(v2[16 * r + 2 * c + 1], x2, x3);
            *reinterpret_cast<float4*>(own + ((c ^ fo) << 4)) = make_float4(x0, x1, x2, x3);
          }
        }
        __syncwarp();
        if (owner) {
#pragma unroll
          for (int d3 = 0; d3 < 4; ++d3) {
            const int tp = (t & ~3) | d3;
            const uint8_t* line = xb + (size_t)tp * LINES * 128;
            const int fp = xslot(tp);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float4 f = *reinterpret_cast<const float4*>(line + (((2 * j + e) ^ fp) << 4));
              u2[d3][4 * r + 2 * e] = pk(f.x, f.y);
              u2[d3][4 * r + 2 * e + 1] = pk(f.z, f.w);
            }
          }
        } else {
#pragma unroll
          for (int d3 = 0; d3 < 4; ++d3)
#pragma unroll
            for (int i = 0; i < 4; ++i) u2[d3][4 * r + i] = pk(0.f, 0.f);
        }
        __syncwarp();
      }
      fence_proxy_async_smem();  // these generic writes precede a later TMA refill of the stage
#pragma unroll
      for (int i = 0; i < 8; ++i) h4_pair<ORDER>(u2[0][i], u2[1][i], u2[2][i], u2[3][i]);
    } else {
#pragma unroll
      for (int d3 = 0; d3 < 4; ++d3)
#pragma unroll
        for (int i = 0; i < 8; ++i) u2[d3][i] = v2[8 * d3 + i];
    }
    // Row maximum of |v|, NaN-propagating: rows holding an Inf or NaN (max bits >= the Inf pattern) take the exact
    // slow path below; every other row needs neither the NaN-ignoring max nor per-element NaN / clamp selects.
    // max|v| = max(max v, -min v): two 3-input operations per pair, no absolute values.
    float m = 0.f;
    if (!ROT_ONLY) {
      float mx = 0.f, mn = 0.f;
#pragma unroll
      for (int d3 = 0; d3 < 4; ++d3)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float x0, x1;
          upk(u2[d3][i], x0, x1);
          asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(mx) : "f"(mx), "f"(x0), "f"(x1));
          asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(mn) : "f"(mn), "f"(x0), "f"(x1));
        }
      asm("max.NaN.f32 %0, %1, %2;" : "=f"(m) : "f"(mx), "f"(-mn));
    }
    const unsigned mw = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
    const int slot = it % 3;
    if ((t & 31) == 0 && !ROT_ONLY) atomicMax(&s_max[slot], mw);
    if (MOD) {
      // the next row's group sums (it was issued a row earlier), under this row's barrier
      bool ok = true;
      const int64_t nx = row_of(it + 1);
      if (nx < rend) {
        const int ns = (it + 1) % NST;
        ok = mbar_wait_bounded(&full[ns], (uint32_t)((it + 1) / NST) & 1u, &s_abort, err, kDevTimeoutFull);
        partials(qsm + (size_t)ns * stage_bytes, s_red[(it + 1) & 1]);
      }
      stop = !__syncthreads_and(ok);  // the whole row is read out of `stage` and its max is complete
    } else {
      __syncthreads();  // the whole row is read out of `stage` and its max is complete
    }
    if (t == 0) {
      s_max[(it + 1) % 3] = 0u;
      s_max2[(it + 1) % 3] = 0u;
      const int64_t nr = row_of(it + NST);
      if (nr < rend) {
        fence_proxy_async_smem();
        issue(nr, stage);
      }
    }
    unsigned mbits = s_max[slot];
    const bool special = !ROT_ONLY && mbits >= 0x7f800000u;  // the same for every thread of the CTA
    if (special) {
      // the reference's max ignores NaN (fmaxf): reduce again without them
      float mf = 0.f;
#pragma unroll
      for (int d3 = 0; d3 < 4; ++d3)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float x0, x1;
          upk(u2[d3][i], x0, x1);
          mf = fmaxf(mf, fmaxf(fabsf(x0), fabsf(x1)));
        }
      const unsigned mw2 = __reduce_max_sync(0xffffffffu, __float_as_uint(mf));
      if ((t & 31) == 0) atomicMax(&s_max2[slot], mw2);
      __syncthreads();
      mbits = s_max2[slot];
    }
    // scale from the true max (the 1/16 of the rotation is folded in exactly: powers of two)
    const float mx = ORDER == 0 ? __uint_as_float(mbits) : __fmul_rn(__uint_as_float(mbits), 0.0625f);
    const float s = fmaxf(__fdiv_rn(mx, 127.f), 1e-30f);
    const float inv = ORDER == 0 ? __fdiv_rn(1.f, s) : __fmul_rn(__fdiv_rn(1.f, s), 0.0625f);
    if (ROT_ONLY && ORDER == 0) {  // the (modulated) row itself, contiguous columns 64t .. 64t+63
      if (owner) {
        uint4* dst = reinterpret_cast<uint4*>(ybf + row * (int64_t)K + 64 * t);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float y0, y1;
            upk(u2[h >> 1][4 * (h & 1) + e], y0, y1);
            o[e] = pack_bf2(y0, y1);
          }
          dst[h] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      continue;
    }
    if (ROT_ONLY) {
      if (owner) {
        uint16_t* dst = ybf + row * (int64_t)K + (t >> 2) * 256 + 8 * j;
        const f2 q16 = pk(0.0625f, 0.0625f);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const int d3 = h >> 1, i0 = 4 * (h & 1);
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float y0, y1;
            upk(mul2(u2[d3][i0 + e], q16), y0, y1);
            o[e] = pack_bf2(y0, y1);
          }
          *reinterpret_cast<uint4*>(dst + 64 * d3 + 32 * (h & 1)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      continue;
    }
    if (t == 0) scale[row] = s;
    if (owner) {
      const f2 inv2 = pk(inv, inv), rnd2 = pk(12582912.0f, 12582912.0f), zero2 = pk(0.f, 0.f);
      uint32_t w[16];  // w[2*h + k]: bytes of slice h's columns 4k .. 4k+3 (h = 2 d3 + pass)
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        const int d3 = h >> 1, i0 = 4 * (h & 1);
        uint32_t b[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float t0, t1, r0, r1;
          // t = u * inv rounded to f32 first, as the reference's v * inv.  Written as fma(u, inv, +0): ptxas
          // contracts a paired multiply feeding a paired add into one fused op (a single rounding of u * inv +
          // 1.5 * 2^23, which breaks ties differently), and cannot fuse an fma with the add.  A zero product's
          // sign does not matter here.
          const f2 tt = fma2(u2[d3][i0 + e], inv2, zero2);
          if (!special) {
            // |t| <= 127 by construction of inv: the nearest-even integer is the code, no clamp or NaN case
            // the code is the low byte of the sum's bits; the byte permutes below read only that byte
            upk(add2(tt, rnd2), r0, r1);
            b[2 * e] = __float_as_uint(r0);
            b[2 * e + 1] = __float_as_uint(r1);
          } else {
            upk(tt, t0, t1);
            b[2 * e] = code_of<ORDER>(t0);
            b[2 * e + 1] = code_of<ORDER>(t1);
          }
        }
        w[2 * h] = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
        w[2 * h + 1] = __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410);
      }
      if (ORDER != 0) {
        int8_t* dst = q + row * (int64_t)K + (t >> 2) * 256 + 8 * j;
#pragma unroll
        for (int h = 0; h < 8; ++h)
          *reinterpret_cast<uint2*>(dst + 64 * (h >> 1) + 32 * (h & 1)) = make_uint2(w[2 * h], w[2 * h + 1]);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(q + row * (int64_t)K + t * 64);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
    }
  }
  // drain: a CTA that stopped early must not exit with its own row loads in flight
  __syncthreads();
  if (t == 0) {
    int dummy = 0;
    for (int k = 0; k < NST; ++k) {
      const int i2 = it + k;  // loads issued for iterations it .. it+NST-1 may be pending
      const int64_t r = row_of(i2);
      if (r < rend) mbar_wait_bounded(&full[i2 % NST], (uint32_t)(i2 / NST) & 1u, &dummy, err, kDevTimeoutDrain);
    }
  }
  __syncthreads();
}

// The row quantizer without modulation, capped at 96 registers: with the 96-thread team of K = 5120 that is six
// CTAs (18 warps) per SM, where the compiler's own choice (103 registers) left room for five; no spills.
template <int ORDER, typename Tin, bool ROT_ONLY = false>
__global__ void __maxnreg__(96) quant_rows_kernel(const __grid_constant__ CUtensorMap tmx, int8_t* __restrict__ q,
                                                  float* __restrict__ scale, int64_t M, int K, int box_rows,
                                                  int boxes_per_row, int* err, uint16_t* __restrict__ ybf,
                                                  const ModArgs mod) {
  quant_rows_body<ORDER, Tin, ROT_ONLY, false>(tmx, q, scale, M, K, box_rows, boxes_per_row, err, ybf, mod);
}

// RMSNorm + modulate, then the quantizer (or the modulated row alone): the register cap above would spill here.
template <int ORDER, typename Tin, bool ROT_ONLY = false>
__global__ void __launch_bounds__(256) quant_rows_mod_kernel(const __grid_constant__ CUtensorMap tmx,
                                                             int8_t* __restrict__ q, float* __restrict__ scale,
                                                             int64_t M, int K, int box_rows, int boxes_per_row,
                                                             int* err, uint16_t* __restrict__ ybf, const ModArgs mod) {
  quant_rows_body<ORDER, Tin, ROT_ONLY, true>(tmx, q, scale, M, K, box_rows, boxes_per_row, err, ybf, mod);
}

// Unrotated per-row quantization for any K (quant_rows_i8, kernels.rs:296-318): one 256-thread block per row,
// a max pass and a code pass over the row (the second pass hits L2).
__device__ __forceinline__ float load_elem(const float* p, int i) { return p[i]; }
__device__ __forceinline__ float load_elem(const __half* p, int i) { return h2f(reinterpret_cast<const uint16_t*>(p)[i]); }
__device__ __forceinline__ float load_elem(const __nv_bfloat16* p, int i) {
  return bf2f(reinterpret_cast<const uint16_t*>(p)[i]);
}

template <typename Tin>
__global__ void __launch_bounds__(256) quant_rows_plain_kernel(const Tin* __restrict__ x, int8_t* __restrict__ q,
                                                               float* __restrict__ scale, int K) {
  __shared__ float red[8];
  const int64_t r = blockIdx.x;
  const Tin* xr = x + r * (int64_t)K;
  auto ld = [&](int i) -> float { return load_elem(xr, i); };
  float m = 0.f;
  for (int i = threadIdx.x; i < K; i += 256) m = fmaxf(m, fabsf(ld(i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float mx = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
  const float s = fmaxf(__fdiv_rn(mx, 127.f), 1e-30f), inv = __fdiv_rn(1.f, s);
  if (threadIdx.x == 0) scale[r] = s;
  int8_t* qr = q + r * (int64_t)K;
  for (int i = threadIdx.x; i < K; i += 256) qr[i] = (int8_t)code_of<0>(__fmul_rn(ld(i), inv));
}

static PFN_cuTensorMapEncodeTiled_v12000 q_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

template <int ORDER, typename Tin, bool ROT_ONLY = false, bool MOD = false>
static cudaError_t launch_rows(const void* x, int8_t* q, float* scale, int64_t M, int K, int* err, cudaStream_t st,
                               uint16_t* ybf = nullptr, const ModArgs* mod = nullptr) {
  constexpr int ES = sizeof(Tin);
  const int G = K / 256;
  const int threads = ((4 * G + 31) / 32) * 32;
  const int lines = K * ES / 128;  // 128-byte lines per row (4G for 16-bit input, 8G for f32)
  // TMA boxes hold at most 256 lines; each box must start on a 1024-byte (8-line) swizzle atom
  int box_rows = lines;
  if (lines > 256) {
    int d = G < 32 ? G : 32;
    while (G % d != 0) --d;
    box_rows = 8 * d;
  }
  const int boxes = lines / box_rows;
  auto fn = q_encode_fn();
  if (!fn) return cudaErrorInvalidValue;
  const size_t stage_bytes = ((size_t)K * ES + 1023) / 1024 * 1024;
  // MOD adds each owner thread's 64 columns of the current adaLN table row (bf16 scale / shift, 256 bytes); the
  // norm weight, the same for every row, is read through L1
  const size_t smem = 1024 + (MOD ? kQStagesMod : kQStages) * stage_bytes + (MOD ? (size_t)4 * G * 256 : 0);
  auto kern = [] {
    if constexpr (MOD) return quant_rows_mod_kernel<ORDER, Tin, ROT_ONLY>;
    else return quant_rows_kernel<ORDER, Tin, ROT_ONLY>;
  }();
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // the largest shared-memory carveout of the unified L1 / shared array, so the rings of more CTAs fit on an SM;
  // what the kernel reads through L1 (MOD's norm weight and table rows, a few KB per CTA) fits in the rest
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  int dev = 0, per_sm = 0;
  cudaGetDevice(&dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  const int64_t want = (int64_t)per_sm * sm_count(dev);
  // TMA row coordinates are int32: launch in chunks of rows whose line index stays below 2^31
  const int64_t chunk = ((int64_t)INT32_MAX - 256) / lines;
  for (int64_t r0 = 0; r0 < M; r0 += chunk) {
    const int64_t mc = (M - r0) < chunk ? (M - r0) : chunk;
    // the activation rows [r0, r0 + mc) as [mc * lines] x 128 bytes (elements of ES bytes)
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)(128 / ES), (cuuint64_t)mc * lines};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {(cuuint32_t)(128 / ES), (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    const CUtensorMapDataType dt = ES == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    const char* xb = static_cast<const char*>(x) + r0 * (int64_t)K * ES;
    if (fn(&m, dt, 2, const_cast<char*>(xb), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    const unsigned grid = (unsigned)(mc < want ? mc : want);
    ModArgs ma{};
    if (MOD) {
      ma = *mod;
      ma.idx = mod->idx + r0;
    }
    kern<<<grid, threads, smem, st>>>(m, ROT_ONLY ? q : q + r0 * (int64_t)K, ROT_ONLY ? scale : scale + r0, mc, K,
                                      box_rows, boxes, err, ROT_ONLY ? ybf + r0 * (int64_t)K : nullptr, ma);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_quant_rows(const void* x, int kind, int8_t* q, float* scale, int64_t M, int64_t K, int order,
                              int* err, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  if (order < 0 || (order == 0 && (K % 256 != 0 || K / 256 > 64))) {
    if (kind == 0) quant_rows_plain_kernel<float><<<(unsigned)M, 256, 0, st>>>((const float*)x, q, scale, (int)K);
    else if (kind == 1) quant_rows_plain_kernel<__half><<<(unsigned)M, 256, 0, st>>>((const __half*)x, q, scale, (int)K);
    else quant_rows_plain_kernel<__nv_bfloat16><<<(unsigned)M, 256, 0, st>>>((const __nv_bfloat16*)x, q, scale, (int)K);
    return cudaGetLastError();
  }
  if (K == 0) {
    // an empty row: scale = max(0/127, 1e-30), no codes (the reference's kernels write exactly this)
    fill_f32(scale, 1e-30f, M, st);
    return cudaGetLastError();
  }
#define H3Q_Q(O)                                                                        \
  if (kind == 0) return launch_rows<O, float>(x, q, scale, M, (int)K, err, st);          \
  if (kind == 1) return launch_rows<O, __half>(x, q, scale, M, (int)K, err, st);         \
  return launch_rows<O, __nv_bfloat16>(x, q, scale, M, (int)K, err, st);
  if (order == 2) { H3Q_Q(2) }
  if (order == 1) { H3Q_Q(1) }
  H3Q_Q(0)
#undef H3Q_Q
}

cudaError_t launch_rotate_bf16(const uint16_t* x, uint16_t* y, int64_t M, int64_t K, int* err, cudaStream_t st) {
  if (M == 0 || K == 0) return cudaSuccess;
  return launch_rows<2, __nv_bfloat16, true>(x, nullptr, nullptr, M, (int)K, err, st, y);
}

// rms_modulate followed by the quantizer quant_rows_raw would pick for the modulated bf16 row (rot2 order for
// K / 256 <= 56, rot order beyond), or rms_modulate alone (codes == nullptr: the bf16 row goes to y).
cudaError_t launch_rms_modulate(const uint16_t* x, const uint16_t* w, float eps, const float* scale_tab,
                                const float* shift_tab, const uint32_t* idx, int8_t* codes, float* row_scale,
                                uint16_t* y, int64_t M, int64_t K, int* err, cudaStream_t st) {
  if (M == 0 || K == 0) return cudaSuccess;
  ModArgs ma{w, scale_tab, shift_tab, idx, eps};
  if (!codes) return launch_rows<0, __nv_bfloat16, true, true>(x, nullptr, nullptr, M, (int)K, err, st, y, &ma);
  if (K / 256 <= 56)
    return launch_rows<2, __nv_bfloat16, false, true>(x, codes, row_scale, M, (int)K, err, st, nullptr, &ma);
  return launch_rows<1, __nv_bfloat16, false, true>(x, codes, row_scale, M, (int)K, err, st, nullptr, &ma);
}

__global__ void fill_f32_kernel(float* p, float v, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}

void fill_f32(float* p, float v, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  int64_t b = (n + 255) / 256;
  fill_f32_kernel<<<(unsigned)(b < 4096 ? b : 4096), 256, 0, st>>>(p, v, n);
}

}  // namespace h3q
