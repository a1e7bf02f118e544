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
#include <cstdint>
#include <cuda_bf16.h>
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

// One in-register radix-4 stage over the 4 values a[b], a[b+st], a[b+2st], a[b+3st].
template <int ORDER>
__device__ __forceinline__ void h4_inreg(float& a0, float& a1, float& a2, float& a3, bool first) {
  if (ORDER == 2) {
    float s = first ? __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3) : __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    float b0 = __fsub_rn(s, __fmul_rn(2.f, a3)), b1 = __fsub_rn(s, __fmul_rn(2.f, a2));
    float b2 = __fsub_rn(s, __fmul_rn(2.f, a1)), b3 = __fsub_rn(s, __fmul_rn(2.f, a0));
    a0 = b0; a1 = b1; a2 = b2; a3 = b3;
  } else {
    float b0 = __fsub_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
    float b1 = __fadd_rn(__fsub_rn(__fadd_rn(a0, a1), a2), a3);
    float b2 = __fadd_rn(__fadd_rn(__fsub_rn(a0, a1), a2), a3);
    float b3 = __fadd_rn(__fadd_rn(__fsub_rn(a1, a0), a2), a3);
    a0 = b0; a1 = b1; a2 = b2; a3 = b3;
  }
}

// Digit 3: lane j of a quad holds a_j; returns out_j.
template <int ORDER>
__device__ __forceinline__ float h4_quad(float a, int j) {
  if (ORDER == 2) {
    float s1 = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
    float s = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 2));
    float p = __shfl_xor_sync(0xffffffffu, a, 3);
    return __fsub_rn(s, __fmul_rn(2.f, p));
  } else {
    float x1 = __shfl_xor_sync(0xffffffffu, a, 1);
    float x2 = __shfl_xor_sync(0xffffffffu, a, 2);
    float x3 = __shfl_xor_sync(0xffffffffu, a, 3);
    // ((P + Q) + R) + S reproduces each lane's left-to-right formula exactly (x+y == y+x, x-y == x+(-y)).
    float P = j < 2 ? a : x2;
    float Q = j < 2 ? x1 : -x3;
    float R = j == 0 ? x2 : (j == 1 ? -x3 : (j == 2 ? a : x1));
    float S = j == 0 ? -x3 : (j == 1 ? x2 : (j == 2 ? x1 : a));
    return __fadd_rn(__fadd_rn(__fadd_rn(P, Q), R), S);
  }
}

// int8 code of t = v * inv: nearest-even integer through t + 1.5*2^23 (exact for |t| < 2^22; |t| <= 127 here
// by construction of inv), NaN -> 0 (order 2) or -128 (orders 0/1).
template <int ORDER>
__device__ __forceinline__ uint32_t code_of(float t) {
  const float r = __fadd_rn(t, 12582912.0f);
  uint32_t b = (uint32_t)(__float_as_int(r) - 0x4B400000) & 0xffu;
  if (t != t) b = ORDER == 2 ? 0u : 0x80u;
  return b;
}

template <int ORDER, typename Tin>
__global__ void __launch_bounds__(256, 2) quant_rows_kernel(const Tin* __restrict__ x, int8_t* __restrict__ q,
                                                          float* __restrict__ scale, int64_t M, int K, int tpr,
                                                          int rows_per_block) {
  __shared__ unsigned s_max[32];
  const int G = K >> 8;
  const int rl = threadIdx.x / tpr, t = threadIdx.x % tpr;
  const int64_t row = (int64_t)blockIdx.x * rows_per_block + rl;
  const bool active = (row < M) && (t < 4 * G);
  const int g = t >> 2, j = t & 3;
  if (threadIdx.x < 32) s_max[threadIdx.x] = 0u;

  constexpr int V = In<Tin>::kVec;
  float v[64];
  if (active) {
    const uint4* src = reinterpret_cast<const uint4*>(x + row * (int64_t)K + g * 256 + j * 64);
    uint4 raw[64 / V];
#pragma unroll
    for (int i = 0; i < 64 / V; ++i) raw[i] = __ldg(src + i);
#pragma unroll
    for (int i = 0; i < 64 / V; ++i) In<Tin>::cvt(raw[i], v + i * V);
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = 0.f;
  }

  if (ORDER != 0) {
    // digits 0, 1, 2 in registers (element c of the thread has digits c&3, (c>>2)&3, (c>>4)&3)
#pragma unroll
    for (int d = 0, st = 1; d < 3; ++d, st *= 4) {
#pragma unroll
      for (int b = 0; b < 64; ++b) {
        if ((b / st) % 4 != 0) continue;
        h4_inreg<ORDER>(v[b], v[b + st], v[b + 2 * st], v[b + 3 * st], d == 0);
      }
    }
    // digit 3 across the quad, then the 1/16 normalisation
#pragma unroll
    for (int c = 0; c < 64; ++c) v[c] = __fmul_rn(h4_quad<ORDER>(v[c], j), 0.0625f);
  }

  float m = 0.f;
#pragma unroll
  for (int c = 0; c < 64; ++c) m = fmaxf(m, fabsf(v[c]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) atomicMax(&s_max[rl], __float_as_uint(m));
  __syncthreads();
  const float mx = __uint_as_float(s_max[rl]);
  const float s = fmaxf(__fdiv_rn(mx, 127.f), 1e-30f);
  const float inv = __fdiv_rn(1.f, s);
  if (!active) return;
  if (t == 0) scale[row] = s;
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    w[i] = code_of<ORDER>(__fmul_rn(v[4 * i], inv)) | (code_of<ORDER>(__fmul_rn(v[4 * i + 1], inv)) << 8) |
           (code_of<ORDER>(__fmul_rn(v[4 * i + 2], inv)) << 16) | (code_of<ORDER>(__fmul_rn(v[4 * i + 3], inv)) << 24);
  }
  uint4* dst = reinterpret_cast<uint4*>(q + row * (int64_t)K + g * 256 + j * 64);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
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

template <int ORDER, typename Tin>
static cudaError_t launch_rows(const void* x, int8_t* q, float* scale, int64_t M, int K, cudaStream_t st) {
  const int G = K / 256;
  const int tpr = ((4 * G + 31) / 32) * 32;
  int rpb = 1;
  while (rpb * 2 * tpr <= 256 && rpb * 2 <= 32) rpb *= 2;
  const int64_t blocks = (M + rpb - 1) / rpb;
  quant_rows_kernel<ORDER, Tin><<<(unsigned)blocks, tpr * rpb, 0, st>>>(static_cast<const Tin*>(x), q, scale, M, K,
                                                                        tpr, rpb);
  return cudaGetLastError();
}

cudaError_t launch_quant_rows(const void* x, int kind, int8_t* q, float* scale, int64_t M, int64_t K, int order,
                              cudaStream_t st) {
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
  if (kind == 0) return launch_rows<O, float>(x, q, scale, M, (int)K, st);               \
  if (kind == 1) return launch_rows<O, __half>(x, q, scale, M, (int)K, st);              \
  return launch_rows<O, __nv_bfloat16>(x, q, scale, M, (int)K, st);
  if (order == 2) { H3Q_Q(2) }
  if (order == 1) { H3Q_Q(1) }
  H3Q_Q(0)
#undef H3Q_Q
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
