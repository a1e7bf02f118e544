// elementwise.cu -- weight decode and gated-residual kernels of the path (HBM-bound, grid-stride, 16-byte IO).
//   dequant_i8    kernels.rs:40-49      out = q * scale[row or 0]
//   dequant_nvfp4 kernels.rs:65-81      out = E2M1[nibble] * e4m3(block scale, 128x4 swizzle) * global
//   gate_add      kernels.rs:418-428    out = x + y * round_to_kind(gate[idx[s], c])
#include <cstdint>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "h3q_internal.h"

namespace h3q {

__device__ __forceinline__ void st_kind(void* out, int kind, int64_t i, float v) {
  if (kind == 0) reinterpret_cast<float*>(out)[i] = v;
  else if (kind == 1) reinterpret_cast<uint16_t*>(out)[i] = f2h(v);
  else reinterpret_cast<uint16_t*>(out)[i] = (uint16_t)f2bf(v);
}
__device__ __forceinline__ float ld_kind(const void* p, int kind, int64_t i) {
  if (kind == 0) return reinterpret_cast<const float*>(p)[i];
  if (kind == 1) return h2f(reinterpret_cast<const uint16_t*>(p)[i]);
  return bf2f(reinterpret_cast<const uint16_t*>(p)[i]);
}

// 16 codes per thread-iteration when cols % 16 == 0 (one 16-byte load, 16..64-byte store)
__global__ void dequant_i8_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale, int per_row,
                                  void* __restrict__ out, int kind, int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (cols % 16 == 0) {
    const int64_t nv = n / 16;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv; v += stride) {
      const int64_t i = v * 16, r = i / cols;
      const float s = per_row ? __ldg(scale + r) : __ldg(scale);
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(q) + v);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
      float f[16];
#pragma unroll
      for (int b = 0; b < 16; ++b) f[b] = __fmul_rn((float)(int8_t)((w[b >> 2] >> (8 * (b & 3))) & 0xffu), s);
      if (kind == 0) {
        float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + i);
#pragma unroll
        for (int b = 0; b < 4; ++b) d[b] = make_float4(f[4 * b], f[4 * b + 1], f[4 * b + 2], f[4 * b + 3]);
      } else {
        uint32_t o[8];
#pragma unroll
        for (int b = 0; b < 8; ++b)
          o[b] = kind == 2 ? pack_bf2(f[2 * b], f[2 * b + 1])
                           : ((uint32_t)f2h(f[2 * b]) | ((uint32_t)f2h(f[2 * b + 1]) << 16));
        uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + i);
        d[0] = make_uint4(o[0], o[1], o[2], o[3]);
        d[1] = make_uint4(o[4], o[5], o[6], o[7]);
      }
    }
    return;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t r = i / cols;
    st_kind(out, kind, i, __fmul_rn((float)q[i], per_row ? scale[r] : scale[0]));
  }
}

__device__ __forceinline__ float fp8e4m3(uint32_t v) {
  const int sgn = (v >> 7) & 1, e = (v >> 3) & 15, m = v & 7;
  float r;
  if (e == 0) r = ldexpf((float)m / 8.0f, -6);
  else if (e == 15 && m == 7) r = __int_as_float(0x7fc00000);
  else r = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return sgn ? -r : r;
}

__constant__ float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

// One thread per 16-element block (8 packed bytes, one scale byte).
__global__ void dequant_nvfp4_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ bs,
                                     const float* __restrict__ gscale, void* __restrict__ out, int kind, int64_t rows,
                                     int64_t k) {
  const float g = __ldg(gscale);
  const int64_t nb = k / 16, ncb = (nb + 3) / 4;
  const int64_t nblocks = rows * nb;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nblocks; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nb, b = i % nb;
    const int64_t rb = r / 128, rin = r % 128, cb = b / 4, cin = b % 4;
    const int64_t off = (rb * ncb + cb) * 512 + (rin % 32) * 16 + (rin / 32) * 4 + cin;
    const float s = fp8e4m3(bs[off]);
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(q + r * (k / 2) + b * 8));
    const uint32_t w[2] = {raw.x, raw.y};
    float f[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const uint32_t byte = (w[e >> 3] >> (8 * ((e >> 1) & 3))) & 0xffu;
      const uint32_t nib = (e & 1) ? (byte & 15u) : (byte >> 4);
      f[e] = __fmul_rn(__fmul_rn(kE2M1[nib], s), g);
    }
    const int64_t o = r * k + b * 16;
    if (kind == 0) {
      float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + o);
#pragma unroll
      for (int e = 0; e < 4; ++e) d[e] = make_float4(f[4 * e], f[4 * e + 1], f[4 * e + 2], f[4 * e + 3]);
    } else {
      uint32_t p[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        p[e] = kind == 2 ? pack_bf2(f[2 * e], f[2 * e + 1]) : ((uint32_t)f2h(f[2 * e]) | ((uint32_t)f2h(f[2 * e + 1]) << 16));
      uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + o);
      d[0] = make_uint4(p[0], p[1], p[2], p[3]);
      d[1] = make_uint4(p[4], p[5], p[6], p[7]);
    }
  }
}

__global__ void gate_add_kernel(const void* __restrict__ x, const void* __restrict__ y, int kind,
                                const float* __restrict__ gate, const uint32_t* __restrict__ idx, void* __restrict__ out,
                                int64_t S, int64_t C) {
  const int64_t n = S * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i / C, c = i % C;
    float g = gate[(int64_t)idx[s] * C + c];
    g = kind == 1 ? h2f(f2h(g)) : bf16r(g);
    st_kind(out, kind, i, __fmaf_rn(ld_kind(y, kind, i), g, ld_kind(x, kind, i)));
  }
}

// silu(g) * u over interleaved (g, u) pairs or split halves; silu and the product are each rounded to the
// tensor kind, as the reference's candle ops on bf16 / f16 tensors round every op (weights.rs:806-816, ops.rs:39-44)
__global__ void swiglu_kernel(const void* __restrict__ y, void* __restrict__ out, int kind, int64_t rows, int64_t F,
                              int interleaved) {
  const int64_t n = rows * F;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / F, j = i % F;
    const int64_t gi = interleaved ? r * 2 * F + 2 * j : r * 2 * F + j;
    const int64_t ui = interleaved ? gi + 1 : gi + F;
    const float g = ld_kind(y, kind, gi), u = ld_kind(y, kind, ui);
    float s = __fdiv_rn(g, __fadd_rn(1.f, __expf(-g)));
    if (kind == 2) s = bf16r(s);
    else if (kind == 1) s = h2f(f2h(s));
    st_kind(out, kind, i, __fmul_rn(s, u));
  }
}

static unsigned grid_for(int64_t work) {
  int64_t b = (work + 255) / 256;
  const int64_t cap = (int64_t)sm_count(0) * 16;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

cudaError_t launch_dequant_i8(const int8_t* q, const float* scale, int per_row, void* out, int kind, int64_t rows,
                              int64_t cols, cudaStream_t st) {
  if (rows * cols == 0) return cudaSuccess;
  dequant_i8_kernel<<<grid_for(cols % 16 == 0 ? rows * cols / 16 : rows * cols), 256, 0, st>>>(q, scale, per_row, out,
                                                                                             kind, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_dequant_nvfp4(const uint8_t* q, const uint8_t* bs, const float* g, void* out, int kind,
                                 int64_t rows, int64_t k, cudaStream_t st) {
  if (rows * k == 0) return cudaSuccess;
  dequant_nvfp4_kernel<<<grid_for(rows * (k / 16)), 256, 0, st>>>(q, bs, g, out, kind, rows, k);
  return cudaGetLastError();
}

cudaError_t launch_gate_add(const void* x, const void* y, int kind, const float* gate, const uint32_t* idx, void* out,
                            int64_t S, int64_t C, cudaStream_t st) {
  if (S * C == 0) return cudaSuccess;
  gate_add_kernel<<<grid_for(S * C), 256, 0, st>>>(x, y, kind, gate, idx, out, S, C);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const void* y, void* out, int kind, int64_t rows, int64_t F, int interleaved, cudaStream_t st) {
  if (rows * F == 0) return cudaSuccess;
  swiglu_kernel<<<grid_for(rows * F), 256, 0, st>>>(y, out, kind, rows, F, interleaved);
  return cudaGetLastError();
}

}  // namespace h3q
