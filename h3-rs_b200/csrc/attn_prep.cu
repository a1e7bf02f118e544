// attn_prep.cu -- the front end of the int8 attention (attn8.rs:45-93, :395-486): K column mean, per-head
// int8 quantisation of Q and K, and the V relayout the P.V tensor-core product reads.
//
//   kmean       ColMean + `/ S` (attn8.rs:45-52, :429-455, :622): column sums of K [S, H*128] in a FIXED order
//               (row chunks of ceil(S / min(128, S)) rows summed sequentially, chunk sums added in chunk order),
//               then times (float)(1 / S).  The reference adds the chunk sums with atomicAdd in whatever order the
//               blocks finish; this is that computation with the order pinned, so K codes are reproducible.
//   quant_heads QuantHeads (attn8.rs:69-93): v = x - mean, sc = fmaxf(max|v| / 127, 1e-20), q = clamp(rn(v / sc),
//               -127, 127), per (token, head) row; or per 128-token block of one head (block mode).
//   v_layout    VToF16 (attn8.rs:55-65) with a transposed output: [S, H, 128] (row stride, column offset) ->
//               [H, 128, Sp] f16 (or bf16), so V is a K-major operand of the P.V MMA.
//
// Layouts: codes [H, S, 128] int8; scales [H, Sp] f32 with Sp = roundup(S, 128) (block mode: every token of a
// block holds the block's scale; entries S..Sp-1 are zero).
#include <cstdint>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "h3q_internal.h"

namespace h3q {

namespace {
constexpr int HD = 128;

__device__ __forceinline__ void bf8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// quant_heads' rounding: __float2int_rn (NaN -> 0), clamp to [-127, 127]
__device__ __forceinline__ uint32_t q127(float v, float inv) {
  int q = __float2int_rn(v * inv);
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  return (uint32_t)(q & 0xff);
}
}  // namespace

// Row-chunk partition of the column sums (the reference's ColMean launch, attn8.rs:446-450).
void kmean_partition(int64_t S, int& parts, int& rows_per) {
  const int64_t p = S < 128 ? S : 128;
  rows_per = (int)((S + p - 1) / p);
  parts = (int)((S + rows_per - 1) / rows_per);
}

// part[p, c] = sum of x[r, c] over the rows of chunk p, in row order; 8 columns per thread.
__global__ void kmean_partial_kernel(const uint16_t* __restrict__ x, float* __restrict__ part, int64_t S, int C,
                                     int rows_per) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 * 8 >= C) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < S ? r0 + rows_per : S;
  const int64_t stride = C / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x) + r0 * stride + c8;
  float s[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) s[i] = 0.f;
  int64_t r = r0;
  for (; r + 4 <= r1; r += 4, src += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldg(src + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float f[8];
      bf8_to_f32(v[u], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i] = __fadd_rn(s[i], f[i]);
    }
  }
  for (; r < r1; ++r, src += stride) {
    float f[8];
    bf8_to_f32(__ldg(src), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = __fadd_rn(s[i], f[i]);
  }
  float4* dst = reinterpret_cast<float4*>(part + (int64_t)blockIdx.y * C + c8 * 8);
  dst[0] = make_float4(s[0], s[1], s[2], s[3]);
  dst[1] = make_float4(s[4], s[5], s[6], s[7]);
}

// mean[c] = (chunk sums added in chunk order) * inv_s
__global__ void kmean_final_kernel(const float* __restrict__ part, int parts, float* __restrict__ mean, int C,
                                   float inv_s) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float a = 0.f;
  for (int p = 0; p < parts; ++p) a = __fadd_rn(a, __ldg(part + (int64_t)p * C + c));
  mean[c] = __fmul_rn(a, inv_s);
}

// Per-token quantisation: 16 threads per (token, head) row, 8 dims each.  Rows are visited in input order
// (s * H + h); codes go to [H, S, 128], scales to [H, Sp].
__global__ void quant_heads_token_kernel(const uint16_t* __restrict__ x, const float* __restrict__ mean,
                                         int8_t* __restrict__ codes, float* __restrict__ scales, int64_t S, int H,
                                         int64_t Sp) {
  const int64_t rows = S * H;
  const int sub = threadIdx.x & 15;
  const uint32_t gmask = (threadIdx.x & 16) ? 0xffff0000u : 0x0000ffffu;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 4) {
    const int64_t s = row / H;
    const int h = (int)(row - s * H);
    float v[8];
    bf8_to_f32(__ldg(reinterpret_cast<const uint4*>(x + row * HD) + sub), v);
    if (mean) {
      const float4* mp = reinterpret_cast<const float4*>(mean + h * HD + sub * 8);
      const float4 m0 = __ldg(mp), m1 = __ldg(mp + 1);
      const float mm[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fsub_rn(v[i], mm[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fsub_rn(v[i], 0.f);
    }
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(gmask, m, o));
    const float sc = fmaxf(__fdiv_rn(m, 127.f), 1e-20f);
    const float inv = __fdiv_rn(1.f, sc);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo |= q127(v[i], inv) << (8 * i);
      hi |= q127(v[4 + i], inv) << (8 * i);
    }
    *reinterpret_cast<uint2*>(codes + ((int64_t)h * S + s) * HD + sub * 8) = make_uint2(lo, hi);
    if (sub == 0) scales[(int64_t)h * Sp + s] = sc;
  }
}

// Per-128-token-block quantisation: one CTA of 256 threads per (block, head); thread t covers token t / 2 of the
// block, dims (t & 1) * 64 .. +63.
__global__ void __launch_bounds__(256) quant_heads_block_kernel(const uint16_t* __restrict__ x,
                                                                const float* __restrict__ mean,
                                                                int8_t* __restrict__ codes,
                                                                float* __restrict__ scales, int64_t S, int H,
                                                                int64_t Sp) {
  __shared__ float red[8];
  const int h = blockIdx.y;
  const int64_t s = (int64_t)blockIdx.x * 128 + (threadIdx.x >> 1);
  const int half = threadIdx.x & 1;
  const bool valid = s < S;
  float v[64];
  float m = 0.f;
  if (valid) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (s * H + h) * HD + half * 64);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float f[8];
      bf8_to_f32(__ldg(src + c), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float mv = mean ? __ldg(mean + h * HD + half * 64 + c * 8 + i) : 0.f;
        v[c * 8 + i] = __fsub_rn(f[i], mv);
        m = fmaxf(m, fabsf(v[c * 8 + i]));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  const float sc = fmaxf(__fdiv_rn(m, 127.f), 1e-20f);
  const float inv = __fdiv_rn(1.f, sc);
  if (valid) {
    uint4* dst = reinterpret_cast<uint4*>(codes + ((int64_t)h * S + s) * HD + half * 64);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t p = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) p |= q127(v[c * 16 + k * 4 + i], inv) << (8 * i);
        w[k] = p;
      }
      dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (half == 0) scales[(int64_t)h * Sp + s] = sc;
  }
}

// [S, H, 128] 16-bit rows (element stride `rs` between tokens, head h at column col + 128 h) -> [H, 128, Sp],
// converted bf16 -> f16 (cvt.rn, as v_to_f16) unless `keep_bf16`.  One CTA per (64-token chunk, head).
template <bool VEC>
__global__ void __launch_bounds__(256) v_layout_kernel(const uint16_t* __restrict__ x, int64_t rs, int64_t col,
                                                       uint16_t* __restrict__ vt, int64_t S, int64_t Sp,
                                                       int keep_bf16) {
  __shared__ uint16_t tile[HD][64 + 8];
  const int h = blockIdx.y;
  const int64_t s0 = (int64_t)blockIdx.x * 64;
  const int t = threadIdx.x;
  {
    const int tok = t & 63, q = t >> 6;  // token of the chunk, quarter of the 128 dims
    const int64_t s = s0 + tok;
    uint32_t w[16];
    if (s < S) {
      const uint16_t* src = x + s * rs + col + (int64_t)h * HD + q * 32;
      if (VEC) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(src) + c);
          w[4 * c] = u.x; w[4 * c + 1] = u.y; w[4 * c + 2] = u.z; w[4 * c + 3] = u.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = (uint32_t)src[2 * i] | ((uint32_t)src[2 * i + 1] << 16);
      }
      if (!keep_bf16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a = __uint_as_float(w[i] << 16), b = __uint_as_float(w[i] & 0xffff0000u);
          uint32_t r;
          asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
          w[i] = r;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = 0u;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      tile[q * 32 + 2 * i][tok] = (uint16_t)(w[i] & 0xffffu);
      tile[q * 32 + 2 * i + 1][tok] = (uint16_t)(w[i] >> 16);
    }
  }
  __syncthreads();
  {
    const int d = t >> 1, hf = t & 1;  // output row (dim), half of the 64 tokens
    uint16_t* dst = vt + ((int64_t)h * HD + d) * Sp + s0 + hf * 32;
    const uint32_t* srow = reinterpret_cast<const uint32_t*>(&tile[d][hf * 32]);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      reinterpret_cast<uint4*>(dst)[c] = make_uint4(srow[4 * c], srow[4 * c + 1], srow[4 * c + 2], srow[4 * c + 3]);
  }
}

// ------------------------------------------------------------------------------------------------ launchers

size_t kmean_workspace_bytes(int64_t S, int64_t H) {
  if (S <= 0 || H <= 0) return 0;
  int parts, rows_per;
  kmean_partition(S, parts, rows_per);
  return (size_t)parts * (size_t)H * HD * sizeof(float);
}

cudaError_t launch_kmean(const uint16_t* k, int64_t S, int64_t H, float* mean, float* part, cudaStream_t st) {
  if (S <= 0 || H <= 0) return cudaSuccess;
  int parts, rows_per;
  kmean_partition(S, parts, rows_per);
  const int C = (int)(H * HD);
  const int cg = C / 8;
  kmean_partial_kernel<<<dim3((cg + 127) / 128, parts), 128, 0, st>>>(k, part, S, C, rows_per);
  const float inv_s = (float)(1.0 / (double)S);
  kmean_final_kernel<<<(C + 255) / 256, 256, 0, st>>>(part, parts, mean, C, inv_s);
  return cudaGetLastError();
}

cudaError_t launch_quant_heads(const uint16_t* x, const float* mean, int8_t* codes, float* scales, int64_t S,
                               int64_t H, bool block128, cudaStream_t st) {
  if (S <= 0 || H <= 0) return cudaSuccess;
  const int64_t Sp = (S + 127) / 128 * 128;
  cudaError_t e = cudaMemsetAsync(scales, 0, (size_t)H * Sp * sizeof(float), st);
  if (e != cudaSuccess) return e;
  if (block128) {
    quant_heads_block_kernel<<<dim3((unsigned)(Sp / 128), (unsigned)H), 256, 0, st>>>(x, mean, codes, scales, S,
                                                                                     (int)H, Sp);
  } else {
    const int64_t rows = S * H;
    int64_t blocks = (rows * 16 + 255) / 256;
    const int64_t cap = (int64_t)sm_count(0) * 32;
    if (blocks > cap) blocks = cap;
    quant_heads_token_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, mean, codes, scales, S, (int)H, Sp);
  }
  return cudaGetLastError();
}

cudaError_t launch_v_layout(const uint16_t* x, int64_t rs, int64_t col, uint16_t* vt, int64_t S, int64_t H,
                            bool keep_bf16, cudaStream_t st) {
  if (S <= 0 || H <= 0) return cudaSuccess;
  const int64_t Sp = (S + 127) / 128 * 128;
  const dim3 grid((unsigned)(Sp / 64), (unsigned)H);
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && rs % 8 == 0 && col % 8 == 0;
  if (vec) v_layout_kernel<true><<<grid, 256, 0, st>>>(x, rs, col, vt, S, Sp, keep_bf16 ? 1 : 0);
  else v_layout_kernel<false><<<grid, 256, 0, st>>>(x, rs, col, vt, S, Sp, keep_bf16 ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace h3q
