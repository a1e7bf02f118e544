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
//   qk_norm_rope  (kernels.rs:86-126) per-head RMSNorm + split-half RoPE, standalone, and fused into the K mean and
//               the Q / K quantisation for the DiT's attention step (dit.rs:741-757), so the normalised q and k
//               never reach memory.
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

// ------------------------------------------------------------------------------- q/k RMSNorm + split-half RoPE
//
// qk_norm_rope (kernels.rs:86-126) per (token, head) row of D <= 256 dims, bf16 in and out:
//   ss   = sum of v_d^2 in the reference's order: 32-lane xor trees (levels 16 .. 1) inside each 32-dim slice,
//          then an xor tree over the slice sums (lane 0's view: ((t0 + t4) + (t2 + t6)) + ((t1 + t5) + (t3 + t7)),
//          absent slices zero); squares of bf16 values are exact in f32, so no contraction question arises.
//   v    = (v * rsqrtf(ss / D + eps)) * w_d                                   (when normalising)
//   o    = fma(v_d, cos, -(v_{d+half} * sin))  for d < half,
//          fma(v_d, cos,   v_{d-half} * sin)   for half <= d < rot,           (cos, sin = table[s, d mod half])
//          v_d otherwise;  the reference's compiled kernel rounds the second product and fuses the first (measured
//          against it: every other association differs in about 1e-5 of the outputs).
//   out  = bf16(o), nearest even, NaN -> 0x7fc0 (the reference's f2bf).
namespace {

__device__ __forceinline__ uint16_t f2bf_ref(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

__device__ __forceinline__ float rope_lo(float v, float c, float partner, float sn) {
  return __fmaf_rn(v, c, -__fmul_rn(partner, sn));
}
__device__ __forceinline__ float rope_hi(float v, float c, float partner, float sn) {
  return __fmaf_rn(v, c, __fmul_rn(partner, sn));
}

// The general form: one warp per row, lane l holding dims 32 i + l (the reference's thread d sits in slice d / 32 at
// lane d % 32); partners of the rotation through a per-warp row buffer.
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const uint16_t* __restrict__ x, int64_t rs, int64_t col,
                                                           int64_t hs, const uint16_t* __restrict__ w, int do_norm,
                                                           float eps, const float* __restrict__ cs, int rot,
                                                           uint16_t* __restrict__ out, int64_t S, int H, int D) {
  __shared__ float buf[8][256];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int NS = (D + 31) >> 5, half = rot >> 1;
  const int64_t rows = S * H;
  for (int64_t row = (int64_t)blockIdx.x * 8 + wp; row < rows; row += (int64_t)gridDim.x * 8) {
    const int64_t s = row / H;
    const int h = (int)(row - s * H);
    const uint16_t* xr = x + s * rs + col + (int64_t)h * hs;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = 32 * i + lane;
      v[i] = (i < NS && d < D) ? bf2f(__ldg(xr + d)) : 0.f;
    }
    if (do_norm) {
      float t[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float a = __fmul_rn(v[i], v[i]);
        if (i < NS) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        }
        t[i] = a;
      }
      const float ss = __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[4]), __fadd_rn(t[2], t[6])),
                                 __fadd_rn(__fadd_rn(t[1], t[5]), __fadd_rn(t[3], t[7])));
      const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int d = 32 * i + lane;
        if (i < NS) v[i] = __fmul_rn(__fmul_rn(v[i], inv), (w && d < D) ? bf2f(__ldg(w + d)) : 1.f);
      }
    }
    if (half > 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < NS) buf[wp][32 * i + lane] = v[i];
      __syncwarp();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = 32 * i + lane;
      if (i >= NS || d >= D) continue;
      float o = v[i];
      if (d < rot) {
        const int j = d < half ? d : d - half;
        const float c = __ldg(cs + s * half + j), sn = __ldg(cs + (S + s) * half + j);
        o = d < half ? rope_lo(v[i], c, buf[wp][d + half], sn) : rope_hi(v[i], c, buf[wp][d - half], sn);
      }
      out[row * D + d] = f2bf_ref(o);
    }
    if (half > 0) __syncwarp();  // the row buffer is rewritten by the next row
  }
}

// The D = 128 forms.  Slice layout: lane 4r + w of a warp holds dims 32w .. 32w+31 of row r (r < 8) -- exactly the
// 32 values the reference's warp w reduces, so its 32-lane xor tree runs inside the thread (level 16 pairs dims j
// and j + 16, ...) and the four slice sums meet over lanes xor 2 then xor 1.  The rotation reads partners from a
// per-warp row buffer of 8 x 128 f32 whose 16-byte chunks are swizzled by the writing lane (conflict-free).
constexpr int kRowsPerWarp = 8;

__device__ __forceinline__ int buf_off(int ls, int chunk) { return 32 * ls + 4 * (chunk ^ (ls & 7)); }

__device__ __forceinline__ void load_slice(const uint16_t* __restrict__ p, uint32_t (&raw)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + c);
    raw[4 * c] = u.x;
    raw[4 * c + 1] = u.y;
    raw[4 * c + 2] = u.z;
    raw[4 * c + 3] = u.w;
  }
}

__device__ __forceinline__ float lo16(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float hi16(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float elem(const uint32_t (&p)[16], int i) { return (i & 1) ? hi16(p[i >> 1]) : lo16(p[i >> 1]); }

// bf16x2 of (a, b), a in the low half: nearest even with the reference's f2bf NaN pattern 0x7fc0 (cvt.rn agrees
// with f2bf on every other input).
__device__ __forceinline__ uint32_t pack_bf16_ref(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  if ((r & 0x7fffu) > 0x7f80u) r = (r & 0xffff0000u) | 0x7fc0u;
  if ((r & 0x7fff0000u) > 0x7f800000u) r = (r & 0xffffu) | 0x7fc00000u;
  return r;
}

// qk_norm_rope of the thread's slice of row (token s): packed bf16 in (raw) -> the reference's packed bf16 q / k
// values out (res).  `w` points at the slice's 32 norm weights (or is NULL); half % 4 == 0.  Every lane of the warp
// takes part (shuffles, the row buffer).  Values stream through in 4-dim chunks, so only the packed slices stay live.
__device__ __forceinline__ void slice_norm_rope(const uint32_t (&raw)[16], uint32_t (&res)[16], int lane,
                                                const uint16_t* __restrict__ w, int do_norm, float eps,
                                                const float* __restrict__ cs, int half, int64_t s, int64_t S,
                                                float* buf) {
  const int sl = lane & 3;
  float inv = 1.f;
  if (do_norm) {
    float a[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float x0 = elem(raw, i), x1 = elem(raw, i + 16);
      a[i] = __fadd_rn(__fmul_rn(x0, x0), __fmul_rn(x1, x1));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < o; ++i) a[i] = __fadd_rn(a[i], a[i + o]);
    float t = __fadd_rn(a[0], __shfl_xor_sync(0xffffffffu, a[0], 2));
    t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
    inv = rsqrtf(__fadd_rn(__fdiv_rn(t, 128.f), eps));
  }
  // normalised chunk c: (x * inv) * w
  auto norm4 = [&](int c, float (&n)[4]) {
    float wv[4] = {1.f, 1.f, 1.f, 1.f};
    if (do_norm && w) {
      const uint2 wr = __ldg(reinterpret_cast<const uint2*>(w) + c);
      wv[0] = lo16(wr.x); wv[1] = hi16(wr.x); wv[2] = lo16(wr.y); wv[3] = hi16(wr.y);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x = elem(raw, 4 * c + i);
      n[i] = do_norm ? __fmul_rn(__fmul_rn(x, inv), wv[i]) : x;
    }
  };
  if (half > 0) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float n[4];
      norm4(c, n);
      *reinterpret_cast<float4*>(buf + buf_off(lane, c)) = make_float4(n[0], n[1], n[2], n[3]);
    }
    __syncwarp();
    const int r4 = lane & ~3;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 own = *reinterpret_cast<const float4*>(buf + buf_off(lane, c));
      float v[4] = {own.x, own.y, own.z, own.w};
      const int d = 32 * sl + 4 * c;
      if (d < 2 * half) {
        const bool lo = d < half;
        const int p = lo ? d + half : d - half, ls = r4 + (p >> 5);
        const float4 pv = *reinterpret_cast<const float4*>(buf + buf_off(ls, (p & 31) >> 2));
        const int jj = lo ? d : d - half;
        const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs + s * half + jj));
        const float4 s4 = __ldg(reinterpret_cast<const float4*>(cs + (S + s) * half + jj));
        const float pp[4] = {pv.x, pv.y, pv.z, pv.w}, cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = lo ? rope_lo(v[i], cc[i], pp[i], ss[i]) : rope_hi(v[i], cc[i], pp[i], ss[i]);
      }
      res[2 * c] = pack_bf16_ref(v[0], v[1]);
      res[2 * c + 1] = pack_bf16_ref(v[2], v[3]);
    }
    __syncwarp();  // the buffer is rewritten next
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float n[4];
      norm4(c, n);
      res[2 * c] = pack_bf16_ref(n[0], n[1]);
      res[2 * c + 1] = pack_bf16_ref(n[2], n[3]);
    }
  }
}

// Standalone qk_norm_rope for D = 128, rot % 8 == 0 and 16-byte aligned rows: CTA of 8 warps = 64 tokens, looping
// over `hb` heads (the tokens' rope rows stay in L1); out = f2bf exactly (NaN -> 0x7fc0).
__global__ void __launch_bounds__(256) qk_norm_rope128_kernel(const uint16_t* __restrict__ x, int64_t rs, int64_t col,
                                                              int64_t hs, const uint16_t* __restrict__ w, int do_norm,
                                                              float eps, const float* __restrict__ cs, int half,
                                                              uint16_t* __restrict__ out, int64_t S, int H, int hb) {
  __shared__ __align__(16) float buf[8][kRowsPerWarp * 128];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5, sl = lane & 3;
  const int64_t s = (int64_t)blockIdx.x * 64 + wp * kRowsPerWarp + (lane >> 2);
  const bool valid = s < S;
  const int h1 = min(H, (int)(blockIdx.y + 1) * hb);
  for (int h = blockIdx.y * hb; h < h1; ++h) {
    uint32_t raw[16], res[16];
    if (valid) load_slice(x + s * rs + col + (int64_t)h * hs + 32 * sl, raw);
    else {
#pragma unroll
      for (int i = 0; i < 16; ++i) raw[i] = 0u;
    }
    slice_norm_rope(raw, res, lane, w ? w + 32 * sl : nullptr, do_norm, eps, cs, half, valid ? s : 0, S, buf[wp]);
    if (valid) {
      uint4* dst = reinterpret_cast<uint4*>(out + (s * H + h) * HD + 32 * sl);
#pragma unroll
      for (int c = 0; c < 4; ++c) dst[c] = make_uint4(res[4 * c], res[4 * c + 1], res[4 * c + 2], res[4 * c + 3]);
    }
  }
}

// K column sums of the normalised, rotated K rows, chunked as kmean_partial_kernel: warp = (chunk, head), 8 rows of
// the chunk at a time in the slice layout, then turned through the row buffer so lane l adds dims 4l .. 4l+3 of the
// 8 rows in row order.  part[p, h*128 + d].  CTA = 8 heads of one chunk (their rope rows are the same).
__global__ void __launch_bounds__(256) kmean_rope_partial_kernel(const uint16_t* __restrict__ x, int64_t rs,
                                                                 int64_t col, const uint16_t* __restrict__ w,
                                                                 int do_norm, float eps,
                                                                 const float* __restrict__ cs, int half,
                                                                 float* __restrict__ part, int64_t S, int H,
                                                                 int rows_per) {
  __shared__ __align__(16) float buf[8][kRowsPerWarp * 128];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5, sl = lane & 3;
  const int h = blockIdx.y * 8 + wp;
  if (h >= H) return;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per;
  const int64_t r1 = r0 + rows_per < S ? r0 + rows_per : S;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float* b = buf[wp];
  for (int64_t g = r0; g < r1; g += kRowsPerWarp) {
    const int64_t s = g + (lane >> 2);
    const bool valid = s < r1;
    uint32_t raw[16], res[16];
    if (valid) load_slice(x + s * rs + col + (int64_t)h * HD + 32 * sl, raw);
    else {
#pragma unroll
      for (int i = 0; i < 16; ++i) raw[i] = 0u;
    }
    slice_norm_rope(raw, res, lane, w ? w + 32 * sl : nullptr, do_norm, eps, cs, half, valid ? s : 0, S, b);
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(b + buf_off(lane, c)) =
          make_float4(lo16(res[2 * c]), hi16(res[2 * c]), lo16(res[2 * c + 1]), hi16(res[2 * c + 1]));
    __syncwarp();
    const int nr = (int)(r1 - g < kRowsPerWarp ? r1 - g : kRowsPerWarp);
    for (int r = 0; r < nr; ++r) {
      const int ls = 4 * r + (lane >> 3);
      const float4 f = *reinterpret_cast<const float4*>(b + buf_off(ls, lane & 7));
      acc[0] = __fadd_rn(acc[0], f.x);
      acc[1] = __fadd_rn(acc[1], f.y);
      acc[2] = __fadd_rn(acc[2], f.z);
      acc[3] = __fadd_rn(acc[3], f.w);
    }
    __syncwarp();
  }
  reinterpret_cast<float4*>(part + (int64_t)blockIdx.x * H * HD + (int64_t)h * HD)[lane] =
      make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// Normalise + rotate + (K: subtract the column mean) + quantise, as qk_norm_rope then quant_heads.  8 tokens per
// warp (slice layout); a CTA covers 64 tokens (per-token scales) or, with BLOCK, one 128-token scale block, and
// loops over `hb` heads.  Writes every scale entry of its tokens, zero past S.
template <bool BLOCK>
__global__ void __launch_bounds__(BLOCK ? 512 : 256, BLOCK ? 2 : 3) qk_rope_quant_kernel(const uint16_t* __restrict__ x, int64_t rs, int64_t col,
                                                            const uint16_t* __restrict__ w, int do_norm, float eps,
                                                            const float* __restrict__ cs, int half,
                                                            const float* __restrict__ mean,
                                                            int8_t* __restrict__ codes, float* __restrict__ scales,
                                                            int64_t S, int64_t Sp, int H, int hb) {
  extern __shared__ __align__(16) float qbuf[];  // warps x 8 x 128
  __shared__ float red[2][16];
  constexpr int TOK = BLOCK ? 128 : 64;  // tokens per CTA: the scale block, or 8 warps of 8
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5, sl = lane & 3;
  const int64_t s = (int64_t)blockIdx.x * TOK + wp * kRowsPerWarp + (lane >> 2);
  const bool valid = s < S;
  float* b = qbuf + wp * kRowsPerWarp * 128;
  const int h0 = blockIdx.y * hb, h1 = min(H, h0 + hb);
  for (int h = h0; h < h1; ++h) {
    uint32_t raw[16], res[16];
    if (valid) load_slice(x + s * rs + col + (int64_t)h * HD + 32 * sl, raw);
    else {
#pragma unroll
      for (int i = 0; i < 16; ++i) raw[i] = 0u;
    }
    slice_norm_rope(raw, res, lane, w ? w + 32 * sl : nullptr, do_norm, eps, cs, half, valid ? s : 0, S, b);
    // v = bf16 value - mean (quant_heads), formed twice: for the row maximum and for the codes
    const float4* mp = reinterpret_cast<const float4*>(mean + (int64_t)h * HD + 32 * sl);
    auto centred = [&](int c, float (&v)[4]) {
      v[0] = lo16(res[2 * c]); v[1] = hi16(res[2 * c]); v[2] = lo16(res[2 * c + 1]); v[3] = hi16(res[2 * c + 1]);
      const float4 m4 = mean ? __ldg(mp + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[0] = __fsub_rn(v[0], m4.x); v[1] = __fsub_rn(v[1], m4.y);
      v[2] = __fsub_rn(v[2], m4.z); v[3] = __fsub_rn(v[3], m4.w);
    };
    float m = 0.f;
    if (valid) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float v[4];
        centred(c, v);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
      }
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    if (BLOCK) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const int par = (h - h0) & 1;  // two slots: the next head's writes cannot meet this head's reads
      if (lane == 0) red[par][wp] = m;
      __syncthreads();
      m = red[par][0];
#pragma unroll
      for (int i = 1; i < 16; ++i) m = fmaxf(m, red[par][i]);
    }
    const float sc = fmaxf(__fdiv_rn(m, 127.f), 1e-20f);
    if (valid) {
      const float inv = __fdiv_rn(1.f, sc);
      uint32_t p[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float v[4];
        centred(c, v);
        p[c] = q127(v[0], inv) | (q127(v[1], inv) << 8) | (q127(v[2], inv) << 16) | (q127(v[3], inv) << 24);
      }
      uint4* dst = reinterpret_cast<uint4*>(codes + ((int64_t)h * S + s) * HD + 32 * sl);
      dst[0] = make_uint4(p[0], p[1], p[2], p[3]);
      dst[1] = make_uint4(p[4], p[5], p[6], p[7]);
    }
    if (sl == 0 && s < Sp) scales[(int64_t)h * Sp + s] = valid ? sc : 0.f;
  }
}

// Pair layout (D = 128, rot % 32 == 0): thread t of a row's four holds the rotation pairs (j, j + half) for j in
// the 4-pair chunks t, t + 4, t + 8, ... of [0, half) (Q = half / 4 pairs in all) and the unrotated dims in the same
// interleave over [rot, 128) (N = (128 - rot) / 4 of them): 32 values, each cos / sin entry read once, both
// elements of a pair in the same thread, and every load and store contiguous over the row's four threads.  The
// sum of squares still comes from the thread's 32-dim slice (the reference's order); that load brings the row
// into L1 for the pair-layout loads after it.
template <int ROT>
struct Pairs {
  static constexpr int HALF = ROT / 2, Q = HALF / 4, N = (128 - ROT) / 4;
  static_assert(ROT % 32 == 0 && ROT <= 128, "pair layout: rot % 32 == 0");
  // first dim of chunk c (4 values) of segment sg (0: low pair halves, 1: high halves, 2: unrotated) of thread t
  __device__ static int dim(int t, int sg, int c) { return (sg == 0 ? 0 : (sg == 1 ? HALF : ROT)) + 16 * c + 4 * t; }
  __device__ static constexpr int count(int sg) { return sg < 2 ? Q : N; }
  __device__ static constexpr int first(int sg) { return sg == 0 ? 0 : (sg == 1 ? Q : 2 * Q); }  // index in v[]
};

// 4 bf16 values (8-byte aligned) -> f32
__device__ __forceinline__ void load4(const uint16_t* __restrict__ p, float* v) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  v[0] = lo16(u.x);
  v[1] = hi16(u.x);
  v[2] = lo16(u.y);
  v[3] = hi16(u.y);
}

template <int ROT>
__device__ __forceinline__ void pair_norm_rope(const uint16_t* __restrict__ xr, int t, const uint16_t* __restrict__ w,
                                               int do_norm, float eps, const float* __restrict__ cs, int64_t s,
                                               int64_t S, uint32_t (&res)[16]) {
  using L = Pairs<ROT>;
  constexpr int Q = L::Q, HALF = L::HALF;
  float inv = 1.f;
  if (do_norm) {
    uint32_t raw[16];
    load_slice(xr + 32 * t, raw);
    float a[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float x0 = elem(raw, i), x1 = elem(raw, i + 16);
      a[i] = __fadd_rn(__fmul_rn(x0, x0), __fmul_rn(x1, x1));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < o; ++i) a[i] = __fadd_rn(a[i], a[i + o]);
    float tt = __fadd_rn(a[0], __shfl_xor_sync(0xffffffffu, a[0], 2));
    tt = __fadd_rn(tt, __shfl_xor_sync(0xffffffffu, tt, 1));
    inv = rsqrtf(__fadd_rn(__fdiv_rn(tt, 128.f), eps));
  }
  float v[32];
#pragma unroll
  for (int sg = 0; sg < 3; ++sg)
#pragma unroll
    for (int c = 0; c < L::count(sg) / 4; ++c) load4(xr + L::dim(t, sg, c), v + L::first(sg) + 4 * c);
  if (do_norm) {
    float wv[32];
    if (w) {
#pragma unroll
      for (int sg = 0; sg < 3; ++sg)
#pragma unroll
        for (int c = 0; c < L::count(sg) / 4; ++c) load4(w + L::dim(t, sg, c), wv + L::first(sg) + 4 * c);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) wv[i] = 1.f;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], inv), wv[i]);
  }
  if (Q > 0) {
#pragma unroll
    for (int c = 0; c < Q / 4; ++c) {
      const float4 cc = __ldg(reinterpret_cast<const float4*>(cs + s * HALF + L::dim(t, 0, c)));
      const float4 ss = __ldg(reinterpret_cast<const float4*>(cs + (S + s) * HALF + L::dim(t, 0, c)));
      const float cv[4] = {cc.x, cc.y, cc.z, cc.w}, sv[4] = {ss.x, ss.y, ss.z, ss.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = v[4 * c + i], b = v[Q + 4 * c + i];
        v[4 * c + i] = rope_lo(a, cv[i], b, sv[i]);
        v[Q + 4 * c + i] = rope_hi(b, cv[i], a, sv[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) res[i] = pack_bf16_ref(v[2 * i], v[2 * i + 1]);
}

// Standalone qk_norm_rope, pair layout: CTA of 8 warps = 64 tokens looping over `hb` heads.
template <int ROT>
__global__ void __launch_bounds__(256, 3) qk_norm_rope_pairs_kernel(const uint16_t* __restrict__ x, int64_t rs,
                                                                 int64_t col, int64_t hs,
                                                                 const uint16_t* __restrict__ w, int do_norm,
                                                                 float eps, const float* __restrict__ cs,
                                                                 uint16_t* __restrict__ out, int64_t S, int H, int hb) {
  using L = Pairs<ROT>;
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5, t = lane & 3;
  int64_t s = (int64_t)blockIdx.x * 64 + wp * kRowsPerWarp + (lane >> 2);
  const bool valid = s < S;
  if (!valid) s = S - 1;  // a real row: its lanes compute alongside (shuffles) and store nothing
  const int h1 = min(H, (int)(blockIdx.y + 1) * hb);
  for (int h = blockIdx.y * hb; h < h1; ++h) {
    uint32_t res[16];
    pair_norm_rope<ROT>(x + s * rs + col + (int64_t)h * hs, t, w, do_norm, eps, cs, s, S, res);
    if (valid) {
      uint16_t* o = out + (s * H + h) * HD;
#pragma unroll
      for (int sg = 0; sg < 3; ++sg)
#pragma unroll
        for (int c = 0; c < L::count(sg) / 4; ++c) {
          const int i = (L::first(sg) + 4 * c) / 2;
          *reinterpret_cast<uint2*>(o + L::dim(t, sg, c)) = make_uint2(res[i], res[i + 1]);
        }
    }
  }
}

// K column sums, pair layout: as kmean_rope_partial_kernel, the rows turned through a padded row buffer.
template <int ROT>
__global__ void __launch_bounds__(256, 3) kmean_rope_pairs_kernel(const uint16_t* __restrict__ x, int64_t rs,
                                                               int64_t col, const uint16_t* __restrict__ w,
                                                               int do_norm, float eps, const float* __restrict__ cs,
                                                               float* __restrict__ part, int64_t S, int H,
                                                               int rows_per) {
  using L = Pairs<ROT>;
  constexpr int RS = 132;  // padded row stride (floats)
  __shared__ __align__(16) float buf[8][kRowsPerWarp * RS];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5, t = lane & 3, r = lane >> 2;
  const int h = blockIdx.y * 8 + wp;
  if (h >= H) return;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per;
  const int64_t r1 = r0 + rows_per < S ? r0 + rows_per : S;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float* b = buf[wp];
  for (int64_t g = r0; g < r1; g += kRowsPerWarp) {
    int64_t s = g + r;
    if (s >= r1) s = r1 - 1;  // a real row whose values are not added
    uint32_t res[16];
    pair_norm_rope<ROT>(x + s * rs + col + (int64_t)h * HD, t, w, do_norm, eps, cs, s, S, res);
#pragma unroll
    for (int sg = 0; sg < 3; ++sg)
#pragma unroll
      for (int c = 0; c < L::count(sg) / 4; ++c) {
        const int i = (L::first(sg) + 4 * c) / 2;
        *reinterpret_cast<float4*>(b + r * RS + L::dim(t, sg, c)) =
            make_float4(lo16(res[i]), hi16(res[i]), lo16(res[i + 1]), hi16(res[i + 1]));
      }
    __syncwarp();
    const int nr = (int)(r1 - g < kRowsPerWarp ? r1 - g : kRowsPerWarp);
    for (int rr = 0; rr < nr; ++rr) {
      const float4 f = *reinterpret_cast<const float4*>(b + rr * RS + 4 * lane);
      acc[0] = __fadd_rn(acc[0], f.x);
      acc[1] = __fadd_rn(acc[1], f.y);
      acc[2] = __fadd_rn(acc[2], f.z);
      acc[3] = __fadd_rn(acc[3], f.w);
    }
    __syncwarp();
  }
  reinterpret_cast<float4*>(part + (int64_t)blockIdx.x * H * HD + (int64_t)h * HD)[lane] =
      make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// Normalise + rotate + (K: subtract the column mean) + quantise, pair layout; CTA as qk_rope_quant_kernel.
template <int ROT, bool BLOCK>
__global__ void __launch_bounds__(BLOCK ? 512 : 256, BLOCK ? 1 : 3) qk_rope_quant_pairs_kernel(
    const uint16_t* __restrict__ x, int64_t rs, int64_t col, const uint16_t* __restrict__ w, int do_norm, float eps,
    const float* __restrict__ cs, const float* __restrict__ mean, int8_t* __restrict__ codes,
    float* __restrict__ scales, int64_t S, int64_t Sp, int H, int hb) {
  using L = Pairs<ROT>;
  __shared__ float red[2][16];
  constexpr int TOK = BLOCK ? 128 : 64;
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5, t = lane & 3;
  const int64_t s = (int64_t)blockIdx.x * TOK + wp * kRowsPerWarp + (lane >> 2);
  const bool valid = s < S;
  const int64_t sr = valid ? s : S - 1;  // rows past S compute on a real row and take no part
  const int h0 = blockIdx.y * hb, h1 = min(H, h0 + hb);
  for (int h = h0; h < h1; ++h) {
    uint32_t res[16];
    pair_norm_rope<ROT>(x + sr * rs + col + (int64_t)h * HD, t, w, do_norm, eps, cs, sr, S, res);
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[2 * i] = lo16(res[i]);
      v[2 * i + 1] = hi16(res[i]);
    }
#pragma unroll
    for (int sg = 0; sg < 3; ++sg)
#pragma unroll
      for (int c = 0; c < L::count(sg) / 4; ++c) {
        const int i = L::first(sg) + 4 * c;
        const float4 m4 = mean ? __ldg(reinterpret_cast<const float4*>(mean + (int64_t)h * HD + L::dim(t, sg, c)))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i] = __fsub_rn(v[i], m4.x);
        v[i + 1] = __fsub_rn(v[i + 1], m4.y);
        v[i + 2] = __fsub_rn(v[i + 2], m4.z);
        v[i + 3] = __fsub_rn(v[i + 3], m4.w);
      }
    float m = 0.f;
    if (valid) {
#pragma unroll
      for (int i = 0; i < 32; ++i) m = fmaxf(m, fabsf(v[i]));
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    if (BLOCK) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const int par = (h - h0) & 1;
      if (lane == 0) red[par][wp] = m;
      __syncthreads();
      m = red[par][0];
#pragma unroll
      for (int i = 1; i < 16; ++i) m = fmaxf(m, red[par][i]);
    }
    const float sc = fmaxf(__fdiv_rn(m, 127.f), 1e-20f);
    if (valid) {
      const float inv = __fdiv_rn(1.f, sc);
      int8_t* row = codes + ((int64_t)h * S + s) * HD;
#pragma unroll
      for (int sg = 0; sg < 3; ++sg)
#pragma unroll
        for (int c = 0; c < L::count(sg) / 4; ++c) {
          const int i = L::first(sg) + 4 * c;
          *reinterpret_cast<uint32_t*>(row + L::dim(t, sg, c)) =
              q127(v[i], inv) | (q127(v[i + 1], inv) << 8) | (q127(v[i + 2], inv) << 16) | (q127(v[i + 3], inv) << 24);
        }
    }
    if (t == 0 && s < Sp) scales[(int64_t)h * Sp + s] = valid ? sc : 0.f;
  }
}

}  // namespace

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

cudaError_t launch_qk_norm_rope(const uint16_t* x, int64_t rs, int64_t col, int64_t hs, const uint16_t* w,
                                int do_norm, float eps, const float* cs, int rot, uint16_t* out, int64_t S, int64_t H,
                                int64_t D, cudaStream_t st) {
  if (S <= 0 || H <= 0 || D <= 0) return cudaSuccess;
  const bool a16 = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0 &&
                   rs % 8 == 0 && col % 8 == 0 && hs % 8 == 0;
  const bool wa = !w || (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
  const bool ca = rot == 0 || (reinterpret_cast<uintptr_t>(cs) & 15u) == 0;
  if (D == HD && rot % 8 == 0 && a16 && wa && ca) {
    const int hb = H < 8 ? (int)H : 8;
    const dim3 grid((unsigned)((S + 63) / 64), (unsigned)((H + hb - 1) / hb));
    switch (rot) {  // rotation pairs held by one thread where the pairs split evenly over a row's four threads
#define H3Q_PAIRS(R)                                                                                            \
  case R:                                                                                                      \
    qk_norm_rope_pairs_kernel<R><<<grid, 256, 0, st>>>(x, rs, col, hs, w, do_norm, eps, cs, out, S, (int)H, hb); \
    return cudaGetLastError();
      H3Q_PAIRS(0) H3Q_PAIRS(32) H3Q_PAIRS(64) H3Q_PAIRS(96) H3Q_PAIRS(128)
#undef H3Q_PAIRS
      default: break;
    }
    qk_norm_rope128_kernel<<<grid, 256, 0, st>>>(x, rs, col, hs, w, do_norm, eps, cs, rot / 2, out, S, (int)H, hb);
    return cudaGetLastError();
  }
  const int64_t rows = S * H;
  int64_t blocks = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count(0) * 16;
  if (blocks > cap) blocks = cap;
  qk_norm_rope_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, rs, col, hs, w, do_norm, eps, cs, rot, out, S, (int)H,
                                                        (int)D);
  return cudaGetLastError();
}

cudaError_t launch_kmean_rope(const uint16_t* x, int64_t rs, int64_t col, const uint16_t* w, int do_norm, float eps,
                              const float* cs, int rot, int64_t S, int64_t H, float* mean, float* part,
                              cudaStream_t st) {
  if (S <= 0 || H <= 0) return cudaSuccess;
  int parts, rows_per;
  kmean_partition(S, parts, rows_per);
  const dim3 grid((unsigned)parts, (unsigned)((H + 7) / 8));
  switch (rot) {
#define H3Q_PAIRS(R)                                                                                             \
  case R:                                                                                                       \
    kmean_rope_pairs_kernel<R><<<grid, 256, 0, st>>>(x, rs, col, w, do_norm, eps, cs, part, S, (int)H, rows_per); \
    break;
    H3Q_PAIRS(0) H3Q_PAIRS(32) H3Q_PAIRS(64) H3Q_PAIRS(96) H3Q_PAIRS(128)
#undef H3Q_PAIRS
    default:
      kmean_rope_partial_kernel<<<grid, 256, 0, st>>>(x, rs, col, w, do_norm, eps, cs, rot / 2, part, S, (int)H,
                                                      rows_per);
  }
  const int C = (int)(H * HD);
  const float inv_s = (float)(1.0 / (double)S);
  kmean_final_kernel<<<(C + 255) / 256, 256, 0, st>>>(part, parts, mean, C, inv_s);
  return cudaGetLastError();
}

cudaError_t launch_qk_rope_quant(const uint16_t* x, int64_t rs, int64_t col, const uint16_t* w, int do_norm,
                                 float eps, const float* cs, int rot, const float* mean, int8_t* codes, float* scales,
                                 int64_t S, int64_t H, bool block128, cudaStream_t st) {
  if (S <= 0 || H <= 0) return cudaSuccess;
  const int64_t Sp = (S + 127) / 128 * 128;
  const int tok = block128 ? 128 : 64, threads = tok * 4;
  // heads per CTA: the tokens' rope rows are read from L2 once per CTA; keep at least ~3 CTAs per SM busy
  const int64_t blocks = Sp / tok;
  int hb = 8;
  while (hb > 1 && blocks * ((H + hb - 1) / hb) < 3 * (int64_t)sm_count(0)) hb >>= 1;
  const dim3 grid((unsigned)blocks, (unsigned)((H + hb - 1) / hb));
  switch (rot) {
#define H3Q_PAIRS(R)                                                                                               \
  case R:                                                                                                         \
    if (block128)                                                                                                 \
      qk_rope_quant_pairs_kernel<R, true><<<grid, threads, 0, st>>>(x, rs, col, w, do_norm, eps, cs, mean, codes,  \
                                                                    scales, S, Sp, (int)H, hb);                   \
    else                                                                                                          \
      qk_rope_quant_pairs_kernel<R, false><<<grid, threads, 0, st>>>(x, rs, col, w, do_norm, eps, cs, mean, codes, \
                                                                     scales, S, Sp, (int)H, hb);                  \
    return cudaGetLastError();
    H3Q_PAIRS(0) H3Q_PAIRS(32) H3Q_PAIRS(64) H3Q_PAIRS(96) H3Q_PAIRS(128)
#undef H3Q_PAIRS
    default: break;
  }
  const size_t smem = (size_t)(threads / 32) * kRowsPerWarp * 128 * sizeof(float);
  auto kern = block128 ? qk_rope_quant_kernel<true> : qk_rope_quant_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, threads, smem, st>>>(x, rs, col, w, do_norm, eps, cs, rot / 2, mean, codes, scales, S, Sp, (int)H, hb);
  return cudaGetLastError();
}

}  // namespace h3q
