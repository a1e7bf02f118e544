// lora.cu -- folding LoRA deltas into a layer's weight once, at load time (QLinear::merge_loras,
// weights.rs:692-761; run for every DiT linear when a LoRA is applied, dit.rs:599-611), so the int8 hot path
// serves the merged layer with no per-step LoRA work.
//
// int8 layer (weights.rs:716-757), per row:
//   w = (float)q * s                          dequant_i8 (kernels.rs:40-48; s per row or one scalar)
//   w = rotate_activation(w, 256)             ConvRot layers only: back to the plain basis (H symmetric, H H = I)
//   w = w + sum_l f32(scale_l) * (B_l A_l)    the deltas (weights.rs:696-707), B_l [n, r_l], A_l [r_l, k]
//   w = rotate_activation(w, 256)             ConvRot layers only
//   s' = max(max|w| * f32(1/127), 1e-30)      candle's `/ 127.0` is an affine multiply by f32(1/127)
//   q' = clamp(round(w / s'), -128, 127)      IEEE division, round half away from zero (weights.rs:735-738)
// dense layer (weights.rs:710-715): w' = dtype(f32(w) + sum_l f32(scale_l) * (B_l A_l)).
//
// The reference forms B A and the rotations as f32 matmuls whose summation order it leaves to the BLAS.  This
// library fixes one order, which the CPU oracle restates: a delta element is the chain fma(B[i,j], A[j,c], acc)
// over j = 0, 1, ... from acc = 0, times f32(scale_l), and deltas are summed in LoRA order; the rotation is the
// fused quantizer's radix-4 butterfly (digit 0 summed ((a0+a1)+a2)+a3, digits 1-3 (a0+a1)+(a2+a3),
// out_p = s - 2 a_{3-p}, then times 1/16).
//
// Layout: one CTA per (32 rows) x (256 columns = one rotation group); thread (row r, quarter j) owns the row's 64
// contiguous columns 64j .. 64j+63, so rotation digits 0-2 run in registers and digit 3 crosses the row's four
// lanes by shuffles.  The deltas are computed in a different thread layout first: thread (warp w, lane l) owns an
// 8-row x 8-column micro-tile (rows 8w .. 8w+7, columns 4l .. 4l+3 and 128+4l .. 128+4l+3), register-accumulated
// from rank chunks of A and B staged in shared memory as f32, two columns per paired fma.rn.f32x2, so every staged
// value feeds eight FMAs (each element's chain is the same sequence of rounded fmas in either layout).  The summed
// delta tile then passes once through shared memory into the rotation layout.  int8 layers write the merged f32 rows to a workspace and the row maxima by atomics; a second kernel
// requantizes.  Rows are processed in chunks that fit the caller's workspace.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include "../../include/h3q.h"
#include "ptx.cuh"

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

constexpr int kMaxLoras = 16;
constexpr int kRows = 32;       // rows per CTA
constexpr int kCols = 256;      // columns per CTA (one rotation group)
constexpr int kChunk = 32;      // rank entries staged per shared-memory round
constexpr int kSeg = 68;        // f32 stride of a thread quarter's 64 columns in the staged A rows (+4: no conflicts)
constexpr int kThreads = 128;   // kRows x 4 quarters

struct Term {
  const void* a;   // [rank, k]
  const void* b;   // [n, rank]
  int64_t rank;
  int kind;        // 0 f32, 1 f16, 2 bf16
  float scale;
};

struct MergeArgs {
  const void* w;         // int8 codes [n, k] or a dense f32 / f16 / bf16 weight
  int w_kind;            // dense: 0 f32, 1 f16, 2 bf16
  const float* w_scale;  // int8: [n] or one scalar
  int per_row;
  int64_t n, k;
  int64_t row0, rows;    // this chunk of rows
  Term l[kMaxLoras];
  int n_loras;
  float* vals;           // int8: merged f32 rows of the chunk [rows, k]
  unsigned* rowmax;      // int8: bits of max |merged| per chunk row (non-negative floats order as integers)
  void* out;             // dense: merged weight [n, k] in w_kind
};

__device__ __forceinline__ float ld_f32(const void* p, int kind, int64_t i) {
  if (kind == 0) return static_cast<const float*>(p)[i];
  if (kind == 1) return __half2float(static_cast<const __half*>(p)[i]);
  return __uint_as_float((uint32_t) static_cast<const uint16_t*>(p)[i] << 16);
}

// One radix-4 stage over (a0, a1, a2, a3) = the values of one digit (0..3): out_p = s - 2 a_{3-p}, with s summed
// ((a0+a1)+a2)+a3 for digit 0 and (a0+a1)+(a2+a3) for digits 1-3.  fma(-2, a, s) rounds s - 2a once (2a is exact).
__device__ __forceinline__ void h4(float& a0, float& a1, float& a2, float& a3, bool first) {
  const float s = first ? __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3)
                        : __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
  const float b0 = __fmaf_rn(-2.f, a3, s), b1 = __fmaf_rn(-2.f, a2, s);
  const float b2 = __fmaf_rn(-2.f, a1, s), b3 = __fmaf_rn(-2.f, a0, s);
  a0 = b0; a1 = b1; a2 = b2; a3 = b3;
}

// rotate_activation of a 256-group whose columns 64j .. 64j+63 sit in v of lane j of an aligned lane quad
// (element e of the thread = digits d0 + 4 d1 + 16 d2, digit 3 = j).  Every lane of the warp must call it.
__device__ __forceinline__ void rotate256(float (&v)[64]) {
#pragma unroll
  for (int b = 0; b < 16; ++b) h4(v[4 * b], v[4 * b + 1], v[4 * b + 2], v[4 * b + 3], true);
#pragma unroll
  for (int b = 0; b < 4; ++b)
#pragma unroll
    for (int i = 0; i < 4; ++i) h4(v[16 * b + i], v[16 * b + i + 4], v[16 * b + i + 8], v[16 * b + i + 12], false);
#pragma unroll
  for (int i = 0; i < 16; ++i) h4(v[i], v[i + 16], v[i + 32], v[i + 48], false);
  // digit 3: lane j holds the value of digit j; s = (v_j + v_{j^1}) + (v_{j^2} + v_{j^3}), the same sum in every
  // lane, and out_j = s - 2 v_{3-j} (3 - j = j ^ 3)
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const float s1 = __fadd_rn(v[i], __shfl_xor_sync(0xffffffffu, v[i], 1));
    const float s = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 2));
    v[i] = __fmul_rn(__fmaf_rn(-2.f, __shfl_xor_sync(0xffffffffu, v[i], 3), s), 0.0625f);
  }
}

template <bool I8, bool ROT>
__global__ void __launch_bounds__(kThreads, 1) lora_merge_kernel(const MergeArgs p) {
  __shared__ __align__(16) float As[kChunk][4 * kSeg];  // read as float4
  __shared__ __align__(16) float Bs[kChunk][kRows];      // transposed: (rank entry, row)
  const int t = threadIdx.x, r = t >> 2, j = t & 3;
  const int64_t rloc = (int64_t)blockIdx.y * kRows + r;  // row within the chunk
  const int64_t row = p.row0 + rloc;
  const bool rv = rloc < p.rows;
  const int64_t cg = (int64_t)blockIdx.x * kCols;         // first column of the CTA
  const int64_t c0 = cg + 64 * j;                          // first column of the thread
  const int nv = p.k - c0 >= 64 ? 64 : (p.k - c0 > 0 ? (int)(p.k - c0) : 0);
  // delta micro-tile of the thread: rows 8 mw .. 8 mw + 7, columns 4 ml .. 4 ml + 3 and 128 + 4 ml .. + 3; element
  // pairs [4 i + h] = row 8 mw + i, columns (c_h, c_h + 1) with c_0 = 4 ml, c_1 = 4 ml + 2, c_2 = 128 + 4 ml, c_3 = +2
  const int mw = t >> 5, ml = t & 31;
  const int ca = ((4 * ml) >> 6) * kSeg + ((4 * ml) & 63);                  // staged-A offset of column 4 ml
  const int cb = ((128 + 4 * ml) >> 6) * kSeg + ((128 + 4 * ml) & 63);      // and of column 128 + 4 ml

  h3q::f2 tot2[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) tot2[i] = h3q::pk(0.f, 0.f);
  for (int l = 0; l < p.n_loras; ++l) {
    const Term tm = p.l[l];
    h3q::f2 acc2[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc2[i] = h3q::pk(0.f, 0.f);
    // bf16 factors whose column group is whole and 16-byte aligned are staged 8 values per load
    const bool vec_a = tm.kind == 2 && (p.k & 7) == 0 && cg + kCols <= p.k &&
                       (reinterpret_cast<uintptr_t>(tm.a) & 15u) == 0;
    for (int64_t j0 = 0; j0 < tm.rank; j0 += kChunk) {
      const int nj = tm.rank - j0 < kChunk ? (int)(tm.rank - j0) : kChunk;
      __syncthreads();  // the previous chunk has been consumed
      if (vec_a) {
        for (int idx = t; idx < kChunk * (kCols / 8); idx += kThreads) {
          const int jj = idx >> 5, c = (idx & 31) * 8;
          uint4 raw = make_uint4(0u, 0u, 0u, 0u);
          if (jj < nj)
            raw = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(tm.a) + (j0 + jj) * p.k + cg + c);
          float4* dst = reinterpret_cast<float4*>(&As[jj][(c >> 6) * kSeg + (c & 63)]);
          dst[0] = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                               __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u));
          dst[1] = make_float4(__uint_as_float(raw.z << 16), __uint_as_float(raw.z & 0xffff0000u),
                               __uint_as_float(raw.w << 16), __uint_as_float(raw.w & 0xffff0000u));
        }
      } else {
        for (int idx = t; idx < kChunk * kCols; idx += kThreads) {
          const int jj = idx >> 8, c = idx & (kCols - 1);
          float a = 0.f;
          if (jj < nj && cg + c < p.k) a = ld_f32(tm.a, tm.kind, (j0 + jj) * p.k + cg + c);
          As[jj][(c >> 6) * kSeg + (c & 63)] = a;
        }
      }
      for (int idx = t; idx < kRows * kChunk; idx += kThreads) {
        const int rr = idx % kRows, jj = idx / kRows;  // rows fastest: conflict-free transposed stores
        const int64_t rl = (int64_t)blockIdx.y * kRows + rr;
        float b = 0.f;
        if (jj < nj && rl < p.rows) b = ld_f32(tm.b, tm.kind, (p.row0 + rl) * tm.rank + j0 + jj);
        Bs[jj][rr] = b;
      }
      __syncthreads();
      for (int jj = 0; jj < nj; ++jj) {
        const float4 a0 = *reinterpret_cast<const float4*>(&As[jj][ca]);
        const float4 a1 = *reinterpret_cast<const float4*>(&As[jj][cb]);
        const float4 b0 = *reinterpret_cast<const float4*>(&Bs[jj][8 * mw]);
        const float4 b1 = *reinterpret_cast<const float4*>(&Bs[jj][8 * mw + 4]);
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const h3q::f2 a00 = h3q::pk(a0.x, a0.y), a01 = h3q::pk(a0.z, a0.w);
        const h3q::f2 a10 = h3q::pk(a1.x, a1.y), a11 = h3q::pk(a1.z, a1.w);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const h3q::f2 b2 = h3q::pk(bv[i], bv[i]);
          acc2[4 * i] = h3q::fma2(b2, a00, acc2[4 * i]);
          acc2[4 * i + 1] = h3q::fma2(b2, a01, acc2[4 * i + 1]);
          acc2[4 * i + 2] = h3q::fma2(b2, a10, acc2[4 * i + 2]);
          acc2[4 * i + 3] = h3q::fma2(b2, a11, acc2[4 * i + 3]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float a0, a1, t0, t1;
      h3q::upk(acc2[i], a0, a1);
      h3q::upk(tot2[i], t0, t1);
      const float d0 = __fmul_rn(a0, tm.scale), d1 = __fmul_rn(a1, tm.scale);
      tot2[i] = l == 0 ? h3q::pk(d0, d1) : h3q::pk(__fadd_rn(t0, d0), __fadd_rn(t1, d1));
    }
  }
  // the summed delta tile into the rotation layout, through the A staging area (32 rows x 4 x kSeg floats)
  float tot[64];
  if (p.n_loras > 0) {
    __syncthreads();  // the last chunk has been consumed
    float* ds = &As[0][0];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x0, x1, x2, x3, y0, y1, y2, y3;
      h3q::upk(tot2[4 * i], x0, x1);
      h3q::upk(tot2[4 * i + 1], x2, x3);
      h3q::upk(tot2[4 * i + 2], y0, y1);
      h3q::upk(tot2[4 * i + 3], y2, y3);
      float* drow = ds + (8 * mw + i) * (4 * kSeg);
      *reinterpret_cast<float4*>(drow + ca) = make_float4(x0, x1, x2, x3);
      *reinterpret_cast<float4*>(drow + cb) = make_float4(y0, y1, y2, y3);
    }
    __syncthreads();
    const float4* src = reinterpret_cast<const float4*>(ds + r * (4 * kSeg) + j * kSeg);
#pragma unroll
    for (int c4 = 0; c4 < 16; ++c4) {
      const float4 v4 = src[c4];
      tot[4 * c4] = v4.x; tot[4 * c4 + 1] = v4.y; tot[4 * c4 + 2] = v4.z; tot[4 * c4 + 3] = v4.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) tot[i] = 0.f;
  }

  float v[64];
  if (I8) {
    const float s = rv ? (p.per_row ? p.w_scale[row] : p.w_scale[0]) : 0.f;
    const int8_t* q = static_cast<const int8_t*>(p.w) + row * p.k + c0;
    if (rv && nv == 64 && ((reinterpret_cast<uintptr_t>(q) & 15u) == 0)) {
#pragma unroll
      for (int c16 = 0; c16 < 4; ++c16) {
        const int4 raw = reinterpret_cast<const int4*>(q)[c16];
        const uint32_t wd[4] = {(uint32_t)raw.x, (uint32_t)raw.y, (uint32_t)raw.z, (uint32_t)raw.w};
#pragma unroll
        for (int e = 0; e < 16; ++e)
          v[16 * c16 + e] = __fmul_rn((float)(int8_t)(wd[e >> 2] >> (8 * (e & 3))), s);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 64; ++e) v[e] = (rv && e < nv) ? __fmul_rn((float)q[e], s) : 0.f;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 64; ++e) v[e] = (rv && e < nv) ? ld_f32(p.w, p.w_kind, row * p.k + c0 + e) : 0.f;
  }
  if (ROT) rotate256(v);
#pragma unroll
  for (int e = 0; e < 64; ++e) v[e] = __fadd_rn(v[e], tot[e]);
  if (ROT) rotate256(v);

  if (I8) {
    float m = 0.f;
    float* dst = p.vals + rloc * p.k + c0;
    if (rv) {
      if (nv == 64 && (p.k & 3) == 0) {
#pragma unroll
        for (int c4 = 0; c4 < 16; ++c4)
          reinterpret_cast<float4*>(dst)[c4] = make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
      } else {
#pragma unroll
        for (int e = 0; e < 64; ++e)
          if (e < nv) dst[e] = v[e];
      }
#pragma unroll
      for (int e = 0; e < 64; ++e)
        if (e < nv) m = fmaxf(m, fabsf(v[e]));
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    if (rv && j == 0) atomicMax(p.rowmax + rloc, __float_as_uint(m));
  } else if (rv) {
#pragma unroll
    for (int e = 0; e < 64; ++e) {
      if (e >= nv) continue;
      const int64_t i = row * p.k + c0 + e;
      if (p.w_kind == 0) static_cast<float*>(p.out)[i] = v[e];
      else if (p.w_kind == 1) static_cast<__half*>(p.out)[i] = __float2half_rn(v[e]);
      else {
        uint16_t h;
        asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(v[e]));
        static_cast<uint16_t*>(p.out)[i] = h;
      }
    }
  }
}

// s' = max(max|w| * f32(1/127), 1e-30), q' = clamp(round(w / s'), -128, 127) for each row of the chunk.
__global__ void __launch_bounds__(256) lora_requant_kernel(const float* __restrict__ vals,
                                                           const unsigned* __restrict__ rowmax, int8_t* __restrict__ q,
                                                           float* __restrict__ scale, int64_t row0, int64_t k) {
  const int64_t rl = blockIdx.x;
  const float m = __uint_as_float(rowmax[rl]);
  const float s = fmaxf(__fmul_rn(m, (float)(1.0 / 127.0)), 1e-30f);
  if (threadIdx.x == 0) scale[row0 + rl] = s;
  const float* src = vals + rl * k;
  int8_t* dst = q + (row0 + rl) * k;
  for (int64_t c = threadIdx.x; c < k; c += blockDim.x) {
    const float r = roundf(__fdiv_rn(src[c], s));
    dst[c] = (int8_t)(int)fminf(fmaxf(r, -128.f), 127.f);
  }
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

h3q_status fill_terms(const h3q_lora* loras, int n_loras, MergeArgs& a, const char* what) {
  if (n_loras < 0 || n_loras > kMaxLoras)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: %d LoRA deltas (this build merges up to %d per call)", what, n_loras,
                kMaxLoras);
  if (n_loras > 0 && !loras) return fail(H3Q_ERR_ARG, "%s: null LoRA array", what);
  for (int i = 0; i < n_loras; ++i) {
    const h3q_lora& l = loras[i];
    if (l.rank < 0) return fail(H3Q_ERR_ARG, "%s: LoRA %d has a negative rank", what, i);
    if (l.dtype != H3Q_DT_F32 && l.dtype != H3Q_DT_F16 && l.dtype != H3Q_DT_BF16)
      return fail(H3Q_ERR_ARG, "%s: LoRA %d factors must be f32, f16 or bf16", what, i);
    if (l.rank > 0 && (!l.a || !l.b)) return fail(H3Q_ERR_ARG, "%s: LoRA %d has a null factor", what, i);
    a.l[i] = Term{l.a, l.b, l.rank, l.dtype, (float)l.scale};
  }
  a.n_loras = n_loras;
  return H3Q_OK;
}

}  // namespace

extern "C" {

size_t h3q_lora_merge_i8_workspace_size(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0) return 0;
  return align256((size_t)n * 4) + (size_t)n * (size_t)k * 4;
}

h3q_status h3q_lora_merge_i8(const int8_t* w, const float* w_scale, int64_t scale_numel, int convrot,
                             const h3q_lora* loras, int n_loras, int8_t* w_out, float* scale_out, int64_t n, int64_t k,
                             void* workspace, size_t workspace_bytes, void* stream) {
  const char* what = "h3q_lora_merge_i8";
  if (n < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (convrot != 0 && convrot != 256)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: ConvRot group %d (this build rotates groups of 256)", what, convrot);
  if (convrot && k % 256 != 0)
    return fail(H3Q_ERR_ARG, "ConvRot group 256 does not divide [%lld, %lld]", (long long)n, (long long)k);
  MergeArgs a{};
  if (h3q_status st = fill_terms(loras, n_loras, a, what)) return st;
  if (n == 0 || k == 0 || n_loras == 0) return H3Q_OK;  // nothing to merge: the layer is left as it is
  if (!w || !w_scale || !w_out || !scale_out || !workspace) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  const bool per_row = scale_numel == n;
  if (!per_row && scale_numel != 1)
    return fail(H3Q_ERR_ARG, "%s: %lld weight scales for %lld rows (one per row or one)", what,
                (long long)scale_numel, (long long)n);
  if (!per_row && n > 1 && (const void*)scale_out == (const void*)w_scale)
    return fail(H3Q_ERR_ARG, "%s: scale_out holds one scale per row and cannot alias a scalar w_scale", what);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(H3Q_ERR_ARG, "%s: the workspace must be 256-byte aligned", what);
  // rows per chunk: the row maxima (256-byte aligned block) and the f32 rows must fit the workspace
  int64_t chunk = n;
  while (chunk > 0 && align256((size_t)chunk * 4) + (size_t)chunk * (size_t)k * 4 > workspace_bytes)
    chunk = chunk > kRows ? (chunk / 2 + kRows - 1) / kRows * kRows : chunk - 1;
  if (chunk < 1)
    return fail(H3Q_ERR_ARG, "%s: workspace of %zu bytes is below the %zu bytes of one row", what, workspace_bytes,
                align256(4) + (size_t)k * 4);
  if ((k + kCols - 1) / kCols > 0x7fffffff || (chunk + kRows - 1) / kRows > 65535)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: shape [%lld, %lld] exceeds this build's grid", what, (long long)n,
                (long long)k);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned* rowmax = static_cast<unsigned*>(workspace);
  float* vals = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256((size_t)chunk * 4));
  a.w = w;
  a.w_scale = w_scale;
  a.per_row = per_row ? 1 : 0;
  a.n = n;
  a.k = k;
  a.vals = vals;
  a.rowmax = rowmax;
  for (int64_t r0 = 0; r0 < n; r0 += chunk) {
    const int64_t rows = n - r0 < chunk ? n - r0 : chunk;
    a.row0 = r0;
    a.rows = rows;
    if (h3q_status s = cuda_status(cudaMemsetAsync(rowmax, 0, (size_t)rows * 4, st), what)) return s;
    const dim3 grid((unsigned)((k + kCols - 1) / kCols), (unsigned)((rows + kRows - 1) / kRows));
    if (convrot) lora_merge_kernel<true, true><<<grid, kThreads, 0, st>>>(a);
    else lora_merge_kernel<true, false><<<grid, kThreads, 0, st>>>(a);
    if (h3q_status s = cuda_status(cudaGetLastError(), what)) return s;
    lora_requant_kernel<<<(unsigned)rows, 256, 0, st>>>(vals, rowmax, w_out, scale_out, r0, k);
    if (h3q_status s = cuda_status(cudaGetLastError(), what)) return s;
  }
  return H3Q_OK;
}

h3q_status h3q_lora_merge_dense(const void* w, int dtype, const h3q_lora* loras, int n_loras, void* w_out, int64_t n,
                                int64_t k, void* stream) {
  const char* what = "h3q_lora_merge_dense";
  if (n < 0 || k < 0) return fail(H3Q_ERR_ARG, "%s: negative shape", what);
  if (dtype != H3Q_DT_F32 && dtype != H3Q_DT_F16 && dtype != H3Q_DT_BF16)
    return fail(H3Q_ERR_ARG, "%s: the weight must be f32, f16 or bf16", what);
  MergeArgs a{};
  if (h3q_status st = fill_terms(loras, n_loras, a, what)) return st;
  if (n == 0 || k == 0 || n_loras == 0) return H3Q_OK;
  if (!w || !w_out) return fail(H3Q_ERR_ARG, "%s: null pointer", what);
  if ((n + kRows - 1) / kRows > 65535 || (k + kCols - 1) / kCols > 0x7fffffff)
    return fail(H3Q_ERR_UNSUPPORTED, "%s: shape [%lld, %lld] exceeds this build's grid", what, (long long)n,
                (long long)k);
  a.w = w;
  a.w_kind = dtype;
  a.n = n;
  a.k = k;
  a.row0 = 0;
  a.rows = n;
  a.out = w_out;
  const dim3 grid((unsigned)((k + kCols - 1) / kCols), (unsigned)((n + kRows - 1) / kRows));
  lora_merge_kernel<false, false><<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cuda_status(cudaGetLastError(), what);
}

}  // extern "C"
