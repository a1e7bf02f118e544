// gemm_common.cuh -- pieces shared by the tcgen05 GEMM kernels: tile raster, broadcast loads, output packing,
// the TMA-store epilogue helper and host-side tensor-map encoding.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include "ptx.cuh"

namespace h3q {

constexpr int EPI_BUF = 4096;              // one staging buffer: 32 rows x up to 128 bytes
constexpr int EPI_SMEM = 4 * 2 * EPI_BUF;  // 4 epilogue warps, double buffered

// Tile order: groups of `group_m` tile-rows sweep all tile-columns, column-fastest inside a group when
// group_m == 1.  The host picks group_m so the operands re-read across the sweep stay in L2.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group_m, int& mb, int& nb) {
  const int per_group = group_m * num_n;
  const int group = t / per_group;
  const int first_m = group * group_m;
  const int gsz = min(num_m - first_m, group_m);
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

// 32 f32 values -> packed words of the output kind (0 f32, 1 f16, 2 bf16); returns the row-chunk width in bytes.
// bf16: the hardware's paired round-to-nearest-even conversion (one instruction per two values, the same bits as
// f2bf for every non-NaN value, subnormals, infinities and overflow to infinity included), then, only when the
// chunk holds a NaN, f2bf for the chunk so every NaN becomes the reference's 0x7fc0.
__device__ __forceinline__ int pack_out(const float (&v)[32], int kind, uint32_t (&w)[32]) {
  if (kind == 0) {
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(v[i]);
    return 128;
  }
  if (kind == 2) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w[i]) : "f"(v[2 * i + 1]), "f"(v[2 * i]));
      asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(m), "f"(v[2 * i]), "f"(v[2 * i + 1]));
    }
    if (m != m) {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = pack_bf2(v[2 * i], v[2 * i + 1]);
    }
    return 64;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = (uint32_t)f2h(v[2 * i]) | ((uint32_t)f2h(v[2 * i + 1]) << 16);
  return 64;
}

// One warp's TMA-store epilogue: each lane stages its row of a 32-row box into a swizzled shared-memory buffer
// (the TMA swizzle of the box's row width W, which also makes the 16-byte writes bank-conflict free), then lane
// 0 stores the box.  Two buffers alternate; a buffer is rewritten only after its previous store has read it.
// Output tensor maps of a GEMM launch: one per destination buffer.  The all-gather GEMM stores every output box to
// each rank's copy of the output (peer memory over NVLink); every other launch has one destination.
template <int NDST>
struct OutMaps {
  CUtensorMap m[NDST];
  int n;  // destinations in use (1..NDST)
};

struct EpiWarp {
  const CUtensorMap* map;  // `nmaps` consecutive maps
  int nmaps;
  uint8_t* buf;  // 2 * EPI_BUF bytes, 1024-aligned
  int sel;
  int lane;

  __device__ __forceinline__ void store(const uint32_t (&w)[32], int W, int32_t x, int32_t y, bool do_store) {
    if (lane == 0) bulk_wait_read<1>();
    __syncwarp();
    uint8_t* b = buf + sel * EPI_BUF + lane * W;
    const int sw = W == 128 ? (lane & 7) : (W == 64 ? ((lane >> 1) & 3) : ((lane >> 2) & 1));
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < W / 16)
        *reinterpret_cast<uint4*>(b + ((i ^ sw) << 4)) = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    // one bulk group per call, empty when the box lies outside the output: the wait at the top of the next call
    // that reuses this buffer then always covers the store that last read it
    if (lane == 0) {
      if (do_store)
        for (int d = 0; d < nmaps; ++d) tma_store_2d(map + d, buf + sel * EPI_BUF, x, y);
      bulk_commit();
    }
    sel ^= 1;
  }
};

// ---------------------------------------------------------------------------------------------- host side

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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
inline bool make_tmap_i8(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {128, box_rows};  // 128 bytes of K: one 128-byte swizzle row
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output tensor map for the epilogue's TMA stores: [M, nout] row-major (row pitch `pitch` elements, default nout),
// box = (W / es) columns x 32 rows, swizzle matching the box's row width W.
inline bool make_tmap_out(CUtensorMap* m, void* base, uint64_t rows, uint64_t cols, int es, int W,
                          uint64_t pitch = 0) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {(pitch ? pitch : cols) * (uint64_t)es};
  cuuint32_t box[2] = {(cuuint32_t)(W / es), 32};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      es == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  const CUtensorMapSwizzle sw =
      W == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : (W == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  return fn(m, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace h3q
