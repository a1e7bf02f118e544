// attn.cu -- SageAttention-style attention for head_dim 128 on the 5th-generation tensor cores: int8 Q.K^T
// (tcgen05 kind::i8, int32 scores in TMEM), online softmax in base 2, P.V in f16 (or bf16) with f32 accumulation
// (tcgen05 kind::f16, O in TMEM).  It computes what the reference's attn_qk8 computes (attn8.rs:107-246):
//   p   = acc_i32 * (qs * log2(e) / sqrt(128)) * ks          (attn8.rs:130-131, :187-190, :625)
//   out = bf16( sum_j f16(2^(p_j - m)) v_j / sum_j 2^(p_j - m) )
// with keys >= S masked out; non-causal, no mask otherwise.
//
// One CTA per (head, 256 query rows) = two 128-row Q tiles; 384 threads:
//   warp 0     one elected lane: TMA loads of the two Q tiles, then per 128-key tile the K codes (3-stage ring),
//              the 128 key scales (1-D bulk copy, 4-stage ring) and the V^T tile (2-stage ring);
//   warp 1     allocates 512 TMEM columns (S0, S1: int32 scores; O0, O1: f32 outputs) and issues the MMAs:
//              S_t = Q_t K_j^T for the next key tile as soon as softmax t has read S_t, then O_t += P_t V_j;
//   (warps 2-3 idle; warpgroup 0 runs with 96 registers per thread, the softmax warpgroups with 200)
//   warps 4-7  softmax for Q tile 0, warps 8-11 for Q tile 1: thread = query row = TMEM lane.  Each reads its
//              row's 128 scores, scales them by the key scales, takes the row maximum, writes
//              P = 2^(s * qs' - m) as 16-bit values into shared memory (the K-major 128-byte-swizzle layout the
//              MMA reads), and accumulates the row sum.  The running maximum m is only moved when a tile raises
//              it by more than 2^8; the O row in TMEM is then rescaled in place.  Between moves the unnormalised
//              P may reach 256, which f16 holds exactly as it holds values below 1; O / l is unchanged.
// Every wait is bounded: on time-out the CTA latches an error code, drains its own loads and MMAs, frees TMEM
// and returns.
#include <cstdint>
#include <cstdio>
#include <cmath>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "h3q_internal.h"
#include "gemm_common.cuh"

namespace h3q {

namespace {
constexpr int BM = 128;                 // query rows per Q tile
constexpr int BN = 128;                 // keys per key tile
constexpr int HD = 128;                 // head dim
constexpr int NQ = 2;                   // Q tiles per CTA
constexpr int KST = 3, VST = 2, SST = 4;
constexpr int THREADS = 128 + NQ * 128;  // warpgroup 0: loads + MMA; one softmax warpgroup per Q tile
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 = 64,512 of the 65,536), warpgroup 0 gives
// back to 96 and the softmax warpgroups grow to 200: 128 x 96 + 256 x 200 = 63,488 <= 64,512, and per SM
// sub-partition (one warp of each warpgroup) 96 + 200 + 200 = 496 <= 512 registers per lane.  Neither side spills.
constexpr int REGS_LOW = 96, REGS_HIGH = 200;
static_assert(128 * REGS_LOW + NQ * 128 * REGS_HIGH <= THREADS * 168, "setmaxnreg split exceeds the launch");
constexpr uint32_t TMEM_COLS = 512;
constexpr int Q_TILE = BM * HD;         // 16 KiB of int8 codes
constexpr int K_TILE = BN * HD;         // 16 KiB
constexpr int V_SLAB = 64 * HD * 2;     // 16 KiB: 128 dims x 64 keys, 16-bit
constexpr int V_TILE = 2 * V_SLAB;
constexpr int P_SLAB = BM * 64 * 2;     // 16 KiB: 128 rows x 64 keys, 16-bit
constexpr int P_TILE = 2 * P_SLAB;
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + NQ * Q_TILE;
constexpr int OFF_V = OFF_K + KST * K_TILE;
constexpr int OFF_P = OFF_V + VST * V_TILE;
constexpr int OFF_SC = OFF_P + NQ * P_TILE;
constexpr int OFF_BAR = OFF_SC + SST * BN * 4;
constexpr int NBAR = 1 + 2 * KST + 2 * VST + 2 * SST + 4 * NQ + 1;
constexpr size_t SMEM = 1024 + OFF_BAR + NBAR * 8 + 16;
constexpr float kMoveMax = 8.0f;        // log2 of the largest unnormalised probability
static_assert(SMEM <= 232448, "attention shared memory exceeds the sm_100 per-CTA limit");

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_pv(float lo, float hi, bool bf16) {
  uint32_t r;
  if (bf16) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
}  // namespace

struct AttnArgs {
  const float* qs;     // [H, Sqp] query scales
  const float* ks;     // [H, Sp] key scales
  uint16_t* out;       // [Sq, H, 128] bf16
  int32_t* scores;     // optional [H, Sq, S] int32 accumulators (diagnostic instantiation only)
  int S, H, Sp, nqb;   // keys, heads, padded keys, 256-row query blocks per head
  int Sq, Sqp;         // query rows and their padded count (Sq == S unless the queries are a shard)
  float scale_log2;
  int* err;
};

template <bool BF16PV, bool DUMP>
__global__ void __launch_bounds__(THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AttnArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + KST;
  uint64_t* v_full = k_empty + KST;
  uint64_t* v_empty = v_full + VST;
  uint64_t* sc_full = v_empty + VST;
  uint64_t* sc_empty = sc_full + SST;
  uint64_t* s_full = sc_empty + SST;
  uint64_t* s_free = s_full + NQ;
  uint64_t* p_full = s_free + NQ;
  uint64_t* pv_done = p_full + NQ;
  uint64_t* mma_done = pv_done + NQ;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = (int)blockIdx.x / p.nqb, qb = (int)blockIdx.x % p.nqb;
  const int nkv = (p.S + BN - 1) / BN;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KST; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
    for (int i = 0; i < VST; ++i) { mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1); }
    for (int i = 0; i < SST; ++i) { mbar_init(&sc_full[i], 1); mbar_init(&sc_empty[i], 4 * NQ); }
    for (int t = 0; t < NQ; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], 4);
      mbar_init(&p_full[t], 4);
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_LOW));
    if (warp == 0 && elect_one()) {
      // ------------------------------------------------------------------ TMA producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, NQ * Q_TILE);
      for (int t = 0; t < NQ; ++t)
        tma_load_3d(smem + OFF_Q + t * Q_TILE, &tmQ, q_full, 0, (qb * NQ + t) * BM, h);
      int last = -1;  // last key tile whose loads were all issued
      for (int j = 0; j < nkv; ++j) {
        const int ks = j % KST, ss = j % SST, vs = j % VST;
        if (!mbar_wait_bounded(&k_empty[ks], ((j / KST) & 1) ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&k_full[ks], K_TILE);
        tma_load_3d(smem + OFF_K + ks * K_TILE, &tmK, &k_full[ks], 0, j * BN, h);
        if (!mbar_wait_bounded(&sc_empty[ss], ((j / SST) & 1) ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) {
          mbar_drain(&k_full[ks], (j / KST) & 1, p.err, kDevTimeoutDrain);
          break;
        }
        mbar_arrive_expect_tx(&sc_full[ss], BN * 4);
        bulk_load_1d(smem + OFF_SC + ss * BN * 4, p.ks + (int64_t)h * p.Sp + (int64_t)j * BN, BN * 4, &sc_full[ss]);
        if (!mbar_wait_bounded(&v_empty[vs], ((j / VST) & 1) ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) {
          mbar_drain(&k_full[ks], (j / KST) & 1, p.err, kDevTimeoutDrain);
          mbar_drain(&sc_full[ss], (j / SST) & 1, p.err, kDevTimeoutDrain);
          break;
        }
        mbar_arrive_expect_tx(&v_full[vs], V_TILE);
        uint8_t* vdst = smem + OFF_V + vs * V_TILE;
        tma_load_3d(vdst, &tmV, &v_full[vs], j * BN, 0, h);
        tma_load_3d(vdst + V_SLAB, &tmV, &v_full[vs], j * BN + 64, 0, h);
        last = j;
      }
      // drain: every load this thread issued lands before the CTA exits
      mbar_drain(q_full, 0, p.err, kDevTimeoutDrain);
      for (int j = last - KST + 1; j <= last; ++j)
        if (j >= 0) mbar_drain(&k_full[j % KST], (j / KST) & 1, p.err, kDevTimeoutDrain);
      for (int j = last - SST + 1; j <= last; ++j)
        if (j >= 0) mbar_drain(&sc_full[j % SST], (j / SST) & 1, p.err, kDevTimeoutDrain);
      for (int j = last - VST + 1; j <= last; ++j)
        if (j >= 0) mbar_drain(&v_full[j % VST], (j / VST) & 1, p.err, kDevTimeoutDrain);
    }
    if (warp == 1 && elect_one()) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t idq = idesc_i8(BM, BN);
      constexpr uint32_t idp = idesc_f16(BM, HD, BF16PV);
      auto issue_qk = [&](int t, int j) {
        const uint64_t da = smem_desc_k128(smem_u32(smem + OFF_Q + t * Q_TILE));
        const uint64_t db = smem_desc_k128(smem_u32(smem + OFF_K + (j % KST) * K_TILE));
#pragma unroll
        for (int k = 0; k < HD / 32; ++k)
          mma_i8(tmem_base + t * BN, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idq, k != 0);
        mma_commit(&s_full[t]);
      };
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, p.err, kDevTimeoutFull) &&
                mbar_wait_bounded(&k_full[0], 0, abort_flag, p.err, kDevTimeoutFull);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < NQ; ++t) issue_qk(t, 0);
        mma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int jn = j + 1;
        // next key tile's scores for both Q tiles first (each as soon as its softmax has read the current S),
        // so neither softmax group waits behind the other group's P.V
        if (jn < nkv) {
          if (!mbar_wait_bounded(&k_full[jn % KST], (jn / KST) & 1, abort_flag, p.err, kDevTimeoutFull)) break;
          for (int t = 0; t < NQ; ++t) {
            if (!mbar_wait_bounded(&s_free[t], j & 1, abort_flag, p.err, kDevTimeoutAccEmpty)) { ok = false; break; }
            tc_fence_after();
            issue_qk(t, jn);
          }
          if (!ok) break;
          mma_commit(&k_empty[jn % KST]);
        }
        if (!mbar_wait_bounded(&v_full[j % VST], (j / VST) & 1, abort_flag, p.err, kDevTimeoutFull)) break;
        for (int t = 0; t < NQ; ++t) {
          if (!mbar_wait_bounded(&p_full[t], j & 1, abort_flag, p.err, kDevTimeoutProbs)) { ok = false; break; }
          tc_fence_after();
          const uint8_t* pt = smem + OFF_P + t * P_TILE;
          const uint8_t* vt = smem + OFF_V + (j % VST) * V_TILE;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t da = smem_desc_k128(smem_u32(pt + (kk >> 2) * P_SLAB)) + (uint64_t)(2 * (kk & 3));
            const uint64_t db = smem_desc_k128(smem_u32(vt + (kk >> 2) * V_SLAB)) + (uint64_t)(2 * (kk & 3));
            mma_f16(tmem_base + NQ * BN + t * HD, da, db, idp, (j | kk) != 0);
          }
          mma_commit(&pv_done[t]);
        }
        if (!ok) break;
        mma_commit(&v_empty[j % VST]);
      }
      // every MMA this thread issued completes before TMEM is released
      mma_commit(mma_done);
      mbar_drain(mma_done, 0, p.err, kDevTimeoutDrain);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_HIGH));
    // -------------------------------------------------------------------- softmax warps
    const int g = (warp - 4) >> 2;        // Q tile of this warp
    const int quarter = warp & 3;         // TMEM lane quarter the warp may access
    const int rloc = quarter * 32 + lane; // row within the Q tile
    const int row = (qb * NQ + g) * BM + rloc;
    const bool rv = row < p.Sq;
    const float qsl = rv ? __fmul_rn(__ldg(p.qs + (int64_t)h * p.Sqp + row), p.scale_log2) : p.scale_log2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + g * BN;
    const uint32_t tO = tmem_base + lane_off + NQ * BN + g * HD;
    const uint32_t prow = smem_u32(smem + OFF_P + g * P_TILE) + rloc * 128;
    const uint32_t swz = rloc & 7;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[g], j & 1, abort_flag, p.err, kDevTimeoutScores))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[BN / 32][32];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld_32x32b_x32(tS + 32 * c, r[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[g]);
      const int nvalid = p.S - j * BN < BN ? p.S - j * BN : BN;
      if (DUMP && rv) {
        int32_t* dst = p.scores + ((int64_t)h * p.Sq + row) * p.S + (int64_t)j * BN;
        for (int i = 0; i < nvalid; ++i) dst[i] = (int32_t)r[i >> 5][i & 31];
      }
      const int ss = j % SST;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&sc_full[ss], (j / SST) & 1, abort_flag, p.err, kDevTimeoutScale))) {
        ok = false;
        break;
      }
      const float4* ksm = reinterpret_cast<const float4*>(smem + OFF_SC + ss * BN * 4);
      // s = (float)acc * ks.  |acc| <= 128 * 127 * 127 < 2^22, so the bits of acc + 1.5 * 2^23 read as a float
      // minus 1.5 * 2^23 is (float)acc exactly: an integer add and a paired subtract in place of the
      // quarter-rate int-to-float conversion.
      f2 s2[BN / 2];
      const f2 magic = pk(12582912.f, 12582912.f);
#pragma unroll
      for (int i4 = 0; i4 < BN / 4; ++i4) {
        const float4 kv = ksm[i4];
        const int i = 4 * i4;
        const f2 a = pk(__int_as_float((int)r[i >> 5][i & 31] + 0x4B400000),
                        __int_as_float((int)r[(i + 1) >> 5][(i + 1) & 31] + 0x4B400000));
        const f2 b = pk(__int_as_float((int)r[(i + 2) >> 5][(i + 2) & 31] + 0x4B400000),
                        __int_as_float((int)r[(i + 3) >> 5][(i + 3) & 31] + 0x4B400000));
        s2[2 * i4] = mul2(sub2(a, magic), pk(kv.x, kv.y));
        s2[2 * i4 + 1] = mul2(sub2(b, magic), pk(kv.z, kv.w));
      }
      if (nvalid < BN) {  // the last key tile: keys >= S take no part
#pragma unroll
        for (int i2 = 0; i2 < BN / 2; ++i2) {
          float lo, hi;
          upk(s2[i2], lo, hi);
          s2[i2] = pk(2 * i2 < nvalid ? lo : -INFINITY, 2 * i2 + 1 < nvalid ? hi : -INFINITY);
        }
      }
      float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i2 = 0; i2 < BN / 2; ++i2) {
        float lo, hi;
        upk(s2[i2], lo, hi);
        mq[i2 & 3] = max3f(mq[i2 & 3], lo, hi);
      }
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      __syncwarp();
      if (lane == 0) mbar_arrive(&sc_empty[ss]);
      const float m_new = __fmul_rn(mx, qsl);
      const bool move = m_new > m_used + kMoveMax;
      float alpha = 1.f;
      if (move) {
        alpha = ex2(m_used - m_new);
        m_used = m_new;
      }
      l = __fmul_rn(l, alpha);
      const f2 q2 = pk(qsl, qsl), nm2 = pk(-m_used, -m_used);
      uint32_t pk16[BN / 2];
      f2 la = pk(0.f, 0.f), lb = pk(0.f, 0.f);
#pragma unroll
      for (int i2 = 0; i2 < BN / 2; ++i2) {
        float t0, t1;
        upk(fma2(s2[i2], q2, nm2), t0, t1);
        const float p0 = ex2(t0), p1 = ex2(t1);
        if (i2 & 1) lb = add2(lb, pk(p0, p1));
        else la = add2(la, pk(p0, p1));
        pk16[i2] = pack_pv(p0, p1, BF16PV);
      }
      {
        float a0, a1, b0, b1;
        upk(la, a0, a1);
        upk(lb, b0, b1);
        l = __fadd_rn(l, __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(b0, b1)));
      }
      // P_g and O_g are free once the previous tile's P.V product has completed
      if (j > 0) {
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(&pv_done[g], (j - 1) & 1, abort_flag, p.err, kDevTimeoutPV))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, move)) {
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(tO + 32 * c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__fmul_rn(__uint_as_float(o[i]), alpha));
            tmem_st_32x32b_x32(tO + 32 * c, o);
          }
          tmem_wait_st();
        }
      }
#pragma unroll
      for (int sl = 0; sl < 2; ++sl)
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* q4 = &pk16[sl * 32 + c * 4];
          sts128(prow + sl * P_SLAB + ((c ^ swz) << 4), q4[0], q4[1], q4[2], q4[3]);
        }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
    }
    if (ok && nkv > 0 &&
        __all_sync(0xffffffffu, mbar_wait_bounded(&pv_done[g], (nkv - 1) & 1, abort_flag, p.err, kDevTimeoutPV))) {
      tc_fence_after();
      const float inv = l > 0.f ? __fdiv_rn(1.f, l) : 0.f;
      uint16_t* orow = p.out + ((int64_t)row * p.H + h) * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tO + 32 * c, o);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack_bf2(__fmul_rn(__uint_as_float(o[2 * i]), inv), __fmul_rn(__uint_as_float(o[2 * i + 1]), inv));
        if (rv) {
          uint4* d4 = reinterpret_cast<uint4*>(orow + 32 * c);
#pragma unroll
          for (int k = 0; k < 4; ++k) d4[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
        }
      }
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

// [H][S][128] int8 as a 3-D tensor (128 bytes, S rows, H heads); box 128 x 128 x 1, 128-byte swizzle.
static bool make_tmap_codes(CUtensorMap* m, const void* base, int64_t S, int64_t H) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)S, (cuuint64_t)H};
  const cuuint64_t strides[2] = {(cuuint64_t)HD, (cuuint64_t)(S * HD)};
  const cuuint32_t box[3] = {(cuuint32_t)HD, (cuuint32_t)BN, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [H][128][Sp] 16-bit V^T as a 3-D tensor (S keys, 128 dims, H heads); box 64 x 128 x 1, 128-byte swizzle.
static bool make_tmap_vt(CUtensorMap* m, const void* base, int64_t S, int64_t Sp, int64_t H) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)S, (cuuint64_t)HD, (cuuint64_t)H};
  const cuuint64_t strides[2] = {(cuuint64_t)(Sp * 2), (cuuint64_t)(Sp * 2 * HD)};
  const cuuint32_t box[3] = {64, (cuuint32_t)HD, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// scale_log2 as the reference computes it in f32: (1 / sqrt(128)) * LOG2_E (attn8.rs:625)
float attn_scale_log2() {
  volatile float d = 128.0f;
  const float r = 1.0f / sqrtf(d);
  return r * 1.44269504088896340736f;
}

template <bool BF16PV, bool DUMP>
static cudaError_t launch_attn_variant(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                       const AttnArgs& a, cudaStream_t st) {
  auto kern = attn_kernel<BF16PV, DUMP>;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  const unsigned grid = (unsigned)((int64_t)a.nqb * a.H);
  kern<<<grid, THREADS, SMEM, st>>>(tq, tk, tv, a);
  return cudaGetLastError();
}

cudaError_t launch_attention(const int8_t* q8, const float* qs, int64_t Sq, const int8_t* k8, const float* ks,
                             const uint16_t* vt, uint16_t* out, int64_t S, int64_t H, bool bf16pv,
                             int32_t* scores, int* err, cudaStream_t st) {
  if (S <= 0 || Sq <= 0 || H <= 0) return cudaSuccess;
  const int64_t Sp = (S + 127) / 128 * 128;
  CUtensorMap tq, tk, tv;
  if (!make_tmap_codes(&tq, q8, Sq, H) || !make_tmap_codes(&tk, k8, S, H) || !make_tmap_vt(&tv, vt, S, Sp, H))
    return cudaErrorInvalidValue;
  AttnArgs a{};
  a.qs = qs;
  a.ks = ks;
  a.out = out;
  a.scores = scores;
  a.S = (int)S;
  a.H = (int)H;
  a.Sp = (int)Sp;
  a.Sq = (int)Sq;
  a.Sqp = (int)((Sq + 127) / 128 * 128);
  a.nqb = (int)((Sq + NQ * BM - 1) / (NQ * BM));
  a.scale_log2 = attn_scale_log2();
  a.err = err;
  if (scores) {
    return bf16pv ? launch_attn_variant<true, true>(tq, tk, tv, a, st)
                  : launch_attn_variant<false, true>(tq, tk, tv, a, st);
  }
  return bf16pv ? launch_attn_variant<true, false>(tq, tk, tv, a, st)
                : launch_attn_variant<false, false>(tq, tk, tv, a, st);
}

}  // namespace h3q
