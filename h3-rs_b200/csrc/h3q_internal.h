// h3q_internal.h -- declarations shared by the kernel translation units and the C-ABI layer.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace h3q {

// Epilogue applied to the int32 tile accumulators (see gemm_i8.cu).
enum Epilogue : int {
  kEpiLinear = 0,        // out = acc*xs*ws + bias in the output kind (f32 / f16 / bf16)
  kEpiSwigluPairs = 1,   // gate/up interleaved column pairs -> silu(gate)*up, bf16 (gemm_s8, attn8.rs:334-337)
  kEpiSwigluHalves = 2,  // gate = column j, up = column F+j -> silu(gate)*up (int8_epilogue_swiglu, kernels.rs:353-373)
  kEpiGelu = 3,          // bf16(gelu_tanh(bf16 y))
  kEpiGateResid = 4,     // bf16(resid + bf16(y) * bf16(gate[idx[m], n]))  (gate_add fused, kernels.rs:418-428)
  kEpiAccI32 = 5,        // raw int32 accumulators
};

struct GemmArgs {
  int64_t M, N, K;        // A [M,K] int8, B [N,K] int8; N counts B rows
  const float* xs;        // [M] per-row activation scale
  const float* ws;        // [N] per-output-row weight scale, or one scalar
  int ws_per_row;
  const float* bias;      // [N] or null
  void* out;              // output (layout by epilogue)
  int out_kind;           // 0 f32, 1 f16, 2 bf16 (kEpiLinear, kEpiSwigluHalves)
  int epi;
  const float* gate;      // kEpiGateResid: f32 table [R, N]
  const uint32_t* gate_idx;  // kEpiGateResid: row of the table for each output row, or null (row 0)
  const uint16_t* resid;  // kEpiGateResid: bf16 [M, N]
  int* err;               // device error word
};

cudaError_t launch_quant_rows(const void* x, int kind, int8_t* q, float* scale, int64_t M, int64_t K, int order,
                              int* err, cudaStream_t st);
void fill_f32(float* p, float v, int64_t n, cudaStream_t st);
// bf16 x [M,K] -> bf16 rotate_activation(x, 256) (K % 256 == 0, K / 256 <= 64)
cudaError_t launch_rotate_bf16(const uint16_t* x, uint16_t* y, int64_t M, int64_t K, int* err, cudaStream_t st);
// out = silu(gate) * up with bf16-style re-rounding (weights.rs:806-816, ops.rs:39-44); y [rows, 2F] of kind
// `kind`, interleaved (g0,u0,g1,u1,...) or split halves (gates then ups); out [rows, F]
cudaError_t launch_swiglu(const void* y, void* out, int kind, int64_t rows, int64_t F, int interleaved, cudaStream_t st);
cudaError_t launch_gemm_i8(const int8_t* A, const int8_t* B, const GemmArgs& a, cudaStream_t st);
// rms_modulate (kernels.rs:376-401) of bf16 rows, fused into the quantizer (codes != nullptr) or alone (y)
cudaError_t launch_rms_modulate(const uint16_t* x, const uint16_t* w, float eps, const float* scale_tab,
                                const float* shift_tab, const uint32_t* idx, int8_t* codes, float* row_scale,
                                uint16_t* y, int64_t M, int64_t K, int* err, cudaStream_t st);
// GEMM whose output columns [n_offset, n_offset + a.N) of an [M, n_total] bf16 result go to every buffer of outs
constexpr int kMaxGatherRanks = 8;
cudaError_t launch_gemm_i8_allgather(const int8_t* A, const int8_t* B, const GemmArgs& a, void* const* outs, int n_out,
                                     int64_t n_total, int64_t n_offset, cudaStream_t st);
int sm_count(int device);
// the per-device error word kernels latch bounded-wait time-outs into (allocated once per device)
int* error_word_current();
// the status word of h3q_gemm_s8_static's fixed scratch array on the current device (reserving the array there on
// the first look-up), or null
int* static_status_word_current();

}  // namespace h3q
