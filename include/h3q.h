/*
 * h3q.h -- C ABI of the B200 (sm_100a) quantized-linear library that stands in for h3-rs's CUDA hot path.
 *
 * Every entry point takes raw device pointers, explicit sizes and a cudaStream_t (passed as void*), launches
 * asynchronously on that stream, allocates no device memory on the hot path (callers pass outputs and, where
 * needed, a workspace sized by the matching *_workspace_size function) and reports failures through a status
 * code plus h3q_last_error() text.  Nothing aborts the process.  A kernel that gives up waiting inside the
 * GPU latches a code into a per-device error word, read by h3q_device_status().
 *
 * Each declaration names the h3-rs function it replaces (paths inside the h3-rs source tree).  Tensors are
 * row-major and contiguous; "kind" codes follow kernels.rs's kind_of (kernels.rs:547-554): 0 = f32,
 * 1 = f16, 2 = bf16.
 */
#ifndef H3Q_H_
#define H3Q_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  H3Q_OK = 0,
  H3Q_ERR_ARG = 1,         /* invalid arguments: the reference's `bail!` checks, plus null/alignment checks */
  H3Q_ERR_UNSUPPORTED = 2, /* valid for the reference but outside what this build implements */
  H3Q_ERR_CUDA = 3,        /* a CUDA runtime / driver call failed */
  H3Q_ERR_TIMEOUT = 4,     /* a kernel gave up waiting on one of its own barriers (h3q_device_status) */
  H3Q_ERR_NCCL = 5,        /* NCCL missing or a collective failed (multi-GPU entry points) */
  H3Q_ERR_WORKSPACE = 6    /* the caller's workspace is smaller than *_workspace_size */
} h3q_status;

enum { H3Q_KIND_F32 = 0, H3Q_KIND_F16 = 1, H3Q_KIND_BF16 = 2 };

/* Epilogues of h3q_gemm_s8_quantized. */
enum {
  H3Q_EPI_LINEAR = 0,        /* out[m,n] = acc*xs[m]*ws[n] + bias[n]   (gemm_s8 / int8_epilogue)            */
  H3Q_EPI_SWIGLU_PAIRS = 1,  /* interleaved (gate, up) columns -> out[m, n/2], bf16 (attn8.rs:334-337)       */
  H3Q_EPI_SWIGLU_HALVES = 2, /* gate = column j, up = column N/2 + j -> out[m, j] (kernels.rs:353-373)      */
  H3Q_EPI_GELU_TANH = 3,     /* out = gelu_tanh(bf16 y), bf16 (ops.rs:46-48 applied to the linear output)  */
  H3Q_EPI_GATE_RESID = 4,    /* out = resid + bf16(y) * bf16(gate[idx[m], n]), bf16 (kernels.rs:418-428)   */
  H3Q_EPI_ACC_I32 = 5        /* raw int32 accumulators [M, N] (the cuBLASLt path's int32 result)          */
};

/* Text of the last error raised on the calling thread ("" if none). */
const char* h3q_last_error(void);

/* Library version string. */
const char* h3q_version(void);

/* attn8::available_arch (attn8.rs:584-589): 1 when `device` can run these kernels (sm_100), else 0. */
int h3q_available_arch(int device);

/* Per-device set-up, once per device and optional: creates the state the entry points otherwise create on their
 * first call on a device (the device error word, a 4-byte allocation, and the SM count), so that the first call
 * of an entry point does not allocate it, and reserves the fixed 64 MiB scratch array of h3q_gemm_s8_static on
 * the device (the array's module loads lazily; call h3q_init before another pool takes the GPU's memory).
 * H3Q_ERR_UNSUPPORTED on a device that is not an sm_100 GPU.  Safe to call again. */
h3q_status h3q_init(int device);

/* Failure-path self-test (no counterpart in the reference; the reference's kernels have no device-side error
 * reporting).  Launches one CTA with the roles of a pipeline kernel that waits on a barrier nothing completes:
 * its producer's wait gives up after `limit_ns` (0 < limit_ns <= 1e9) through the same bounded-wait code every
 * kernel of the library uses, the other roles leave on the CTA's abort flag, TMEM is freed and the kernel
 * returns.  The time-out is latched into the device error word (target 0, read by h3q_device_status) or the
 * static-scratch status word (target 1, read by h3q_gemm_s8_static_status).  `done` (device int, zeroed by the
 * caller, or NULL) receives 1 when the CTA reached its exit path plus 2 when the producer's wait gave up. */
h3q_status h3q_selftest_wait_timeout(int target, uint64_t limit_ns, int* done, void* stream);

/* kernels::can_fuse_rotation (kernels.rs:1081-1085): whether the rotation fuses into the quantizer for an
 * input width k and ConvRot group size.  Always on here (group 256, k % 256 == 0, k / 256 <= 64); the
 * reference gates it behind H3_FUSED_ROT=1 because its butterfly was slow on RTX 4090. */
int h3q_can_fuse_rotation(size_t k, size_t group);

/* Reads and clears the error word that kernels on `device` latch when a bounded wait runs out.  Synchronizes
 * the device.  *code receives 0 when no kernel reported a failure.  Returns H3Q_ERR_TIMEOUT if one did. */
h3q_status h3q_device_status(int device, int* code);

/* kernels::quant_rows_raw (kernels.rs:1133-1161): x [m,k] of kind x_kind -> int8 codes q [m,k] and f32
 * scales [m].  rotate selects the fused ConvRot-256 rotation; like the reference, bf16 input with
 * k / 256 <= 56 uses the quant_rows_i8_rot2 summation order (kernels.rs:220-293), any other rotated call the
 * quant_rows_i8_rot order (kernels.rs:166-213).  Rotation needs k % 256 == 0 and k / 256 <= 64. */
h3q_status h3q_quant_rows_i8(const void* x, int x_kind, int8_t* q, float* scale, int64_t m, int64_t k, int rotate,
                             void* stream);

/* Workspace bytes h3q_gemm_s8 needs for an [m,k] activation (int8 codes + f32 row scales). */
size_t h3q_gemm_s8_workspace_size(int64_t m, int64_t k);

/* attn8::gemm_s8 (attn8.rs:570-581, kernel attn8.rs:258-344): bf16 x [m,k] is quantized per row (optionally
 * ConvRot-rotated) and multiplied by the int8 weight w [n,k]:
 *   out[m,n] = bf16(sum_k q[m,k] w[n,k] * xs[m] * ws[n] + bias[n])
 * ws has ws_numel entries: per output row when ws_numel == n && n > 1, else ws[0] for all (attn8.rs:553).
 * bias is f32 [n] or NULL.  swiglu: rows of w interleave (gate, up) pairs and out is [m, n/2] =
 * silu(gate) * up.  Requires k % 64 == 0 (the reference's check, attn8.rs:571-573). */
h3q_status h3q_gemm_s8(const uint16_t* x, const int8_t* w, const float* ws, int64_t ws_numel, const float* bias,
                       uint16_t* out, int64_t m, int64_t n, int64_t k, int swiglu, int rotate, void* workspace,
                       size_t workspace_bytes, void* stream);

/* gemm_s8 on activations in host memory (no counterpart in the reference, whose ops take device tensors): the
 * rows are processed in chunks whose copy in (one copy stream), GEMM (the caller's stream) and copy out (a second
 * copy stream) overlap, double-buffered, so both PCIe directions and the tensor cores work at once.  Set-up
 * allocates two chunk buffers for inputs of up to max_k columns and outputs of up to max_n columns, the GEMM's
 * workspace and the streams. */
typedef struct h3q_host_pipeline h3q_host_pipeline;
h3q_status h3q_host_pipeline_create(int64_t chunk_rows, int64_t max_k, int64_t max_n, h3q_host_pipeline** out);
/* The same with in_slots input and out_slots output chunk buffers (each in [2, 4096]; the plain create uses 2 and 2).
 * More input buffers let the copies in run further ahead of the GEMMs. */
h3q_status h3q_host_pipeline_create_ex(int64_t chunk_rows, int64_t max_k, int64_t max_n, int in_slots, int out_slots,
                                       h3q_host_pipeline** out);
void h3q_host_pipeline_destroy(h3q_host_pipeline* p);
/* out_host [m, n] (or [m, n/2] with swiglu) = h3q_gemm_s8(x_host [m, k]) with host buffers (pinned, for the copies
 * to overlap).  Ordered after the work already on `stream`; `stream` waits for the last copy out, so the output
 * is in host memory once `stream` has reached that point, and one call's output can feed the next call. */
h3q_status h3q_host_pipeline_gemm_s8(h3q_host_pipeline* p, const uint16_t* x_host, const int8_t* w, const float* ws,
                                     int64_t ws_numel, const float* bias, uint16_t* out_host, int64_t m, int64_t n,
                                     int64_t k, int swiglu, int rotate, void* stream);
/* One linear of a batch: the arguments of h3q_host_pipeline_gemm_s8. */
typedef struct h3q_host_linear {
  const uint16_t* x_host;
  const int8_t* w;
  const float* ws;
  int64_t ws_numel;
  const float* bias;
  uint16_t* out_host;
  int64_t m, n, k;
  int swiglu, rotate;
} h3q_host_linear;
/* The `count` linears of `items` as one pipelined sequence (a DiT block's linears on host activations): linear
 * i + 1 copies in while linear i still computes and copies out, where separate calls would wait for each call's
 * last copy out.  A linear whose host input overlaps the host output of an earlier linear of the batch starts its
 * copies in after every copy out enqueued before it.  Every item is checked before anything is enqueued; the batch
 * as a whole keeps the stream contract of h3q_host_pipeline_gemm_s8 (which is this call with one item). */
h3q_status h3q_host_pipeline_run(h3q_host_pipeline* p, const h3q_host_linear* items, int count, void* stream);

/* Workspace bytes h3q_int8_linear_ex needs. */
size_t h3q_int8_linear_workspace_size(int64_t m, int64_t k);

/* kernels::int8_linear_ex (kernels.rs:1088-1097, op kernels.rs:955-1070): x [m,k] (kind x_kind) quantized per
 * row (rotated with the quant_rows_i8_rot order when rotate && k % 256 == 0 && k / 256 <= 64, otherwise
 * unrotated, exactly as the reference), times w [n,k], epilogue int8_epilogue or, with swiglu, the split-half
 * int8_epilogue_swiglu (gate = column j, up = column n/2 + j), written in out_kind.  The reference's int32
 * accumulator round trip through HBM is fused away.  Requires k % 4 == 0 and an output width % 4 == 0
 * (kernels.rs:977, :1062); this build also needs k % 16 == 0. */
h3q_status h3q_int8_linear_ex(const void* x, int x_kind, const int8_t* w, const float* scale, int64_t scale_numel,
                              const float* bias, void* out, int out_kind, int64_t m, int64_t n, int64_t k, int swiglu,
                              int rotate, void* workspace, size_t workspace_bytes, void* stream);

/* The tensor-core GEMM on already-quantized activations a [m,k] (scales xs [m]) and weight w [n,k], with any
 * epilogue above.  The building block of h3q_gemm_s8 / h3q_int8_linear_ex, exported so callers can reuse one
 * quantization across several weights (the DiT's fused qkv and gate/up share their input).
 *   H3Q_EPI_GATE_RESID: gate is an f32 table [R, n], gate_idx u32 [m] selects its row (NULL: row 0), resid is
 *   bf16 [m, n]; out = bf16(resid + bf16(y) * bf16(gate)).  out_kind is ignored for bf16-only epilogues. */
h3q_status h3q_gemm_s8_quantized(const int8_t* a, const float* xs, const int8_t* w, const float* ws,
                                 int64_t ws_numel, const float* bias, void* out, int out_kind, int64_t m, int64_t n,
                                 int64_t k, int epilogue, const float* gate, const uint32_t* gate_idx,
                                 const uint16_t* resid, void* stream);

/* Raw int32 accumulators acc[m,n] = sum_k a[m,k] w[n,k] (the cuBLASLt IMMA result of kernels.rs:1026-1044). */
h3q_status h3q_gemm_s8_acc(const int8_t* a, const int8_t* w, int32_t* acc, int64_t m, int64_t n, int64_t k,
                           void* stream);

/* kernels::dequant_i8 (kernels.rs:607-638, kernel :40-49): out[r,c] = q[r,c] * scale[r or 0] in out_kind;
 * per row when scale_numel == rows && rows > 1 (kernels.rs:616). */
h3q_status h3q_dequant_i8(const int8_t* q, const float* scale, int64_t scale_numel, void* out, int out_kind,
                          int64_t rows, int64_t cols, void* stream);

/* kernels::dequant_nvfp4 (kernels.rs:640-680, kernel :65-81): q [rows, k/2] (even column in the high nibble),
 * block scales e4m3 in the 128x4 swizzled layout, f32 global scale (device pointer) -> out [rows, k]. */
h3q_status h3q_dequant_nvfp4(const uint8_t* q, const uint8_t* block_scale, const float* global_scale, void* out,
                             int out_kind, int64_t rows, int64_t k, void* stream);

/* kernels::gate_add (kernels.rs:849-883, kernel :418-428): out = x + y * gate[idx[s], c] (gate rounded to
 * the kind of x), x/y/out [s, c] of kind `kind` (f16 or bf16), gate f32 [R, c], idx u32 [s]. */
h3q_status h3q_gate_add(const void* x, const void* y, int kind, const float* gate, const uint32_t* idx, void* out,
                        int64_t s, int64_t c, void* stream);

/* rotate_activation(x, 256) (weights.rs:482-489) for bf16 rows: y = x . H256 per 256-column group (H256 the
 * normalised regular Hadamard of weights.rs:441-465), formed by the quantizer's f32 butterfly in its rot2 order and
 * rounded to bf16 once.  The reference multiplies by H in bf16 through cuBLAS, whose rounding no reference test
 * pins.  x, y bf16 [m, k]; k % 256 == 0, k <= 16384. */
h3q_status h3q_rotate_activation(const uint16_t* x, uint16_t* y, int64_t m, int64_t k, void* stream);

/* swiglu_interleaved (weights.rs:806-816; interleaved = 1: gate and up in adjacent columns) and ops::swiglu
 * (ops.rs:39-44; interleaved = 0: gate = columns [0, f), up = [f, 2f)): out [rows, f] = silu(gate) * up with the
 * bf16 re-roundings of the reference's epilogue, y [rows, 2f] and out of kind `kind` (0 f32, 1 f16, 2 bf16). */
h3q_status h3q_swiglu(const void* y, void* out, int kind, int64_t rows, int64_t f, int interleaved, void* stream);

/* Workspace bytes h3q_nvfp4_linear needs (the AWQ-scaled activations and, for narrow outputs, split-K partials). */
size_t h3q_nvfp4_linear_workspace_size(int64_t m, int64_t n, int64_t k, int has_pre_quant_scale);

/* QLinear::apply for an NVFP4 layer (weights.rs:612-635; weight decode kernels.rs:65-81), fused:
 *   x2 = bf16(x * pre_quant_scale)      (AWQ, bf16 [k] or NULL; weights.rs:617-620)
 *   out = bf16(x2 @ W^T) (+ bias)       (bias f32 [n] added in bf16, weights.rs:633-635)
 * with W decoded from q [n, k/2] (even column in the high nibble), e4m3 block scales in the 128x4 swizzled layout
 * and the f32 global scale (device pointer) inside the GEMM.  x bf16 [m, k], out bf16 [m, n].  This build needs
 * k % 64 == 0 and n % 128 == 0 (the text encoder's 5120 / 25600). */
h3q_status h3q_nvfp4_linear(const uint16_t* x, const uint16_t* pre_quant_scale, const uint8_t* q,
                            const uint8_t* block_scale, const float* global_scale, const float* bias, uint16_t* out,
                            int64_t m, int64_t n, int64_t k, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * QLinear: the layer-level dispatch of weights.rs (QLinear::prepare / run / run_swiglu / try_gemm_s8 /
 * apply_int8, weights.rs:833-947) over the entry points above.  The reference reads its switches from the
 * environment once (H3_INT8 weights.rs:821, H3_GEMM :891, H3_ROT :899, H3_FUSED_ROT kernels.rs:1083); here they
 * are an explicit struct, defaults = the reference's defaults with no variable set. */
enum { H3Q_FMT_DENSE = 0, H3Q_FMT_INT8 = 1, H3Q_FMT_NVFP4 = 2 }; /* QFormat (weights.rs:389-397) */

typedef struct {
  int format;             /* H3Q_FMT_* */
  int convrot;            /* ConvRot group size (QFormat::Int8 { convrot }), 0 = none */
  int interleaved;        /* rows of the weight interleave (gate, up) pairs (QLinear::interleaved) */
  int n_loras;            /* attached LoRA deltas (the runtime LoRA path is not part of this library) */
  int64_t out_features, in_features;
  const int8_t* weight;   /* int8 [out_features, in_features] */
  const float* scale;     /* f32 [out_features] or scalar */
  int64_t scale_numel;
  const float* bias;      /* f32 [out_features] or NULL */
} h3q_qlinear;

typedef struct {
  int int8;               /* H3_INT8 != "0": int8 weights run on int8 tensor cores (default 1) */
  int gemm_fused;         /* H3_GEMM != "cublaslt": the fused gemm_s8 path (default 1) */
  int rot_fused;          /* H3_ROT != "gemm": ConvRot fused into gemm_s8's quantizer (default 1) */
  int fused_rot_linear;   /* H3_FUSED_ROT == "1": ConvRot fused into int8_linear_ex's quantizer (default 0) */
} h3q_switches;

/* Dispatch decision of h3q_qlinear_forward (bit flags). */
enum {
  H3Q_PATH_GEMM_S8 = 1,          /* attn8::gemm_s8 (try_gemm_s8 applied) */
  H3Q_PATH_INT8_LINEAR = 2,      /* kernels::int8_linear_ex (the cuBLASLt-path semantics) */
  H3Q_PATH_ROTATE_FUSED = 4,     /* ConvRot inside the quantizer */
  H3Q_PATH_ROTATE_SEPARATE = 8,  /* rotate_activation first (bf16), then an unrotated quantizer */
  H3Q_PATH_SWIGLU_FUSED = 16,    /* SwiGLU in the GEMM epilogue */
  H3Q_PATH_SWIGLU_AFTER = 32     /* SwiGLU as a separate pass over the linear output */
};

/* The reference's defaults (no environment variable set). */
h3q_switches h3q_default_switches(void);

/* Which path h3q_qlinear_forward takes for this layer, an activation of kind x_kind and swiglu (0 = run,
 * 1 = run_swiglu); H3Q_PATH_* flags, or a negative h3q_status when the layer is not served here (dense / NVFP4
 * layers, int8 disabled, LoRA deltas on a path that would need them).  Host logic only, no device work. */
int h3q_qlinear_plan(const h3q_qlinear* layer, int x_kind, int64_t in_width, int swiglu, const h3q_switches* sw);

/* Workspace bytes h3q_qlinear_forward needs for `rows` activation rows. */
size_t h3q_qlinear_workspace_size(const h3q_qlinear* layer, int x_kind, int64_t rows, int swiglu,
                                  const h3q_switches* sw);

/* QLinear::forward_raw / run (swiglu = 0) and run_swiglu (swiglu = 1) for an int8 layer: x [rows, in_features]
 * of kind x_kind -> out [rows, out_features] (or [rows, out_features / 2] with swiglu) in the activation kind. */
h3q_status h3q_qlinear_forward(const h3q_qlinear* layer, const void* x, int x_kind, int64_t rows, int swiglu,
                               void* out, void* workspace, size_t workspace_bytes, const h3q_switches* sw,
                               void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * ComfyUI checkpoints: the safetensors files the reference reads with SafeFile (weights.rs:23-139) and the layer
 * description QLinear::load derives from them (weights.rs:493-534).  Host code; uploads use the caller's stream.
 * ------------------------------------------------------------------------------------------------------- */
enum { /* storage dtypes (SafeFile::storage_dtype, weights.rs:99-112) */
  H3Q_DT_F32 = 0, H3Q_DT_F16 = 1, H3Q_DT_BF16 = 2, H3Q_DT_I8 = 3, H3Q_DT_U8 = 4, H3Q_DT_F8_E4M3 = 5,
  H3Q_DT_BOOL = 6, H3Q_DT_I32 = 7, H3Q_DT_I64 = 8, H3Q_DT_F64 = 9
};
typedef struct h3q_checkpoint h3q_checkpoint;

/* SafeFile::open (weights.rs:33-58): reads and checks the header (every tensor's offsets inside the file and its
 * byte count equal to its element count times its dtype size); tensor names lose the "model.diffusion_model."
 * prefix as in the reference.  Close with h3q_checkpoint_close. */
h3q_status h3q_checkpoint_open(const char* path, h3q_checkpoint** out);
void h3q_checkpoint_close(h3q_checkpoint* f);
/* Tensor names in sorted order (i < count); NULL past the end. */
int64_t h3q_checkpoint_count(const h3q_checkpoint* f);
const char* h3q_checkpoint_name(const h3q_checkpoint* f, int64_t i);
/* SafeFile::has (weights.rs:60-62): 1 if the tensor exists. */
int h3q_checkpoint_has(const h3q_checkpoint* f, const char* name);
/* The "__metadata__" value of `key` (non-string values as their JSON text), or NULL. */
const char* h3q_checkpoint_metadata(const h3q_checkpoint* f, const char* key);
/* SafeFile::info / shape (weights.rs:64-78): storage dtype (H3Q_DT_*), rank, shape (up to 8 dims), bytes. */
h3q_status h3q_checkpoint_info(const h3q_checkpoint* f, const char* name, int* dtype, int* ndim, int64_t* shape,
                               uint64_t* nbytes);
/* SafeFile::read_into (weights.rs:80-87): the tensor's bytes into host memory (pread). */
h3q_status h3q_checkpoint_read(const h3q_checkpoint* f, const char* name, void* dst, uint64_t dst_bytes);
/* The tensor's bytes to device memory: pread into two pinned staging buffers whose copies run on `stream`, so
 * reading and copying overlap; returns when the data is on the device.  With interleave_halves the first
 * dimension's two halves (gate rows, then up rows) land interleaved, row i of each half at rows 2i and 2i + 1:
 * QLinear::interleave_swiglu (weights.rs:679-687, :765-800) done by the copy itself. */
h3q_status h3q_checkpoint_upload(const h3q_checkpoint* f, const char* name, void* dst, uint64_t dst_bytes,
                                 int interleave_halves, void* stream);

typedef struct {
  int format;             /* H3Q_FMT_* from "<prefix>.comfy_quant" ({"format": ...}; absent: dense) */
  int convrot;            /* int8_tensorwise with "convrot": true -> "convrot_groupsize" (default 256); else 0 */
  int64_t out_features;   /* weight rows */
  int64_t in_features;    /* weight columns (NVFP4: twice the packed byte columns) */
  int weight_dtype;       /* H3Q_DT_* of "<prefix>.weight" */
  int scale_dtype;        /* H3Q_DT_* of "<prefix>.weight_scale" (int8: f32 per row or scalar; NVFP4: e4m3 blocks) */
  int64_t scale_numel;    /* elements of "<prefix>.weight_scale" */
  int has_bias;           /* "<prefix>.bias" exists */
  int has_pre_quant_scale;/* NVFP4 AWQ "<prefix>.pre_quant_scale" exists ("<prefix>.weight_scale_2" is required) */
} h3q_qlinear_spec;

/* QLinear::load's format decision (weights.rs:495-525) for the layer at `prefix`: which tensors the layer has and
 * how to run it.  Unknown formats fail with the reference's message. */
h3q_status h3q_checkpoint_qlinear(const h3q_checkpoint* f, const char* prefix, h3q_qlinear_spec* spec);

/* One low-rank delta scale * (b @ a) of a layer (LoraDelta, weights.rs:399-405; lora.rs:15-23): a = lora_down /
 * lora_A [rank, in_features], b = lora_up / lora_B [out_features, rank], row-major device tensors;
 * scale = alpha / rank * strength (lora.rs:56-62, dit.rs:664), applied as an f32 multiply. */
typedef struct {
  const void* a;
  const void* b;
  int64_t rank;
  int dtype;     /* H3Q_DT_BF16 (the reference loads its factors as bf16, lora.rs:51-53), H3Q_DT_F16 or H3Q_DT_F32 */
  double scale;
} h3q_lora;

/* Workspace bytes for h3q_lora_merge_i8 to merge all n rows in one pass (a smaller workspace merges in row
 * chunks; one row needs 256 + 4 k bytes). */
size_t h3q_lora_merge_i8_workspace_size(int64_t n, int64_t k);

/* QLinear::merge_loras for an int8 layer (weights.rs:716-757): per row, dequantize (q * s, w_scale per row when
 * scale_numel == n, else one scalar), undo the ConvRot rotation (convrot 256; 0 = none), add the deltas in order,
 * rotate again, and requantize: s' = max(max|w| * f32(1/127), 1e-30), q' = clamp(round(w / s'), -128, 127).
 * w_out [n, k] int8 and scale_out [n] f32 may be w and w_scale (in place) unless w_scale is a scalar.  The
 * reference leaves the order of its f32 matmul sums to the BLAS; this build's order (k-ordered fma chains for the
 * deltas, the quantizer's butterfly for the rotations) is the one its oracle restates.  With n_loras == 0 nothing
 * is written, as the reference returns early (weights.rs:693-695).  The workspace must be 256-byte aligned.  The
 * caller merges before QLinear::interleave_swiglu, as the reference does (dit.rs:599-616). */
h3q_status h3q_lora_merge_i8(const int8_t* w, const float* w_scale, int64_t scale_numel, int convrot,
                             const h3q_lora* loras, int n_loras, int8_t* w_out, float* scale_out, int64_t n, int64_t k,
                             void* workspace, size_t workspace_bytes, void* stream);

/* QLinear::merge_loras for a dense layer (weights.rs:710-715): w_out = dtype(f32(w) + sum of the deltas), w and
 * w_out [n, k] of dtype H3Q_DT_F32, H3Q_DT_F16 or H3Q_DT_BF16 (w_out may be w). */
h3q_status h3q_lora_merge_dense(const void* w, int dtype, const h3q_lora* loras, int n_loras, void* w_out, int64_t n,
                                int64_t k, void* stream);

/* Weight streaming (weights.rs:185-273 upload_u8_async on a per-device copy stream; the per-block fetch of
 * dit.rs:1160-1186): for weights that stay in host memory (pinned, for the copies to overlap), a ring of device
 * slots filled on the streamer's own copy stream.  Everything is ordered by events on the device, the host never
 * waits: a fetch into a slot waits (on the copy stream) for the release of the slot's previous contents and makes
 * the compute stream wait for its copy.  The ring's slot count bounds how far uploads run ahead. */
typedef struct h3q_streamer h3q_streamer;
/* Set-up on the current device: `slots` device slots of slot_bytes (rounded up to 256) and a copy stream. */
h3q_status h3q_streamer_create(size_t slot_bytes, int slots, h3q_streamer** out);
/* Waits for the streamer's outstanding work and frees it. */
void h3q_streamer_destroy(h3q_streamer* s);
/* Bytes per slot (after rounding). */
size_t h3q_streamer_slot_bytes(const h3q_streamer* s);
/* Copies the n host regions src[i] (bytes[i] each) into the ring's next slot, each region at a 256-byte aligned
 * offset, and returns the slot index and each region's device address (dst[i]).  Kernels enqueued on
 * compute_stream after the call see the data: the call places the wait for the copy on compute_stream at this
 * point, so enqueue the current layer's kernels first and fetch the next layer after them, and the copy overlaps
 * them.  The slot must not be held: release each slot (below) before the ring comes back to it. */
h3q_status h3q_streamer_fetch(h3q_streamer* s, const void* const* src, const size_t* bytes, int n,
                              void* compute_stream, int* slot, void** dst);
/* Marks the slot free once compute_stream reaches this point: call it after enqueuing the slot's last reader. */
h3q_status h3q_streamer_release(h3q_streamer* s, int slot, void* compute_stream);

/* kernels::rms_modulate (kernels.rs:1201-1204, kernel :376-401) for bf16 rows: out = bf16(fma(n, 1 + bf16(scale[
 * idx[s], c]), bf16(shift[idx[s], c]))) with n = bf16((x * rsqrt(mean(x^2) + eps)) * w[c]), the mean summed in
 * the reference kernel's order.  x, out bf16 [S, C]; w bf16 [C]; scale, shift f32 [R, C]; idx u32 [S].  This build
 * needs C % 256 == 0 and C <= 16384. */
h3q_status h3q_rms_modulate(const uint16_t* x, const uint16_t* w, float eps, const float* scale, const float* shift,
                            const uint32_t* idx, uint16_t* out, int64_t S, int64_t C, void* stream);

/* rms_modulate fused with the quantizer the next linear applies to its output (no counterpart in the reference,
 * which writes the bf16 row to memory and reads it back): the modulated row is ConvRot-rotated and quantized per
 * row exactly as h3q_quant_rows_i8(rotate = 1) would quantize h3q_rms_modulate's output (rot2 order for
 * C / 256 <= 56), giving int8 codes [S, C] and f32 row scales [S] for h3q_gemm_s8_quantized.  Same limits. */
h3q_status h3q_rms_modulate_quant(const uint16_t* x, const uint16_t* w, float eps, const float* scale,
                                  const float* shift, const uint32_t* idx, int8_t* codes, float* row_scale, int64_t S,
                                  int64_t C, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * int8 attention (attn8.rs): non-causal SageAttention-style attention over [S, H, 128] bf16 q / k / v, int8
 * Q.K^T with K smoothed by its mean over the sequence, online softmax, 16-bit P.V with f32 accumulation.
 * Layouts of the stage buffers: codes int8 [H, S, 128]; scales f32 [H, Sp] with Sp = roundup(S, 128) (entries
 * S..Sp-1 zero); V^T 16-bit [H, 128, Sp].  Output bf16 [S, H, 128].
 * ------------------------------------------------------------------------------------------------------- */
enum {
  H3Q_ATTN_SCALE_TOKEN = 0,    /* per-token Q / K scales (QuantHeads, attn8.rs:69-93)                        */
  H3Q_ATTN_SCALE_BLOCK128 = 1, /* one scale per 128-token block of a head (every token of the block holds it) */
  H3Q_ATTN_PV_F16 = 0,         /* P and V in f16 (attn8.rs:55-65, :100-104)                                  */
  H3Q_ATTN_PV_BF16 = 2         /* P and V in bf16                                                            */
};

/* available(q) (attn8.rs:591-602): 1 if the int8 attention runs for head_dim on `device` with activations of
 * x_kind (head_dim 128, bf16, an sm_100 device), else 0. */
int h3q_attention_available(int64_t head_dim, int x_kind, int device);

/* Workspace bytes of h3q_attention / h3q_attention_qkv for S tokens and H heads (flags: H3Q_ATTN_*). */
size_t h3q_attention_workspace_size(int64_t S, int64_t H, int flags);

/* attention(q, k, v) (attn8.rs:611-615): q, k, v bf16 [S, H, 128] contiguous -> out bf16 [S, H, 128]. */
h3q_status h3q_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int64_t S,
                         int64_t H, int flags, void* workspace, size_t workspace_bytes, void* stream);

/* attention_qkv(q, k, qkv, v_col) (attn8.rs:604-609): V read from the fused qkv activation [S, qkv_width] at
 * column v_col (head h at v_col + 128 h). */
h3q_status h3q_attention_qkv(const uint16_t* q, const uint16_t* k, const uint16_t* qkv, int64_t qkv_width,
                             int64_t v_col, uint16_t* out, int64_t S, int64_t H, int flags, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Workspace bytes of h3q_attention_rows. */
size_t h3q_attention_rows_workspace_size(int64_t Sq, int64_t S, int64_t H, int flags);

/* attention_qkv / attention for a block of Sq query rows against all S keys (no counterpart in the reference,
 * which attends all rows at once): q bf16 [Sq, H, 128]; k bf16 [S, H, 128]; V from rows of v_src [S,
 * v_row_stride] at column v_col (head h at v_col + 128 h) -> out bf16 [Sq, H, 128].  The rows of the result equal
 * the matching rows of h3q_attention on the whole sequence (per-token scales; with H3Q_ATTN_SCALE_BLOCK128 the
 * query blocks start at the first row of q).  It is the per-GPU step of query-sharded multi-GPU attention. */
h3q_status h3q_attention_rows(const uint16_t* q, int64_t Sq, const uint16_t* k, const uint16_t* v_src,
                              int64_t v_row_stride, int64_t v_col, uint16_t* out, int64_t S, int64_t H, int flags,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Per-head RMSNorm + split-half RoPE, qk_norm_rope (kernels.rs:86-126; op and launch :682-800): for every token s
 * and head h, the D <= 256 values x[s * row_stride + col_off + h * head_stride + d] (bf16) -> out bf16 [S, H, D].
 * do_norm: v * rsqrtf(mean(v^2) + eps) * w[d] (w bf16 [D], or NULL for none); then, with a table, the first rot
 * dims are rotated in halves: rope f32 [2, S, rot/2] holds cos then sin (NULL: no rotation).  rot even, <= D.
 * Bit-exact with the reference's kernel (same reduction order, same hardware rsqrtf, the same FMA contraction). */
h3q_status h3q_qk_norm_rope(const uint16_t* x, int64_t row_stride, int64_t col_off, int64_t head_stride,
                            const uint16_t* w, int do_norm, float eps, const float* rope, int rot, uint16_t* out,
                            int64_t S, int64_t H, int64_t D, void* stream);

/* The DiT's attention step, attend (dit.rs:741-757) with head_dim 128: q = qk_norm_rope(qkv, q_col), k =
 * qk_norm_rope(qkv, k_col) (norm weights q_norm / k_norm when do_norm, rope table and rot as h3q_qk_norm_rope),
 * then attention_qkv(q, k, qkv, v_col) -> out bf16 [S, H, 128].  The normalised, rotated q and k never reach
 * memory: the rotation runs inside the K mean and the Q / K quantisation, and the result equals that sequence
 * bit for bit.  qkv bf16 [S, qkv_width], 16-byte aligned, width and q / k columns multiples of 8; norm weights
 * 16-byte aligned; rot % 8 == 0
 * (other rot: H3Q_ERR_UNSUPPORTED).  Workspace: h3q_attention_workspace_size(S, H, flags). */
h3q_status h3q_attend_qkv(const uint16_t* qkv, int64_t qkv_width, int64_t q_col, int64_t k_col, int64_t v_col,
                          const uint16_t* q_norm, const uint16_t* k_norm, int do_norm, float eps, const float* rope,
                          int rot, uint16_t* out, int64_t S, int64_t H, int flags, void* workspace,
                          size_t workspace_bytes, void* stream);

/* The stages, for callers that keep the intermediates. */
/* Workspace bytes of h3q_attn_kmean (the per-chunk column sums). */
size_t h3q_attn_kmean_workspace_size(int64_t S, int64_t H);
/* ColMean then `/ S` (attn8.rs:429-455, :622): kmean f32 [H, 128] = column sums of k [S, H*128] in a fixed order
 * (chunks of ceil(S / min(128, S)) rows, chunk sums added in chunk order) times (float)(1 / S). */
h3q_status h3q_attn_kmean(const uint16_t* k, int64_t S, int64_t H, float* kmean, void* workspace,
                          size_t workspace_bytes, void* stream);
/* QuantHeads (attn8.rs:395-427, kernel :69-93): x bf16 [S, H, 128] minus mean [H, 128] (NULL: none) -> codes
 * [H, S, 128] (clamp +-127) and scales [H, Sp]; flags H3Q_ATTN_SCALE_*. */
h3q_status h3q_attn_quant_heads(const uint16_t* x, const float* mean, int8_t* codes, float* scales, int64_t S,
                                int64_t H, int flags, void* stream);
/* VToF16 (attn8.rs:457-486, kernel :55-65), transposed: rows of [S, row_stride] bf16 at column col_off ->
 * V^T [H, 128, Sp] in f16 (cvt.rn) or, with H3Q_ATTN_PV_BF16, bf16. */
h3q_status h3q_attn_v_layout(const uint16_t* src, int64_t row_stride, int64_t col_off, uint16_t* vt, int64_t S,
                             int64_t H, int flags, void* stream);
/* Attn (attn8.rs:488-520, kernel :107-246) on prepared stages.  If `scores` is not NULL it also receives the
 * int32 Q.K^T accumulators [H, S, S] (a diagnostic form for small S). */
h3q_status h3q_attention_core(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks,
                              const uint16_t* vt, uint16_t* out, int64_t S, int64_t H, int flags, int32_t* scores,
                              void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Multi-GPU on one node (one process per GPU).  The reference runs on one GPU; these serve the N-split form of
 * the linear: every rank holds a block of weight rows (output columns) and the full activation, and each rank's
 * GEMM writes its column block into every rank's copy of the [m, n_total] output over NVLink, so the all-gather
 * happens inside the GEMM.  Buffers that peers write are shared through CUDA IPC handles, exchanged by the caller.
 * ------------------------------------------------------------------------------------------------------- */
#define H3Q_PEER_HANDLE_BYTES 64

/* Allocates `bytes` of device memory on the current device (set-up, not the hot path) and writes its IPC handle
 * (H3Q_PEER_HANDLE_BYTES bytes) to `handle`. */
h3q_status h3q_peer_buffer_alloc(size_t bytes, void** ptr, void* handle);
/* Maps another process's buffer from its handle into this process (a peer pointer this GPU can write). */
h3q_status h3q_peer_buffer_open(const void* handle, void** ptr);
/* Unmaps a buffer mapped by h3q_peer_buffer_open. */
h3q_status h3q_peer_buffer_close(void* ptr);
/* Frees a buffer from h3q_peer_buffer_alloc. */
h3q_status h3q_peer_buffer_free(void* ptr);

/* N-split linear step: quantized activations a [m, k] (scales xs [m]) times this rank's weight rows w_local
 * [n_local, k] (scales ws_local, per row when ws_numel == n_local > 1; bias_local [n_local] or NULL), written as
 * bf16 into columns [n_offset, n_offset + n_local) of every outs[r] ([m, n_total], r < n_ranks <= 8; outs[r] is
 * rank r's buffer, this rank's own included).  Each output tile is computed once and stored to all ranks.  Ranks
 * own disjoint column blocks; a cross-rank barrier after the call (stream-ordered) makes the full output
 * readable.  n_offset and n_total must be multiples of 8; k % 16 == 0. */
h3q_status h3q_gemm_s8_allgather(const int8_t* a, const float* xs, const int8_t* w_local, const float* ws_local,
                                 int64_t ws_numel, const float* bias_local, void* const* outs, int n_ranks, int64_t m,
                                 int64_t n_total, int64_t n_offset, int64_t n_local, int64_t k, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Multi-GPU data plane (no counterpart in the reference, which runs on one device: backend.rs:5-23).  One process
 * per GPU.  Communicators are NCCL's, loaded at run time (a libnccl.so.2 already in the process is preferred);
 * without NCCL these entry points return H3Q_ERR_NCCL.  Collectives are stream-ordered like every other call. */
#define H3Q_COMM_ID_BYTES 128
typedef struct h3q_comm h3q_comm;

/* A new communicator id (H3Q_COMM_ID_BYTES bytes): made by one rank and handed to the others over the caller's
 * own transport. */
h3q_status h3q_comm_unique_id(void* id);
/* Joins rank `rank` of `nranks` on the current device (collective: every rank calls it with the same id).  Also
 * creates the communicator's barrier operand, copy stream and events (set-up, not the hot path). */
h3q_status h3q_comm_init(int nranks, int rank, const void* id, h3q_comm** comm);
h3q_status h3q_comm_destroy(h3q_comm* comm);
int h3q_comm_rank(const h3q_comm* comm);
int h3q_comm_size(const h3q_comm* comm);
/* recv [nranks][bytes_per_rank] = every rank's send buffer, in rank order (ncclAllGather of bytes). */
h3q_status h3q_comm_allgather(h3q_comm* comm, const void* send, void* recv, size_t bytes_per_rank, void* stream);
/* Cross-rank barrier on the stream: completes on every rank only after every rank's earlier work on its stream. */
h3q_status h3q_comm_barrier(h3q_comm* comm, void* stream);

/* Forms of the N-split all-gather (h3q_gemm_s8_nsplit). */
enum {
  H3Q_NSPLIT_FUSED = 0, /* the GEMM's epilogue stores every output box into every rank's buffer (peer memory) */
  H3Q_NSPLIT_PUSH = 1,  /* GEMM in row chunks into this rank's buffer; copy engines push finished chunks to peers */
  H3Q_NSPLIT_NCCL = 2,  /* local GEMM into a packed block, ncclAllGather, relayout kernel into the output */
  H3Q_NSPLIT_PEER = 3   /* GEMM into this rank's buffer, then every SM stores the column block into every peer's */
};

/* Output columns [lo, hi) of rank `rank` in the N split of n columns: whole 256-column GEMM tiles, spread as evenly
 * as the tile count allows (h3q.parallel.nsplit_range). */
void h3q_nsplit_range(int64_t n, int nranks, int rank, int64_t* lo, int64_t* hi);
/* Workspace bytes of h3q_gemm_s8_nsplit (non-zero for H3Q_NSPLIT_NCCL only). */
size_t h3q_gemm_s8_nsplit_workspace_size(int64_t m, int64_t n_total, int nranks, int mode);
/* attn8::gemm_s8's linear (bf16 out) with the weight rows split over the communicator's ranks: quantized
 * activations a [m, k] with row scales xs [m] (the same on every rank), this rank's weight rows w_local
 * [n_local, k] for its columns h3q_nsplit_range(n_total, nranks, rank) (scales ws_local per row when
 * ws_numel == n_local > 1, bias_local [n_local] or NULL).  Every rank receives the whole output [m, n_total] in
 * outs[rank].  FUSED, PUSH and PEER write into peers' buffers: outs[d] is rank d's output mapped into this process
 * (h3q_peer_buffer_open); NCCL reads only outs[rank].  Barriers inside the call order the peers' writes after every
 * rank's earlier use of its output and make the output complete when the call's work on the stream is done.
 * Collective: every rank calls it with the same mode and shape.  n_total % 8 == 0, k % 16 == 0. */
h3q_status h3q_gemm_s8_nsplit(h3q_comm* comm, int mode, const int8_t* a, const float* xs, const int8_t* w_local,
                              const float* ws_local, int64_t ws_numel, const float* bias_local, void* const* outs,
                              int64_t m, int64_t n_total, int64_t k, void* workspace, size_t workspace_bytes,
                              void* stream);

/* h3q_gemm_s8 for callers that cannot allocate device memory (no counterpart in the reference).  Some callers
 * cannot call cudaMalloc: a plugin inside a host that has already reserved the GPU's whole memory for its own
 * pool, or code where cudaMalloc's implicit synchronisation or failure under memory pressure is not acceptable.
 * This entry point takes no workspace: the quantized activations live in a fixed 64 MiB device array inside the
 * library, and the call allocates nothing.  The array is reserved on a device by h3q_init(device) or, without
 * it, by the first h3q_gemm_s8_static call there (the array's module loads lazily), and held until the process
 * exits; call h3q_init first when another pool will take the GPU's memory.  Same arguments and results as
 * h3q_gemm_s8 (bit-identical outputs).  Limits: 256 + roundup(m*k, 256) + 4*m bytes must fit in the 64 MiB
 * (else H3Q_ERR_ARG); the array's address is looked up once per device (by h3q_init or the first call), which
 * should come before any stream capture, and a device reset after it is not supported; all calls on a device
 * share the array, so calls that overlap on the GPU race.  Kernel time-outs are latched in the array's own
 * status word (sticky: no call clears it), read with h3q_gemm_s8_static_status. */
h3q_status h3q_gemm_s8_static(const uint16_t* x, const int8_t* w, const float* ws, int64_t ws_numel,
                              const float* bias, uint16_t* out, int64_t m, int64_t n, int64_t k, int swiglu,
                              int rotate, void* stream);

/* Reads and clears the status word of h3q_gemm_s8_static's scratch array on `device` (no counterpart in the
 * reference).  Synchronises the device first, allocates nothing.  H3Q_ERR_TIMEOUT (with the kernel's code in
 * *code) when a kernel of an h3q_gemm_s8_static call gave up a bounded wait since the last read, else H3Q_OK. */
h3q_status h3q_gemm_s8_static_status(int device, int* code);

#ifdef __cplusplus
}
#endif

#endif /* H3Q_H_ */
