/*
 * h3q_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement, on the CPU, of the arithmetic that apiplant/h3-rs performs on its quantized-linear
 * and int8-attention hot path.  It is the checker for the CUDA library: tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs are the only callers.  Nothing in the product library links
 * it, and the product path never falls back to it.
 *
 * Every function names the reference file:line it restates (paths inside the h3-rs source tree).  Operation
 * order is kept exactly where the reference's result depends on it (the Hadamard butterflies, the scale
 * computation, the epilogue's multiply-add), so integer codes, scales and int32 accumulators match
 * bit for bit.
 *
 * Build with -ffp-contract=off: the explicit fmaf() calls below are the only fused multiply-adds, placed where
 * the reference's NVRTC build (fmad on by default) contracts `a * b + c`.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define H3O_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- number formats (kernels.rs:17-25) */

static inline float bf2f(uint16_t v) {
    uint32_t u = (uint32_t)v << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* round-to-nearest-even f32 -> bf16, NaN -> 0x7fc0 (kernels.rs:18-23, attn8.rs:27-32) */
static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float bf16r(float f) { return bf2f(f2bf(f)); }

static inline float h2f(uint16_t v) {
    _Float16 h;
    memcpy(&h, &v, 2);
    return (float)h;
}

static inline uint16_t f2h(float f) {
    _Float16 h = (_Float16)f; /* IEEE round-to-nearest-even, as cvt.rn.f16.f32 */
    uint16_t v;
    memcpy(&v, &h, 2);
    return v;
}

/* kind: 0 = f32, 1 = f16, 2 = bf16 (kernels.rs:27-38) */
static inline float ldf(const void* p, int kind, size_t i) {
    if (kind == 0) return ((const float*)p)[i];
    if (kind == 1) return h2f(((const uint16_t*)p)[i]);
    return bf2f(((const uint16_t*)p)[i]);
}

static inline void stf(void* p, int kind, size_t i, float v) {
    if (kind == 0) ((float*)p)[i] = v;
    else if (kind == 1) ((uint16_t*)p)[i] = f2h(v);
    else ((uint16_t*)p)[i] = f2bf(v);
}

H3O_API uint16_t h3o_f2bf(float f) { return f2bf(f); }
H3O_API float h3o_bf2f(uint16_t v) { return bf2f(v); }

/* cvt.rni.s32.f32 / __float2int_rn: round half to even, NaN -> 0, saturating */
static inline int f2i_rn(float v) {
    if (isnan(v)) return 0;
    float r = rintf(v);
    if (r >= 2147483648.0f) return 2147483647;
    if (r < -2147483648.0f) return (-2147483647 - 1);
    return (int)r;
}

/* ---------------------------------------------------------------- seeded generator (rng.rs:8-116) */

typedef struct {
    uint32_t state[624];
    int idx;
    int has_cached;
    double cached;
} h3o_gen;

/* TorchGen::new (rng.rs:15-22): torch.manual_seed(seed) */
H3O_API void h3o_gen_init(h3o_gen* g, uint64_t seed) {
    g->state[0] = (uint32_t)(seed & 0xffffffffu);
    for (int i = 1; i < 624; ++i)
        g->state[i] = 1812433253u * (g->state[i - 1] ^ (g->state[i - 1] >> 30)) + (uint32_t)i;
    g->idx = 624;
    g->has_cached = 0;
    g->cached = 0.0;
}

H3O_API size_t h3o_gen_size(void) { return sizeof(h3o_gen); }

/* TorchGen::twist (rng.rs:24-35) */
static void gen_twist(h3o_gen* g) {
    for (int i = 0; i < 624; ++i) {
        uint32_t y = (g->state[i] & 0x80000000u) | (g->state[(i + 1) % 624] & 0x7fffffffu);
        uint32_t v = g->state[(i + 397) % 624] ^ (y >> 1);
        if (y & 1u) v ^= 0x9908b0dfu;
        g->state[i] = v;
    }
    g->idx = 0;
}

/* TorchGen::next_u32 (rng.rs:37-47) */
H3O_API uint32_t h3o_gen_u32(h3o_gen* g) {
    if (g->idx >= 624) gen_twist(g);
    uint32_t y = g->state[g->idx++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    return y ^ (y >> 18);
}

static uint64_t gen_u64(h3o_gen* g) {
    uint64_t hi = h3o_gen_u32(g), lo = h3o_gen_u32(g);
    return (hi << 32) | lo;
}

/* TorchGen::uniform (rng.rs:55-57): 24-bit uniform in [0, 1) */
H3O_API float h3o_gen_uniform(h3o_gen* g) {
    return (float)(h3o_gen_u32(g) & ((1u << 24) - 1)) * (1.0f / (float)(1u << 24));
}

/* TorchGen::normal_scalar (rng.rs:60-77) */
static float gen_normal_scalar(h3o_gen* g) {
    if (g->has_cached) {
        g->has_cached = 0;
        return (float)g->cached;
    }
    double u1 = (double)(gen_u64(g) & ((1ull << 53) - 1)) * (1.0 / (double)(1ull << 53));
    double u2 = (double)(gen_u64(g) & ((1ull << 53) - 1)) * (1.0 / (double)(1ull << 53));
    double r = sqrt(-2.0 * log1p(-u2));
    double th = 2.0 * 3.14159265358979323846 * u1;
    g->cached = r * sin(th);
    g->has_cached = 1;
    return (float)(r * cos(th));
}

/* fill16 (rng.rs:101-110) */
static void fill16(float* d) {
    const float two_pi = 2.0f * 3.14159265358979323846f;
    for (int j = 0; j < 8; ++j) {
        float u1 = 1.0f - d[j];
        float u2 = d[j + 8];
        float r = sqrtf(-2.0f * logf(u1));
        float th = two_pi * u2;
        d[j] = r * cosf(th);
        d[j + 8] = r * sinf(th);
    }
}

/* TorchGen::randn (rng.rs:80-96): torch.randn(n) for float32 */
H3O_API void h3o_gen_randn(h3o_gen* g, float* d, size_t n) {
    if (n < 16) {
        for (size_t i = 0; i < n; ++i) d[i] = gen_normal_scalar(g);
        return;
    }
    for (size_t i = 0; i < n; ++i) d[i] = h3o_gen_uniform(g);
    size_t i = 0;
    for (; i + 16 <= n; i += 16) fill16(d + i);
    if (n % 16 != 0) {
        size_t s = n - 16;
        for (size_t j = s; j < n; ++j) d[j] = h3o_gen_uniform(g);
        fill16(d + s);
    }
}

/*
 * Synthetic W8A8 linear inputs, drawn from one TorchGen stream in this order:
 *   x [M,K] ~ N(0,1); `n_outliers` distinct channels (next_u32 % K, repeats skipped) scaled x20; x -> bf16
 *   w [N,K] int8 uniform over [-127, 127] (next_u32 % 255 - 127)
 *   ws [N] ~ U(1e-3, 1e-2)
 *   bias [N] ~ N(0, 0.02) rounded to bf16, kept as f32 (the reference loads bias as f32, weights.rs:498)
 */
H3O_API void h3o_make_linear_inputs(uint64_t seed, int64_t M, int64_t K, int64_t N, int n_outliers,
                                    uint16_t* x, int8_t* w, float* ws, float* bias) {
    h3o_gen g;
    h3o_gen_init(&g, seed);
    size_t mk = (size_t)M * (size_t)K;
    float* tmp = (float*)malloc(sizeof(float) * (mk > (size_t)N ? mk : (size_t)N) + 64);
    h3o_gen_randn(&g, tmp, mk);
    int64_t outl[64];
    int no = n_outliers < K ? n_outliers : (int)K;
    if (no > 64) no = 64;
    for (int i = 0; i < no;) {
        int64_t c = (int64_t)(h3o_gen_u32(&g) % (uint32_t)K);
        int dup = 0;
        for (int j = 0; j < i; ++j) dup |= (outl[j] == c);
        if (!dup) outl[i++] = c;
    }
    for (int i = 0; i < no; ++i)
        for (int64_t r = 0; r < M; ++r) tmp[(size_t)r * K + outl[i]] *= 20.0f;
    for (size_t i = 0; i < mk; ++i) x[i] = f2bf(tmp[i]);
    size_t nk = (size_t)N * (size_t)K;
    for (size_t i = 0; i < nk; ++i) w[i] = (int8_t)((int)(h3o_gen_u32(&g) % 255u) - 127);
    for (int64_t i = 0; i < N; ++i) ws[i] = 1e-3f + 9e-3f * h3o_gen_uniform(&g);
    h3o_gen_randn(&g, tmp, (size_t)N);
    for (int64_t i = 0; i < N; ++i) bias[i] = bf16r(0.02f * tmp[i]);
    free(tmp);
}

/* ---------------------------------------------------------------- ConvRot Hadamard (weights.rs:441-489) */

/* hadamard(size) (weights.rs:441-465): Kronecker powers of the regular H4, divided by sqrt(size). */
H3O_API int h3o_hadamard(int size, float* h_out) {
    static const float h4[16] = {1, 1, 1, -1, 1, 1, -1, 1, 1, -1, 1, 1, -1, 1, 1, 1};
    int p4 = 4;
    while (p4 < size) p4 *= 4;
    if (size < 4 || p4 != size) return -1; /* "ConvRot group size is not a power of 4" (weights.rs:460-462) */
    int n = 4;
    float* h = (float*)malloc(sizeof(float) * (size_t)size * size);
    float* t = (float*)malloc(sizeof(float) * (size_t)size * size);
    memcpy(h, h4, sizeof(h4));
    while (n < size) {
        for (int i = 0; i < n; ++i)
            for (int j = 0; j < n; ++j)
                for (int a = 0; a < 4; ++a)
                    for (int b = 0; b < 4; ++b)
                        t[(size_t)(i * 4 + a) * (n * 4) + j * 4 + b] = h[(size_t)i * n + j] * h4[a * 4 + b];
        n *= 4;
        float* s = h;
        h = t;
        t = s;
    }
    int ok = (n == size);
    if (ok) {
        float norm = sqrtf((float)size);
        for (size_t i = 0; i < (size_t)size * size; ++i) h_out[i] = h[i] / norm;
    }
    free(h);
    free(t);
    return ok ? 0 : -1;
}

/* rotate_activation(x, 256) in f64 (weights.rs:482-489): exact-arithmetic reference for property tests */
H3O_API void h3o_rotate_f64(const float* x, double* out, int64_t rows, int64_t K) {
    float H[256 * 256];
    h3o_hadamard(256, H);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t g = 0; g < K / 256; ++g) {
            const float* xr = x + r * K + g * 256;
            for (int j = 0; j < 256; ++j) {
                double s = 0.0;
                for (int i = 0; i < 256; ++i) s += (double)xr[i] * (double)H[i * 256 + j];
                out[r * K + g * 256 + j] = s;
            }
        }
}

/* ---------------------------------------------------------------- per-row int8 quantizers */

/*
 * One 256-group through quant_rows_i8_rot2's warp butterfly (kernels.rs:220-270).  Element i of the group
 * is held by lane i/8 as a[i%8].  Digits of i in base 4 are transformed in the order 0, 1, 2, 3 with the
 * regular H4 (out_p = sum - 2*a_{3-p}, kernels.rs:218).  Digit 0 sums in-thread as ((a0+a1)+a2)+a3
 * (kernels.rs:237-241); digits 1..3 sum pairwise as (a_p + a_{p^1}) + (a_{p^2} + a_{p^3}) through shuffles
 * (kernels.rs:244-265).  The output is multiplied by 1/16 (kernels.rs:268).
 */
static void rot2_group(float v[256]) {
    float a[32][8], b[32][8];
    for (int l = 0; l < 32; ++l)
        for (int e = 0; e < 8; ++e) a[l][e] = v[l * 8 + e];
    /* digit 0 (e & 3): in-thread */
    for (int l = 0; l < 32; ++l)
        for (int hb = 0; hb < 8; hb += 4) {
            float s = ((a[l][hb] + a[l][hb + 1]) + a[l][hb + 2]) + a[l][hb + 3];
            float b0 = s - 2.f * a[l][hb + 3], b1 = s - 2.f * a[l][hb + 2];
            float b2 = s - 2.f * a[l][hb + 1], b3 = s - 2.f * a[l][hb];
            a[l][hb] = b0; a[l][hb + 1] = b1; a[l][hb + 2] = b2; a[l][hb + 3] = b3;
        }
    /* digit 1 = (e >> 2) + 2 * (lane & 1) */
    for (int l = 0; l < 32; ++l)
        for (int e = 0; e < 4; ++e) {
            int p = l ^ 1;
            float s = (a[l][e] + a[l][e + 4]) + (a[p][e] + a[p][e + 4]);
            b[l][e] = s - 2.f * a[p][e + 4];
            b[l][e + 4] = s - 2.f * a[p][e];
        }
    memcpy(a, b, sizeof(a));
    /* digits 2 and 3 = (lane >> 1) & 3, (lane >> 3) & 3 */
    for (int d = 0; d < 2; ++d) {
        int sh = d == 0 ? 1 : 3;
        for (int l = 0; l < 32; ++l)
            for (int e = 0; e < 8; ++e) {
                int l1 = l ^ (1 << sh), l2 = l ^ (2 << sh), l3 = l ^ (3 << sh);
                float s1 = a[l][e] + a[l1][e];
                float s2 = a[l2][e] + a[l2 ^ (1 << sh)][e];
                b[l][e] = (s1 + s2) - 2.f * a[l3][e];
            }
        memcpy(a, b, sizeof(a));
    }
    for (int l = 0; l < 32; ++l)
        for (int e = 0; e < 8; ++e) v[l * 8 + e] = a[l][e] * (1.f / 16.f);
}

/*
 * One 256-group through quant_rows_i8_rot's shared-memory butterfly (kernels.rs:166-197): strides 1, 4, 16,
 * 64, each output from the four inputs a0..a3 of its digit with left-to-right sums
 * p=0: a0+a1+a2-a3, p=1: a0+a1-a2+a3, p=2: a0-a1+a2+a3, p=3: -a0+a1+a2+a3 (kernels.rs:183-187), then * 1/16.
 */
static void rot1_group(float v[256]) {
    float sm[256], o[256];
    memcpy(sm, v, sizeof(sm));
    for (int st = 0, stride = 1; st < 4; ++st, stride *= 4) {
        for (int i = 0; i < 256; ++i) {
            int p = (i / stride) & 3, i0 = i - p * stride;
            float a0 = sm[i0], a1 = sm[i0 + stride], a2 = sm[i0 + 2 * stride], a3 = sm[i0 + 3 * stride];
            float r;
            if (p == 0) r = ((a0 + a1) + a2) - a3;
            else if (p == 1) r = ((a0 + a1) - a2) + a3;
            else if (p == 2) r = ((a0 - a1) + a2) + a3;
            else r = ((-a0 + a1) + a2) + a3;
            o[i] = r;
        }
        memcpy(sm, o, sizeof(sm));
    }
    for (int i = 0; i < 256; ++i) v[i] = sm[i] * (1.f / 16.f);
}

/*
 * Per-row int8 quantization of x [M,K] (kind 0/1/2), optionally ConvRot-rotated.
 *   mode 0: quant_rows_i8 (kernels.rs:296-318): no rotation; q = (s8)min(max(rintf(v*inv), -128), 127)
 *   mode 1: quant_rows_i8_rot (kernels.rs:166-213): smem butterfly; same clamp form as mode 0
 *   mode 2: quant_rows_i8_rot2 (kernels.rs:220-293): warp butterfly, bf16 only; q = clamp(__float2int_rn)
 * Scale s = fmaxf(max|v| / 127, 1e-30), inv = 1/s (IEEE divisions; kernels.rs:206, :278, :313).
 */
H3O_API int h3o_quant_rows(const void* x, int kind, int8_t* q, float* scale, int64_t M, int64_t K, int mode) {
    if (mode != 0 && K % 256 != 0) return -1;
    if (mode == 2 && kind != 2) return -1;
    float* v = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t r = 0; r < M; ++r) {
        size_t base = (size_t)r * K;
        for (int64_t i = 0; i < K; ++i) v[i] = ldf(x, kind, base + i);
        if (mode == 1)
            for (int64_t g = 0; g < K / 256; ++g) rot1_group(v + g * 256);
        if (mode == 2)
            for (int64_t g = 0; g < K / 256; ++g) rot2_group(v + g * 256);
        float m = 0.f;
        for (int64_t i = 0; i < K; ++i) m = fmaxf(m, fabsf(v[i]));
        float s = fmaxf(m / 127.f, 1e-30f), inv = 1.f / s;
        scale[r] = s;
        for (int64_t i = 0; i < K; ++i) {
            float t = v[i] * inv;
            int qi;
            if (mode == 2) {
                qi = f2i_rn(t);
                qi = qi < -128 ? -128 : (qi > 127 ? 127 : qi);
            } else {
                float rr = fminf(fmaxf(rintf(t), -128.f), 127.f); /* NaN -> -128 through fmaxf */
                qi = (int)rr;
            }
            q[base + i] = (int8_t)qi;
        }
    }
    free(v);
    return 0;
}

/* rotate_activation(x, 256) on bf16 rows, computed in the quant_rows_i8_rot2 butterfly order and rounded to
 * bf16 (weights.rs:482-489; the reference runs it as a bf16 matmul, whose accumulation order is unpinned) */
H3O_API int h3o_rotate_bf16(const uint16_t* x, uint16_t* out, int64_t M, int64_t K) {
    if (K % 256 != 0) return -1;
    float v[256];
    for (int64_t r = 0; r < M; ++r)
        for (int64_t g = 0; g < K / 256; ++g) {
            for (int i = 0; i < 256; ++i) v[i] = bf2f(x[r * K + g * 256 + i]);
            rot2_group(v);
            for (int i = 0; i < 256; ++i) out[r * K + g * 256 + i] = f2bf(v[i]);
        }
    return 0;
}

/* swiglu_interleaved (weights.rs:806-816) / ops::swiglu (ops.rs:39-44) on bf16: silu(g) rounded, times u */
H3O_API void h3o_swiglu_bf16(const uint16_t* y, uint16_t* out, int64_t rows, int64_t F, int interleaved) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < F; ++j) {
            int64_t gi = interleaved ? r * 2 * F + 2 * j : r * 2 * F + j;
            int64_t ui = interleaved ? gi + 1 : gi + F;
            float g = bf2f(y[gi]), u = bf2f(y[ui]);
            float s = bf16r(g / (1.f + expf(-g)));
            out[r * F + j] = f2bf(s * u);
        }
}

/* ---------------------------------------------------------------- int8 GEMM core and epilogues */

/* acc[m,n] = sum_k A[m,k] * B[n,k] (int32; attn8.rs:258-318 main loop, kernels.rs:1026-1044 cuBLASLt IMMA) */
H3O_API void h3o_gemm_s8_acc(const int8_t* A, const int8_t* B, int32_t* acc, int64_t M, int64_t N, int64_t K) {
    for (int64_t m = 0; m < M; ++m) {
        const int8_t* a = A + m * K;
        for (int64_t n = 0; n < N; ++n) {
            const int8_t* b = B + n * K;
            int32_t s = 0;
            for (int64_t k = 0; k < K; ++k) s += (int32_t)a[k] * (int32_t)b[k];
            acc[m * N + n] = s;
        }
    }
}

/* bf16(gelu_tanh(bf16 y)), candle's `gelu` (ops.rs:46-48): 0.5 y (1 + tanh(sqrt(2/pi) (y + 0.044715 y^3))) */
static float gelu_tanh_f(float y) {
    const float c = 0.7978845608028654f;
    return 0.5f * y * (1.f + tanhf(c * (y + 0.044715f * y * y * y)));
}

/*
 * Fused-epilogue GEMM output from int32 accumulators, as gemm_s8 computes it (attn8.rs:320-343):
 *   v = fmaf((float)acc * xs[m], ws[n], bias[n])        (NVRTC contracts `acc * x * w + b`)
 * epi 0: out[m,n] = bf16(v)
 * epi 1: SwiGLU over interleaved (gate, up) column pairs (attn8.rs:334-337):
 *        gt = bf16r(v0), up = bf16r(v1), sg = bf16r(gt / (1 + exp(-gt))), out[m,n/2] = bf16(sg * up)
 * epi 3: out = bf16(gelu_tanh(bf16r(v)))  (candle gelu applied to the bf16 linear output, ops.rs:46-48)
 * epi 4: out = bf16(fmaf(bf16r(v), bf16r(gate[idx[m], n]), resid[m,n]))  (gate_add on the bf16 output,
 *        kernels.rs:418-428; `x + y * g` contracted)
 * ws_per_row: ws has N entries, else ws[0] for every column (attn8.rs:553).  bias may be NULL.
 * The epi numbers are the H3Q_EPI_* values of include/h3q.h.
 */
H3O_API void h3o_gemm_s8_epilogue(const int32_t* acc, const float* xs, const float* ws, int ws_per_row,
                                  const float* bias, uint16_t* out, int64_t M, int64_t N, int epi,
                                  const float* gate, const uint32_t* gate_idx, const uint16_t* resid) {
    for (int64_t m = 0; m < M; ++m) {
        float x = xs[m];
        if (epi == 1) {
            for (int64_t n = 0; n + 1 < N; n += 2) {
                float w0 = ws_per_row ? ws[n] : ws[0], w1 = ws_per_row ? ws[n + 1] : ws[0];
                float v0 = fmaf((float)acc[m * N + n] * x, w0, bias ? bias[n] : 0.f);
                float v1 = fmaf((float)acc[m * N + n + 1] * x, w1, bias ? bias[n + 1] : 0.f);
                float gt = bf16r(v0), up = bf16r(v1);
                float sg = bf16r(gt / (1.f + expf(-gt)));
                out[m * (N / 2) + n / 2] = f2bf(sg * up);
            }
            continue;
        }
        for (int64_t n = 0; n < N; ++n) {
            float w = ws_per_row ? ws[n] : ws[0];
            float v = fmaf((float)acc[m * N + n] * x, w, bias ? bias[n] : 0.f);
            float o;
            if (epi == 3) {
                o = gelu_tanh_f(bf16r(v));
            } else if (epi == 4) {
                uint32_t gi = gate_idx ? gate_idx[m] : 0u;
                float g = bf16r(gate[(size_t)gi * N + n]);
                o = fmaf(bf16r(v), g, bf2f(resid[m * N + n]));
            } else {
                o = v;
            }
            out[m * N + n] = f2bf(o);
        }
    }
}

/*
 * cuBLASLt-path epilogues (kernels.rs:333-373): out dtype okind (0 f32, 1 f16, 2 bf16).
 *   swiglu = 0: out[m,n] = fmaf(acc * xs[m], ws[n], bias[n])                       (int8_epilogue)
 *   swiglu = 1: split halves, gate = col j, up = col F+j of acc [M, 2F] (int8_epilogue_swiglu):
 *               out[m,j] = silu_r(gate) * up_r(up), bf16 re-rounding of the operands when okind is bf16
 * N is the output width (F when swiglu).
 */
H3O_API void h3o_int8_epilogue(const int32_t* acc, const float* xs, const float* ws, int ws_per_row,
                               const float* bias, void* out, int okind, int64_t M, int64_t N, int swiglu) {
    for (int64_t m = 0; m < M; ++m) {
        float x = xs[m];
        if (!swiglu) {
            for (int64_t n = 0; n < N; ++n) {
                float w = ws_per_row ? ws[n] : ws[0];
                stf(out, okind, (size_t)(m * N + n), fmaf((float)acc[m * N + n] * x, w, bias ? bias[n] : 0.f));
            }
            continue;
        }
        const int32_t* row = acc + m * 2 * N;
        for (int64_t j = 0; j < N; ++j) {
            float wg = ws_per_row ? ws[j] : ws[0];
            float wu = ws_per_row ? ws[N + j] : wg;
            float g = fmaf((float)row[j] * x, wg, bias ? bias[j] : 0.f);
            float u = fmaf((float)row[N + j] * x, wu, bias ? bias[N + j] : 0.f);
            if (okind == 2) g = bf16r(g);
            float s = g / (1.f + expf(-g));
            if (okind == 2) { s = bf16r(s); u = bf16r(u); }
            stf(out, okind, (size_t)(m * N + j), s * u);
        }
    }
}

/* gate_add (kernels.rs:418-428): out = x + y * round_to_kind(gate[idx[s], c]), contracted to one fma */
H3O_API void h3o_gate_add(const void* x, const void* y, int kind, const float* gate, const uint32_t* idx,
                          void* out, int64_t S, int64_t C) {
    for (int64_t s = 0; s < S; ++s)
        for (int64_t c = 0; c < C; ++c) {
            size_t i = (size_t)(s * C + c);
            float g = gate[(size_t)idx[s] * C + c];
            g = (kind == 1) ? h2f(f2h(g)) : bf16r(g);
            stf(out, kind, i, fmaf(ldf(y, kind, i), g, ldf(x, kind, i)));
        }
}

/* ---------------------------------------------------------------- weight decode */

/* dequant_i8 (kernels.rs:40-49, portable/kernels.rs:14-27): out = (float)q * scale[row or 0] */
H3O_API void h3o_dequant_i8(const int8_t* q, const float* scale, int per_row, void* out, int okind,
                            int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c)
            stf(out, okind, (size_t)(r * cols + c), (float)q[r * cols + c] * (per_row ? scale[r] : scale[0]));
}

/* fp8 e4m3 decode (kernels.rs:51-58, portable/kernels.rs:29-44) */
H3O_API float h3o_fp8e4m3(uint8_t v) {
    int sgn = v >> 7, e = (v >> 3) & 15, m = v & 7;
    float r;
    if (e == 0) r = ldexpf((float)m / 8.0f, -6);
    else if (e == 15 && m == 7) r = NAN;
    else r = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return sgn ? -r : r;
}

static const float E2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                               -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

/* byte offset of block scale (row r, 16-wide block b) in the 128x4 swizzled table (kernels.rs:76-78) */
H3O_API int64_t h3o_nvfp4_scale_offset(int64_t r, int64_t b, int64_t k) {
    int64_t nb = k / 16, ncb = (nb + 3) / 4;
    int64_t rb = r / 128, rin = r % 128, cb = b / 4, cin = b % 4;
    return (rb * ncb + cb) * 512 + (rin % 32) * 16 + (rin / 32) * 4 + cin;
}

/*
 * dequant_nvfp4 (kernels.rs:65-81, portable/kernels.rs:46-70): q [N, K/2] two e2m1 codes per byte, even
 * column in the HIGH nibble; W[r,c] = E2M1[nib] * e4m3(bs[swz(r, c/16)]) * g.
 */
H3O_API void h3o_dequant_nvfp4(const uint8_t* q, const uint8_t* bs, float g, void* out, int okind,
                               int64_t nrows, int64_t k) {
    for (int64_t r = 0; r < nrows; ++r)
        for (int64_t c = 0; c < k; ++c) {
            uint8_t byte = q[r * (k / 2) + c / 2];
            int nib = (c & 1) ? (byte & 15) : (byte >> 4);
            float s = h3o_fp8e4m3(bs[h3o_nvfp4_scale_offset(r, c / 16, k)]);
            stf(out, okind, (size_t)(r * k + c), E2M1[nib] * s * g);
        }
}

/* ---------------------------------------------------------------- int8 attention (attn8.rs) */

/*
 * ColMean + `/ S` (attn8.rs:45-52 col_sum, launch :440-453, mean :622): column sums of k [S, C] (bf16, C = H*128)
 * over row chunks of rows_per = ceil(S / min(128, S)) rows, each chunk summed in row order from 0.f, the chunk
 * sums added in chunk order from 0.f (the reference adds them with atomicAdd in completion order), then
 * multiplied by (float)(1 / S) (candle's affine with mul = 1/S).
 */
H3O_API void h3o_attn_kmean(const uint16_t* k, int64_t S, int64_t H, float* mean) {
    const int64_t C = H * 128;
    const int64_t parts = S < 128 ? S : 128;
    const int64_t rows_per = (S + parts - 1) / parts;
    const float inv_s = (float)(1.0 / (double)S);
    for (int64_t c = 0; c < C; ++c) {
        float a = 0.f;
        for (int64_t r0 = 0; r0 < S; r0 += rows_per) {
            float s = 0.f;
            const int64_t r1 = r0 + rows_per < S ? r0 + rows_per : S;
            for (int64_t r = r0; r < r1; ++r) s += bf2f(k[r * C + c]);
            a += s;
        }
        mean[c] = a * inv_s;
    }
}

/* quant_heads' per-element code (attn8.rs:85-90): clamp(__float2int_rn(v * inv), -127, 127) */
static inline int8_t q127(float v, float inv) {
    int q = f2i_rn(v * inv);
    return (int8_t)(q < -127 ? -127 : (q > 127 ? 127 : q));
}

/*
 * QuantHeads (attn8.rs:69-93): x bf16 [S, H, 128], v = x - mean[h, d] (or - 0), sc = fmaxf(max|v| / 127, 1e-20),
 * inv = 1 / sc, codes [H, S, 128], scales [H, Sp] with Sp = roundup(S, 128), pads zero.
 * block128: one scale per 128-token block of a head (the maximum over the block's valid tokens), stored at
 * every token of the block.
 */
H3O_API void h3o_attn_quant_heads(const uint16_t* x, const float* mean, int8_t* codes, float* scales, int64_t S,
                                  int64_t H, int block128) {
    const int64_t Sp = (S + 127) / 128 * 128;
    memset(scales, 0, (size_t)(H * Sp) * sizeof(float));
    float v[128];
    for (int64_t h = 0; h < H; ++h) {
        if (!block128) {
            for (int64_t s = 0; s < S; ++s) {
                const uint16_t* xr = x + (s * H + h) * 128;
                float m = 0.f;
                for (int d = 0; d < 128; ++d) {
                    v[d] = bf2f(xr[d]) - (mean ? mean[h * 128 + d] : 0.f);
                    m = fmaxf(m, fabsf(v[d]));
                }
                const float sc = fmaxf(m / 127.f, 1e-20f);
                const float inv = 1.f / sc;
                for (int d = 0; d < 128; ++d) codes[(h * S + s) * 128 + d] = q127(v[d], inv);
                scales[h * Sp + s] = sc;
            }
        } else {
            for (int64_t b0 = 0; b0 < S; b0 += 128) {
                const int64_t b1 = b0 + 128 < S ? b0 + 128 : S;
                float m = 0.f;
                for (int64_t s = b0; s < b1; ++s)
                    for (int d = 0; d < 128; ++d)
                        m = fmaxf(m, fabsf(bf2f(x[(s * H + h) * 128 + d]) - (mean ? mean[h * 128 + d] : 0.f)));
                const float sc = fmaxf(m / 127.f, 1e-20f);
                const float inv = 1.f / sc;
                for (int64_t s = b0; s < b1; ++s) {
                    for (int d = 0; d < 128; ++d) {
                        const float vv = bf2f(x[(s * H + h) * 128 + d]) - (mean ? mean[h * 128 + d] : 0.f);
                        codes[(h * S + s) * 128 + d] = q127(vv, inv);
                    }
                    scales[h * Sp + s] = sc;
                }
            }
        }
    }
}

/* int32 Q.K^T accumulators [H, S, S] of codes [H, S, 128] (attn8.rs:177-184 mma_s8 loop) */
H3O_API void h3o_attn_scores(const int8_t* q8, const int8_t* k8, int64_t S, int64_t H, int32_t* out) {
    for (int64_t h = 0; h < H; ++h)
        for (int64_t i = 0; i < S; ++i) {
            const int8_t* a = q8 + (h * S + i) * 128;
            for (int64_t j = 0; j < S; ++j) {
                const int8_t* b = k8 + (h * S + j) * 128;
                int32_t s = 0;
                for (int d = 0; d < 128; ++d) s += (int32_t)a[d] * (int32_t)b[d];
                out[(h * S + i) * S + j] = s;
            }
        }
}

/* scale_log2 = (1 / sqrt(128)) * LOG2_E in f32 (attn8.rs:625) */
H3O_API float h3o_attn_scale_log2(void) {
    volatile float d = 128.0f;
    const float r = 1.0f / sqrtf(d);
    return r * 1.44269504088896340736f;
}

/*
 * attn_qk8 (attn8.rs:107-246) for one head at a time, in its 64-key tiles:
 *   p = (float)acc * (qs * scale_log2) * ks      (keys >= S excluded)
 *   per tile: mn = max(m, tile max); a = 2^(m - mn); p = 2^(p - mn); l = l * a + sum p; o = o * a + sum f16(p) v
 *   out = bf16(o * (1 / l))
 * V is taken from rows of src (bf16, row stride v_rs elements, head h at column v_col + 128 h) and rounded to f16
 * as v_to_f16 does (attn8.rs:55-65), or kept in bf16 with P rounded to bf16 (pv_bf16).  exp2f stands in for
 * ex2.approx; sums run in a fixed order.  Queries: Sq rows (codes [H, Sq, 128], scales [H, roundup(Sq, 128)]);
 * keys and values: S rows.  Output bf16 [Sq, H, 128].
 */
H3O_API void h3o_attn_forward_rows(const int8_t* q8, const float* qs, int64_t Sq, const int8_t* k8, const float* ks,
                                   const uint16_t* vsrc, int64_t v_rs, int64_t v_col, uint16_t* out, int64_t S,
                                   int64_t H, int pv_bf16) {
    const int64_t Sp = (S + 127) / 128 * 128, Sqp = (Sq + 127) / 128 * 128;
    const float sl2 = h3o_attn_scale_log2();
    float* vv = (float*)malloc((size_t)S * 128 * sizeof(float));
    float p[64], o[128];
    for (int64_t h = 0; h < H; ++h) {
        for (int64_t s = 0; s < S; ++s)
            for (int d = 0; d < 128; ++d) {
                const uint16_t b = vsrc[s * v_rs + v_col + h * 128 + d];
                vv[s * 128 + d] = pv_bf16 ? bf2f(b) : h2f(f2h(bf2f(b)));
            }
        for (int64_t i = 0; i < Sq; ++i) {
            const int8_t* a = q8 + (h * Sq + i) * 128;
            const float qs0 = qs[h * Sqp + i] * sl2;
            float m = -INFINITY, l = 0.f;
            for (int d = 0; d < 128; ++d) o[d] = 0.f;
            for (int64_t j0 = 0; j0 < S; j0 += 64) {
                const int64_t nj = S - j0 < 64 ? S - j0 : 64;
                float mx = -INFINITY;
                for (int64_t j = 0; j < nj; ++j) {
                    const int8_t* b = k8 + (h * S + j0 + j) * 128;
                    int32_t acc = 0;
                    for (int d = 0; d < 128; ++d) acc += (int32_t)a[d] * (int32_t)b[d];
                    p[j] = (float)acc * qs0 * ks[h * Sp + j0 + j];
                    mx = fmaxf(mx, p[j]);
                }
                const float mn = fmaxf(m, mx);
                const float al = mn == -INFINITY ? 1.f : exp2f(m - mn);
                const float bb = mn == -INFINITY ? 0.f : mn;
                float sum = 0.f;
                for (int d = 0; d < 128; ++d) o[d] *= al;
                for (int64_t j = 0; j < nj; ++j) {
                    p[j] = exp2f(p[j] - bb);
                    sum += p[j];
                    const float pr = pv_bf16 ? bf16r(p[j]) : h2f(f2h(p[j]));
                    const float* vr = vv + (j0 + j) * 128;
                    for (int d = 0; d < 128; ++d) o[d] += pr * vr[d];
                }
                l = l * al + sum;
                m = mn;
            }
            const float inv = l > 0.f ? 1.f / l : 0.f;
            for (int d = 0; d < 128; ++d) out[(i * H + h) * 128 + d] = f2bf(o[d] * inv);
        }
    }
    free(vv);
}

/* the whole sequence: Sq == S */
H3O_API void h3o_attn_forward(const int8_t* q8, const float* qs, const int8_t* k8, const float* ks,
                              const uint16_t* vsrc, int64_t v_rs, int64_t v_col, uint16_t* out, int64_t S, int64_t H,
                              int pv_bf16) {
    h3o_attn_forward_rows(q8, qs, S, k8, ks, vsrc, v_rs, v_col, out, S, H, pv_bf16);
}

/* ---------------------------------------------------------------- RMSNorm + adaLN modulate (kernels.rs:376-401) */

/*
 * rms_modulate for bf16 rows x [S, C], weight w (bf16 [C]), f32 tables scale / shift [R, C] selected per row by
 * idx: the sum of squares in the reference kernel's order (512 thread partials, thread t summing elements
 * t, t+512, ... with a fused multiply-add; each 32-thread group then reduced by xor shuffles 16, 8, 4, 2, 1; the
 * 16 group sums reduced the same way), inv = 1 / sqrt(sum / C + eps) (the reference calls rsqrtf, an approximate
 * instruction; 1/sqrtf here can differ from it in the last bit), n = bf16((x * inv) * w), out =
 * bf16(fma(n, 1 + bf16(scale), bf16(shift))).  Output bf16 bits [S, C].
 */
static float xor_tree32(const float* v) {
    float a[32];
    for (int i = 0; i < 32; ++i) a[i] = v[i];
    for (int o = 16; o > 0; o >>= 1) {
        float b[32];
        for (int i = 0; i < 32; ++i) b[i] = a[i] + a[i ^ o];
        for (int i = 0; i < 32; ++i) a[i] = b[i];
    }
    return a[0];
}

H3O_API void h3o_rms_modulate(const uint16_t* x, const uint16_t* w, float eps, const float* scale, const float* shift,
                              const uint32_t* idx, uint16_t* out, int64_t S, int64_t C) {
    for (int64_t r = 0; r < S; ++r) {
        const uint16_t* xr = x + r * C;
        float part[512], red[32];
        for (int t = 0; t < 512; ++t) {
            float sq = 0.f;
            for (int64_t c = t; c < C; c += 512) {
                const float v = bf2f(xr[c]);
                sq = fmaf(v, v, sq);
            }
            part[t] = sq;
        }
        for (int wp = 0; wp < 16; ++wp) red[wp] = xor_tree32(part + 32 * wp);
        for (int wp = 16; wp < 32; ++wp) red[wp] = 0.f;
        const float total = xor_tree32(red);
        const float inv = 1.0f / sqrtf(total / (float)C + eps);
        const int64_t row = (int64_t)idx[r] * C;
        for (int64_t c = 0; c < C; ++c) {
            const float n = bf16r((bf2f(xr[c]) * inv) * bf2f(w[c]));
            const float sc = bf16r(scale[row + c]), sh = bf16r(shift[row + c]);
            out[r * C + c] = f2bf(fmaf(n, 1.f + sc, sh));
        }
    }
}

/* qk_norm_rope (kernels.rs:86-126) for bf16 x: per (token s, head h) row of D <= 256 values at
 * x[s * rs + col + h * hs + d] -> out bf16 [S, H, D].  The sum of squares follows the kernel's reduction: a 32-lane
 * xor tree over each 32-dim slice (thread d sits at lane d % 32 of warp d / 32), then an xor tree over the slice
 * sums (absent slices zero).  inv = 1 / sqrtf(ss / D + eps) stands for the device's rsqrtf (an approximate
 * instruction: the two can differ in the last bit).  v = (v * inv) * w[d] (w NULL: 1).  With rot > 0 the first rot
 * dims rotate in halves with cos / sin = cs[0 or 1][s][d mod half]: fma(v, cos, -(partner * sin)) below half,
 * fma(v, cos, partner * sin) above -- the association the reference's compiled kernel uses (one rounded product,
 * one fused).  out = f2bf. */
H3O_API void h3o_qk_norm_rope(const uint16_t* x, int64_t rs, int64_t col, int64_t hs, const uint16_t* w, int do_norm,
                              float eps, const float* cs, int rot, uint16_t* out, int64_t S, int64_t H, int64_t D) {
    const int NS = (int)((D + 31) / 32), half = rot / 2;
    for (int64_t s = 0; s < S; ++s) {
        for (int64_t h = 0; h < H; ++h) {
            const uint16_t* xr = x + s * rs + col + h * hs;
            float v[256], red[32];
            for (int d = 0; d < 32 * NS; ++d) v[d] = d < D ? bf2f(xr[d]) : 0.f;
            if (do_norm) {
                for (int i = 0; i < 32; ++i) {
                    float sq[32];
                    for (int l = 0; l < 32; ++l) sq[l] = i < NS ? v[32 * i + l] * v[32 * i + l] : 0.f;
                    red[i] = i < NS ? xor_tree32(sq) : 0.f;
                }
                const float ss = xor_tree32(red);
                const float inv = 1.0f / sqrtf(ss / (float)D + eps);
                for (int d = 0; d < D; ++d) v[d] = (v[d] * inv) * (w ? bf2f(w[d]) : 1.f);
            }
            uint16_t* o = out + (s * H + h) * D;
            for (int d = 0; d < D; ++d) {
                float r = v[d];
                if (d < rot) {
                    const int j = d < half ? d : d - half;
                    const float c = cs[s * half + j], sn = cs[(S + s) * half + j];
                    r = d < half ? fmaf(v[d], c, -(v[d + half] * sn)) : fmaf(v[d], c, v[d - half] * sn);
                }
                o[d] = f2bf(r);
            }
        }
    }
}

/* ---------------------------------------------------------------- LoRA merge (load time) */

/* The summed deltas of row i: tot[c] = sum over LoRAs l, in order, of f32(scale_l) * (b_l[i, :] . a_l[:, c]),
 * each dot product the j-ordered chain fmaf(b[i, j], a[j, c], acc) from 0 (weights.rs:696-707 forms b @ a as an
 * f32 matmul whose order the BLAS picks; this is the order the CUDA library fixes).  acc is scratch [k]. */
static void lora_row_delta(int n_loras, const float* const* a, const float* const* b, const int64_t* ranks,
                           const double* scales, int64_t i, int64_t k, float* tot, float* acc) {
    for (int l = 0; l < n_loras; ++l) {
        for (int64_t c = 0; c < k; ++c) acc[c] = 0.f;
        for (int64_t j = 0; j < ranks[l]; ++j) {
            const float bv = b[l][i * ranks[l] + j];
            const float* ar = a[l] + j * k;
            for (int64_t c = 0; c < k; ++c) acc[c] = fmaf(bv, ar[c], acc[c]);
        }
        const float sc = (float)scales[l];
        for (int64_t c = 0; c < k; ++c) {
            const float d = acc[c] * sc;
            tot[c] = l == 0 ? d : tot[c] + d;
        }
    }
}

/*
 * QLinear::merge_loras for an int8 layer (weights.rs:716-757), row by row: w = (float)q * s (dequant_i8,
 * kernels.rs:40-48); with ConvRot w = rotate_activation(w) (back to the plain basis, weights.rs:727-730, here the
 * quantizer's butterfly rot2_group); w = w + deltas; rotate again; s' = max(max|w| * f32(1/127), 1e-30) (candle's
 * `/ 127.0` is an affine multiply by f32(1/127), then clamp(1e-30, MAX)); q' = clamp(round(w / s'), -128, 127)
 * (IEEE division, round half away from zero, weights.rs:735-738).  LoRA factors arrive as f32 (bf16 widened).
 * n_loras == 0 writes nothing (weights.rs:693-695).
 */
H3O_API int h3o_lora_merge_i8(const int8_t* q, const float* scale, int per_row, int convrot, int n_loras,
                              const float* const* a, const float* const* b, const int64_t* ranks,
                              const double* scales, int8_t* q_out, float* scale_out, int64_t n, int64_t k) {
    if (convrot != 0 && (convrot != 256 || k % 256 != 0)) return 1;
    if (n_loras == 0) return 0;
    float* w = (float*)malloc((size_t)k * sizeof(float));
    float* tot = (float*)malloc((size_t)k * sizeof(float));
    float* acc = (float*)malloc((size_t)k * sizeof(float));
    if (!w || !tot || !acc) {
        free(w); free(tot); free(acc);
        return 2;
    }
    for (int64_t i = 0; i < n; ++i) {
        const float s = per_row ? scale[i] : scale[0];
        for (int64_t c = 0; c < k; ++c) w[c] = (float)q[i * k + c] * s;
        if (convrot)
            for (int64_t g = 0; g < k; g += 256) rot2_group(w + g);
        lora_row_delta(n_loras, a, b, ranks, scales, i, k, tot, acc);
        for (int64_t c = 0; c < k; ++c) w[c] = w[c] + tot[c];
        if (convrot)
            for (int64_t g = 0; g < k; g += 256) rot2_group(w + g);
        float m = 0.f;
        for (int64_t c = 0; c < k; ++c) m = fmaxf(m, fabsf(w[c]));
        const float sc = fmaxf(m * (float)(1.0 / 127.0), 1e-30f);
        scale_out[i] = sc;
        for (int64_t c = 0; c < k; ++c) {
            const float r = roundf(w[c] / sc);
            q_out[i * k + c] = (int8_t)(int)fminf(fmaxf(r, -128.f), 127.f);
        }
    }
    free(w); free(tot); free(acc);
    return 0;
}

/* QLinear::merge_loras for a dense layer (weights.rs:710-715) before the cast back: out = f32(w) + deltas (f32;
 * the caller rounds to the weight's dtype). */
H3O_API void h3o_lora_merge_dense(const float* w, int n_loras, const float* const* a, const float* const* b,
                                  const int64_t* ranks, const double* scales, float* out, int64_t n, int64_t k) {
    float* tot = (float*)malloc((size_t)k * sizeof(float));
    float* acc = (float*)malloc((size_t)k * sizeof(float));
    if (!tot || !acc) {
        free(tot); free(acc);
        return;
    }
    for (int64_t i = 0; i < n; ++i) {
        lora_row_delta(n_loras, a, b, ranks, scales, i, k, tot, acc);
        for (int64_t c = 0; c < k; ++c) out[i * k + c] = n_loras ? w[i * k + c] + tot[c] : w[i * k + c];
    }
    free(tot); free(acc);
}
