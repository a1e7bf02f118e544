"""TEST INFRASTRUCTURE ONLY -- Python face of the CPU oracle (liboracle.so, h3q_oracle.c) and of the
reference's dequantise-then-matmul CPU path.

Callers: tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs, as the
checker or the timed CPU baseline.  The product library never imports this module.

Every function names the h3-rs file:line it restates (paths inside the h3-rs source tree).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

c_i64, c_int, c_f32, c_u64, c_vp = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_uint64, ctypes.c_void_p


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle not built: {path} (run `make -C oracle`)")
        L = ctypes.CDLL(path)
        L.h3o_gen_size.restype = ctypes.c_size_t
        L.h3o_gen_u32.restype = ctypes.c_uint32
        L.h3o_gen_uniform.restype = c_f32
        L.h3o_fp8e4m3.restype = c_f32
        L.h3o_fp8e4m3.argtypes = [ctypes.c_uint8]
        L.h3o_nvfp4_scale_offset.restype = c_i64
        L.h3o_nvfp4_scale_offset.argtypes = [c_i64, c_i64, c_i64]
        L.h3o_quant_rows.restype = c_int
        L.h3o_hadamard.restype = c_int
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data) if a is not None else ctypes.c_void_p(0)


# ----------------------------------------------------------------------------- bf16 helpers (kernels.rs:17-23)

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16), NaN -> 0x7fc0."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ----------------------------------------------------------------------------- seeded generator (rng.rs:8-116)

class TorchGen:
    """rng.rs TorchGen: PyTorch's CPU mt19937 + normal_fill, one stream shared by consecutive draws."""

    def __init__(self, seed: int):
        self._buf = ctypes.create_string_buffer(lib().h3o_gen_size())
        lib().h3o_gen_init(self._buf, c_u64(seed))

    def randn(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().h3o_gen_randn(self._buf, _p(out), ctypes.c_size_t(n))
        return out

    def next_u32(self) -> int:
        return lib().h3o_gen_u32(self._buf)

    def uniform(self) -> float:
        return lib().h3o_gen_uniform(self._buf)


def make_linear_inputs(seed: int, M: int, K: int, N: int, n_outliers: int = 8):
    """Synthetic W8A8 inputs from one TorchGen stream (x bf16 bits [M,K], w int8 [N,K], ws f32 [N], bias f32 [N]);
    the draw order is documented in h3q_oracle.c (h3o_make_linear_inputs)."""
    x = np.empty((M, K), dtype=np.uint16)
    w = np.empty((N, K), dtype=np.int8)
    ws = np.empty(N, dtype=np.float32)
    bias = np.empty(N, dtype=np.float32)
    lib().h3o_make_linear_inputs(c_u64(seed), c_i64(M), c_i64(K), c_i64(N), c_int(n_outliers),
                                 _p(x), _p(w), _p(ws), _p(bias))
    return x, w, ws, bias


# ----------------------------------------------------------------------------- rotation / quantization

def hadamard(size: int = 256) -> np.ndarray:
    """weights.rs:441-465: normalised regular Hadamard (Kronecker powers of H4) as f32 [size, size]."""
    h = np.empty((size, size), dtype=np.float32)
    if lib().h3o_hadamard(c_int(size), _p(h)) != 0:
        raise ValueError(f"ConvRot group size {size} is not a power of 4")
    return h


def rotate_f64(x: np.ndarray) -> np.ndarray:
    """weights.rs:482-489 rotate_activation in exact (f64) arithmetic; x f32 [rows, K]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.float64)
    lib().h3o_rotate_f64(_p(x), _p(out), c_i64(x.shape[0]), c_i64(x.shape[1]))
    return out


QUANT_PLAIN, QUANT_ROT, QUANT_ROT2 = 0, 1, 2


def quant_rows(x: np.ndarray, kind: int, mode: int):
    """Per-row int8 quantizers: mode 0 quant_rows_i8 (kernels.rs:296-318), 1 quant_rows_i8_rot
    (kernels.rs:166-213), 2 quant_rows_i8_rot2 (kernels.rs:220-293).  x holds raw elements of `kind`
    (f32 array, or uint16 bit patterns for f16/bf16).  Returns (q int8 [M,K], scale f32 [M])."""
    x = np.ascontiguousarray(x)
    M, K = x.shape
    q = np.empty((M, K), dtype=np.int8)
    s = np.empty(M, dtype=np.float32)
    rc = lib().h3o_quant_rows(_p(x), c_int(kind), _p(q), _p(s), c_i64(M), c_i64(K), c_int(mode))
    if rc != 0:
        raise ValueError("unsupported quantizer arguments")
    return q, s


def reference_quant_mode(kind: int, K: int, rotate: bool) -> int:
    """The quantizer kernels::quant_rows_raw selects (kernels.rs:1139-1140)."""
    if rotate and kind == 2 and K % 256 == 0 and K // 256 <= 56:
        return QUANT_ROT2
    return QUANT_ROT if rotate else QUANT_PLAIN


def rotate_bf16(x_bf16: np.ndarray) -> np.ndarray:
    """rotate_activation(x, 256) on bf16 rows (weights.rs:482-489) in the rot2 butterfly order, bf16 bits out."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    out = np.empty_like(x)
    if lib().h3o_rotate_bf16(_p(x), _p(out), c_i64(x.shape[0]), c_i64(x.shape[1])) != 0:
        raise ValueError("ConvRot group 256 does not divide K")
    return out


def swiglu_bf16(y_bf16: np.ndarray, interleaved: bool) -> np.ndarray:
    """swiglu_interleaved (weights.rs:806-816) / ops::swiglu (ops.rs:39-44) on bf16 bits."""
    y = np.ascontiguousarray(y_bf16, dtype=np.uint16)
    rows, n = y.shape
    out = np.empty((rows, n // 2), dtype=np.uint16)
    lib().h3o_swiglu_bf16(_p(y), _p(out), c_i64(rows), c_i64(n // 2), c_int(1 if interleaved else 0))
    return out


def gemm_s8_acc(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """int32 accumulators sum_k a[m,k] b[n,k] (exact)."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    # int64 matmul is exact; the accumulators stay far inside int32 for K <= 2^17
    return (a.astype(np.int64) @ b.astype(np.int64).T).astype(np.int32)


EPI_LINEAR, EPI_SWIGLU_PAIRS, EPI_SWIGLU_HALVES, EPI_GELU, EPI_GATE_RESID, EPI_ACC = 0, 1, 2, 3, 4, 5


def gemm_s8_epilogue(acc, xs, ws, bias, epi=EPI_LINEAR, gate=None, gate_idx=None, resid=None) -> np.ndarray:
    """gemm_s8's fused epilogue (attn8.rs:320-343) plus the GELU / gated-residual variants; bf16 bits out."""
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    M, N = acc.shape
    ws = np.ascontiguousarray(ws, dtype=np.float32)
    per_row = 1 if (ws.size == N and N > 1) else 0
    out = np.empty((M, N // 2 if epi == EPI_SWIGLU_PAIRS else N), dtype=np.uint16)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    g = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32)
    gi = None if gate_idx is None else np.ascontiguousarray(gate_idx, dtype=np.uint32)
    r = None if resid is None else np.ascontiguousarray(resid, dtype=np.uint16)
    lib().h3o_gemm_s8_epilogue(_p(acc), _p(np.ascontiguousarray(xs, dtype=np.float32)), _p(ws), c_int(per_row),
                               _p(b), _p(out), c_i64(M), c_i64(N), c_int(epi), _p(g), _p(gi), _p(r))
    return out


def int8_epilogue(acc, xs, ws, bias, okind: int, swiglu: bool) -> np.ndarray:
    """int8_epilogue / int8_epilogue_swiglu of the cuBLASLt path (kernels.rs:333-373)."""
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    M, Nacc = acc.shape
    N = Nacc // 2 if swiglu else Nacc
    ws = np.ascontiguousarray(ws, dtype=np.float32)
    per_row = 1 if (ws.size == Nacc and Nacc > 1) else 0
    out = np.empty((M, N), dtype=np.float32 if okind == 0 else np.uint16)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().h3o_int8_epilogue(_p(acc), _p(np.ascontiguousarray(xs, dtype=np.float32)), _p(ws), c_int(per_row), _p(b),
                            _p(out), c_int(okind), c_i64(M), c_i64(N), c_int(1 if swiglu else 0))
    return out


def gemm_s8(x_bf16: np.ndarray, w: np.ndarray, ws, bias, swiglu: bool, rotate: bool):
    """attn8::gemm_s8 restated (attn8.rs:570-581 -> quant_rows_raw + gemm_s8 kernel).
    Returns (out bf16 bits, q, xs, acc)."""
    K = x_bf16.shape[1]
    q, xs = quant_rows(x_bf16, 2, reference_quant_mode(2, K, rotate))
    acc = gemm_s8_acc(q, w)
    out = gemm_s8_epilogue(acc, xs, ws, bias, EPI_SWIGLU_PAIRS if swiglu else EPI_LINEAR)
    return out, q, xs, acc


def dequant_i8(q: np.ndarray, scale: np.ndarray, okind: int = 0) -> np.ndarray:
    """kernels.rs:40-49 / portable/kernels.rs:14-27; scale per row iff it has `rows` entries and rows > 1."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    rows, cols = q.shape
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    per_row = 1 if (scale.size == rows and rows > 1) else 0
    out = np.empty((rows, cols), dtype=np.float32 if okind == 0 else np.uint16)
    lib().h3o_dequant_i8(_p(q), _p(scale), c_int(per_row), _p(out), c_int(okind), c_i64(rows), c_i64(cols))
    return out


def fp8e4m3(v: int) -> float:
    return lib().h3o_fp8e4m3(v)


def nvfp4_scale_offset(r: int, b: int, k: int) -> int:
    return lib().h3o_nvfp4_scale_offset(r, b, k)


def dequant_nvfp4(q: np.ndarray, bs: np.ndarray, g: float, okind: int = 0) -> np.ndarray:
    """kernels.rs:65-81 / portable/kernels.rs:46-70."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    rows, kp = q.shape
    k = 2 * kp
    out = np.empty((rows, k), dtype=np.float32 if okind == 0 else np.uint16)
    lib().h3o_dequant_nvfp4(_p(q), _p(np.ascontiguousarray(bs, dtype=np.uint8)), c_f32(g), _p(out), c_int(okind),
                            c_i64(rows), c_i64(k))
    return out


def make_nvfp4_inputs(seed: int, M: int, K: int, N: int):
    """Synthetic NVFP4+AWQ layer: e2m1 codes uniform over the 16 values (two per byte), e4m3
    block scales drawn uniformly from the e4m3 values in [0.5, 4] and laid out in the 128x4 swizzle, global scale
    1/448, AWQ pre-quant scale ~U(0.5, 2) rounded to bf16, x ~N(0, 1) in bf16, bias ~N(0, 0.02).  numpy PCG64
    stream from `seed`.  Returns (x bits, q, bs, g, pqs bits, bias)."""
    rng = np.random.default_rng(seed)
    x = f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    q = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    e4m3_pool = np.array([(e << 3) | m for e in (6, 7, 8) for m in range(8)] + [9 << 3], dtype=np.uint8)
    ncb = (K // 16 + 3) // 4
    bs = np.zeros(((N + 127) // 128) * ncb * 512, dtype=np.uint8)
    vals = rng.choice(e4m3_pool, size=(N, K // 16))
    r_idx, b_idx = np.meshgrid(np.arange(N), np.arange(K // 16), indexing="ij")
    off = (r_idx // 128 * ncb + b_idx // 4) * 512 + (r_idx % 32) * 16 + (r_idx % 128 // 32) * 4 + b_idx % 4
    bs[off.ravel()] = vals.ravel()
    pqs = f32_to_bf16_bits((rng.random(K) * 1.5 + 0.5).astype(np.float32))
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    return x, q, bs, np.float32(1.0 / 448.0), pqs, bias


def nvfp4_linear(x_bf16, q, bs, g, pqs_bf16=None, bias=None, rows=None) -> np.ndarray:
    """QLinear::apply for NVFP4 (weights.rs:612-635): x2 = bf16(x * pqs), W = dequant_nvfp4 -> bf16, y = bf16(x2 W^T)
    (exact f64 products and sums here; cuBLAS accumulates in f32), + bias added in bf16.  bf16 bits out."""
    x = bf16_bits_to_f32(x_bf16 if rows is None else x_bf16[rows])
    if pqs_bf16 is not None:
        x = bf16_round(x * bf16_bits_to_f32(pqs_bf16)[None, :])
    w = bf16_bits_to_f32(dequant_nvfp4(q, bs, float(g), 2))
    y = bf16_round((x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32))
    if bias is not None:
        y = bf16_round(y + bf16_round(np.asarray(bias, dtype=np.float32))[None, :])
    return f32_to_bf16_bits(y)


_E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _e4m3_values() -> np.ndarray:
    """The 127 non-negative finite e4m3 values (bias 7, 3 mantissa bits, subnormals, max 448), in code order."""
    return np.array([fp8e4m3(c) for c in range(127)], dtype=np.float64)


def _round_to_table(a: np.ndarray, table: np.ndarray) -> np.ndarray:
    """|a| rounded to the nearest entry of an ascending table (ties to the even index, as RNE picks the even
    mantissa), saturating at the last entry; the sign of a is kept."""
    m = np.minimum(np.abs(a), table[-1])
    hi = np.clip(np.searchsorted(table, m), 1, len(table) - 1)
    lo = hi - 1
    dlo, dhi = m - table[lo], table[hi] - m
    pick = np.where(dhi < dlo, hi, np.where(dlo < dhi, lo, np.where(lo % 2 == 0, lo, hi)))
    return np.sign(a) * table[pick]


def nvfp4_quantize_activation(x: np.ndarray, block: int = 16):
    """NVFP4 quantization of activations [M, K] as the published two-level NVFP4 recipe defines it: one f32
    global scale gs = amax(x) / (448 * 6), one e4m3 scale per 16 consecutive elements along K,
    sb = e4m3(amax_block / 6 / gs) (RNE, saturating), and e2m1 values q = e2m1(x / (sb * gs)) (RNE, saturating
    at +-6).  The reference has no activation quantizer for this layer (weights.rs:612-635 multiplies bf16
    activations); this is what a W4A4 kernel (tcgen05 kind::mxf4nvf4) would need.  Returns the dequantized
    activations q * sb * gs (f64)."""
    x = np.asarray(x, dtype=np.float64)
    M, K = x.shape
    amax = float(np.max(np.abs(x)))
    if amax == 0.0:
        return np.zeros_like(x)
    gs = amax / (448.0 * 6.0)
    xb = x.reshape(M, K // block, block)
    sb = _round_to_table(np.max(np.abs(xb), axis=2) / 6.0 / gs, _e4m3_values())
    den = (sb * gs)[:, :, None]
    q = _round_to_table(np.divide(xb, den, out=np.zeros_like(xb), where=den > 0), _E2M1_VALUES)
    return (q * den).reshape(M, K)


def nvfp4_linear_w4a4(x_bf16, q, bs, g, pqs_bf16=None, bias=None, rows=None) -> np.ndarray:
    """The NVFP4 linear with the AWQ-scaled activations also quantized to NVFP4 (nvfp4_quantize_activation):
    y = bf16(Q(bf16(x * pqs)) W^T) + bias, with the same weight decode and roundings as nvfp4_linear.  Used to
    measure how far W4A4 moves the layer from the reference's W4A16 result.  bf16 bits out."""
    x = bf16_bits_to_f32(x_bf16 if rows is None else x_bf16[rows])
    if pqs_bf16 is not None:
        x = bf16_round(x * bf16_bits_to_f32(pqs_bf16)[None, :])
    xq = nvfp4_quantize_activation(x)
    w = bf16_bits_to_f32(dequant_nvfp4(q, bs, float(g), 2))
    y = bf16_round((xq @ w.astype(np.float64).T).astype(np.float32))
    if bias is not None:
        y = bf16_round(y + bf16_round(np.asarray(bias, dtype=np.float32))[None, :])
    return f32_to_bf16_bits(y)


def gate_add(x, y, kind: int, gate, idx) -> np.ndarray:
    """kernels.rs:418-428."""
    x = np.ascontiguousarray(x)
    S, C = x.shape
    out = np.empty_like(x)
    lib().h3o_gate_add(_p(x), _p(np.ascontiguousarray(y)), c_int(kind), _p(np.ascontiguousarray(gate, dtype=np.float32)),
                       _p(np.ascontiguousarray(idx, dtype=np.uint32)), _p(out), c_i64(S), c_i64(C))
    return out


# ----------------------------------------------------------------------------- the reference's CPU path

def cpu_dequant_weight(w: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """dequant_i8 to the activation dtype (bf16, held as f32 values): the per-call weight decode of the
    reference's CPU path (portable/kernels.rs:14-27 via weights.rs:598-604)."""
    return bf16_bits_to_f32(dequant_i8(w, scale, 2))


def cpu_linear_rows(x_bf16: np.ndarray, wd: np.ndarray, bias, rotate: bool, swiglu: bool = False) -> np.ndarray:
    """The row-dependent part of portable::int8_linear_ex (portable/kernels.rs:220-242) on bf16 activations:
    rotate_activation as a matmul with the Hadamard in the activation dtype (weights.rs:482-489; result rounded
    to bf16), float matmul with the dequantised weight (f32 accumulation here), + bias, optional split-half
    SwiGLU (ops.rs:39-44), bf16 output (bits).  No activation quantization."""
    x = bf16_bits_to_f32(x_bf16)
    M, K = x.shape
    if rotate:
        h = bf16_round(hadamard(256))
        x = bf16_round((x.reshape(-1, 256) @ h).reshape(M, K))
    y = bf16_round(x @ wd.T)
    if bias is not None:
        y = bf16_round(y + bf16_round(np.asarray(bias, dtype=np.float32))[None, :])
    if swiglu:
        f = y.shape[1] // 2
        g, u = y[:, :f], y[:, f:]
        y = bf16_round(bf16_round(g / (1.0 + np.exp(-g))) * u)
    return f32_to_bf16_bits(y)


def cpu_int8_linear(x_bf16: np.ndarray, w: np.ndarray, scale: np.ndarray, bias, rotate: bool, swiglu: bool = False):
    """portable::int8_linear_ex (portable/kernels.rs:220-242): dequantise, then the float linear.  This is the
    reference's CPU semantics and the timed CPU baseline.  Returns bf16 bits."""
    return cpu_linear_rows(x_bf16, cpu_dequant_weight(w, scale), bias, rotate, swiglu)


def max_abs_rel(y: np.ndarray, r: np.ndarray) -> float:
    """max|y - r| / max|r|, the tolerance measure of the parity contract."""
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    den = np.max(np.abs(r))
    return float(np.max(np.abs(y - r)) / den) if den > 0 else float(np.max(np.abs(y - r)))


# ----------------------------------------------------------------------------- int8 attention (attn8.rs)

ATTN_SCALE_BLOCK128 = 1
ATTN_PV_BF16 = 2


def make_attn_inputs(seed: int, S: int, H: int, k_offset: float = 0.0):
    """Seeded q, k, v bf16 bits [S, H, 128] ~ N(0, 1) drawn in that order from one TorchGen stream.  k_offset > 0
    adds a per-(head, dim) offset ~ N(0, k_offset) to K, the outlier channels of real keys that the reference's
    attention bench builds (examples/attn_bench.rs) and its mean smoothing removes."""
    g = TorchGen(seed)
    n = S * H * 128
    q = f32_to_bf16_bits(g.randn(n).reshape(S, H, 128))
    k = g.randn(n).reshape(S, H, 128)
    v = f32_to_bf16_bits(g.randn(n).reshape(S, H, 128))
    if k_offset:
        k = k + (g.randn(H * 128) * np.float32(k_offset)).reshape(1, H, 128)
    return q, f32_to_bf16_bits(k.astype(np.float32)), v


def attn_kmean(k_bf16: np.ndarray) -> np.ndarray:
    """ColMean / S (attn8.rs:45-52, :429-455, :622) in the fixed chunk order.  f32 [H, 128]."""
    k = np.ascontiguousarray(k_bf16, dtype=np.uint16)
    S, H = k.shape[0], k.shape[1]
    out = np.empty((H, 128), dtype=np.float32)
    lib().h3o_attn_kmean(_p(k), c_i64(S), c_i64(H), _p(out))
    return out


def attn_quant_heads(x_bf16: np.ndarray, mean=None, block128: bool = False):
    """QuantHeads (attn8.rs:69-93): codes int8 [H, S, 128], scales f32 [H, roundup(S, 128)]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    S, H = x.shape[0], x.shape[1]
    Sp = (S + 127) // 128 * 128
    codes = np.empty((H, S, 128), dtype=np.int8)
    scales = np.empty((H, Sp), dtype=np.float32)
    m = None if mean is None else np.ascontiguousarray(mean, dtype=np.float32)
    lib().h3o_attn_quant_heads(_p(x), _p(m), _p(codes), _p(scales), c_i64(S), c_i64(H), c_int(1 if block128 else 0))
    return codes, scales


def attn_scores(q8: np.ndarray, k8: np.ndarray) -> np.ndarray:
    """int32 Q.K^T [H, S, S] of codes [H, S, 128]."""
    H, S = q8.shape[0], q8.shape[1]
    out = np.empty((H, S, S), dtype=np.int32)
    lib().h3o_attn_scores(_p(np.ascontiguousarray(q8)), _p(np.ascontiguousarray(k8)), c_i64(S), c_i64(H), _p(out))
    return out


def attn_scale_log2() -> float:
    lib().h3o_attn_scale_log2.restype = c_f32
    return float(lib().h3o_attn_scale_log2())


def attn_forward(q8, qs, k8, ks, vsrc_bf16, v_rs: int, v_col: int, pv_bf16: bool = False) -> np.ndarray:
    """attn_qk8 (attn8.rs:107-246) on prepared codes / scales, V from rows of vsrc (bf16 bits, row stride v_rs,
    head h at column v_col + 128 h).  bf16 bits [S, H, 128]."""
    H, S = q8.shape[0], q8.shape[1]
    out = np.empty((S, H, 128), dtype=np.uint16)
    v = np.ascontiguousarray(vsrc_bf16, dtype=np.uint16)
    lib().h3o_attn_forward(_p(np.ascontiguousarray(q8)), _p(np.ascontiguousarray(qs, dtype=np.float32)),
                           _p(np.ascontiguousarray(k8)), _p(np.ascontiguousarray(ks, dtype=np.float32)), _p(v),
                           c_i64(v_rs), c_i64(v_col), _p(out), c_i64(S), c_i64(H), c_int(1 if pv_bf16 else 0))
    return out


def attn_forward_rows(q8, qs, k8, ks, vsrc_bf16, v_rs: int, v_col: int, pv_bf16: bool = False) -> np.ndarray:
    """attn_forward for Sq query rows (codes [H, Sq, 128], scales [H, roundup(Sq, 128)]) against S keys.
    bf16 bits [Sq, H, 128]."""
    H, Sq = q8.shape[0], q8.shape[1]
    S = k8.shape[1]
    out = np.empty((Sq, H, 128), dtype=np.uint16)
    v = np.ascontiguousarray(vsrc_bf16, dtype=np.uint16)
    lib().h3o_attn_forward_rows(_p(np.ascontiguousarray(q8)), _p(np.ascontiguousarray(qs, dtype=np.float32)),
                                c_i64(Sq), _p(np.ascontiguousarray(k8)),
                                _p(np.ascontiguousarray(ks, dtype=np.float32)), _p(v), c_i64(v_rs), c_i64(v_col),
                                _p(out), c_i64(S), c_i64(H), c_int(1 if pv_bf16 else 0))
    return out


def attention_rows(q_bf16, k_bf16, v_bf16, flags: int = 0) -> np.ndarray:
    """h3q_attention_rows: query rows q [Sq, H, 128] against keys / values [S, H, 128]; bf16 bits [Sq, H, 128]."""
    S, H = k_bf16.shape[0], k_bf16.shape[1]
    block = bool(flags & ATTN_SCALE_BLOCK128)
    km = attn_kmean(k_bf16)
    q8, qs = attn_quant_heads(q_bf16, None, block)
    k8, ks = attn_quant_heads(k_bf16, km, block)
    return attn_forward_rows(q8, qs, k8, ks, np.ascontiguousarray(v_bf16).reshape(S, H * 128), H * 128, 0,
                             bool(flags & ATTN_PV_BF16))


def attention(q_bf16, k_bf16, v_bf16, flags: int = 0) -> np.ndarray:
    """attention(q, k, v) (attn8.rs:611-627): K mean, Q / K quantisation, int8 attention.  bf16 bits [S, H, 128]."""
    S, H = q_bf16.shape[0], q_bf16.shape[1]
    block = bool(flags & ATTN_SCALE_BLOCK128)
    km = attn_kmean(k_bf16)
    q8, qs = attn_quant_heads(q_bf16, None, block)
    k8, ks = attn_quant_heads(k_bf16, km, block)
    return attn_forward(q8, qs, k8, ks, np.ascontiguousarray(v_bf16).reshape(S, H * 128), H * 128, 0,
                        bool(flags & ATTN_PV_BF16))


def attention_exact(q_bf16, k_bf16, v_bf16) -> np.ndarray:
    """Softmax attention in f64 on the bf16 inputs (no quantisation): the float semantics the int8 attention
    approximates (ops.rs:72-109 attention_fallback, non-causal).  f64 [S, H, 128]."""
    q = bf16_bits_to_f32(q_bf16).astype(np.float64)
    k = bf16_bits_to_f32(k_bf16).astype(np.float64)
    v = bf16_bits_to_f32(v_bf16).astype(np.float64)
    out = np.empty_like(q)
    for h in range(q.shape[1]):
        s = q[:, h, :] @ k[:, h, :].T / np.sqrt(128.0)
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out[:, h, :] = (p / p.sum(axis=1, keepdims=True)) @ v[:, h, :]
    return out


# ----------------------------------------------------------------------------- RMSNorm + adaLN modulate

def rms_modulate(x_bf16, w_bf16, eps: float, scale, shift, idx) -> np.ndarray:
    """rms_modulate (kernels.rs:376-401), the reduction in the reference kernel's order; bf16 bits [S, C].  The
    reference's rsqrtf is an approximate instruction; 1 / sqrtf here can differ from it in the last bit."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    S, C = x.shape
    out = np.empty_like(x)
    lib().h3o_rms_modulate(_p(x), _p(np.ascontiguousarray(w_bf16, dtype=np.uint16)), c_f32(eps),
                           _p(np.ascontiguousarray(scale, dtype=np.float32)),
                           _p(np.ascontiguousarray(shift, dtype=np.float32)),
                           _p(np.ascontiguousarray(idx, dtype=np.uint32)), _p(out), c_i64(S), c_i64(C))
    return out


def qk_norm_rope(x_bf16, col_off: int, heads: int, head_dim: int, w_bf16=None, eps: float = 1e-6,
                 do_norm: bool = True, cs=None, rot: int = 0, head_stride: int | None = None) -> np.ndarray:
    """qk_norm_rope (kernels.rs:86-126) on bf16 bits x [S, width]; w bf16 bits [D] or None; cs f32 [2, S, rot/2] or
    None.  bf16 bits [S, heads, head_dim].  1 / sqrtf stands for the device's rsqrtf."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    S, width = x.shape
    out = np.empty((S, heads, head_dim), dtype=np.uint16)
    wv = None if w_bf16 is None else np.ascontiguousarray(w_bf16, dtype=np.uint16)
    csv = None if cs is None else np.ascontiguousarray(cs, dtype=np.float32)
    lib().h3o_qk_norm_rope(_p(x), c_i64(width), c_i64(col_off), c_i64(head_dim if head_stride is None else head_stride),
                           _p(wv) if wv is not None else None, c_int(1 if do_norm else 0), c_f32(eps),
                           _p(csv) if csv is not None else None, c_int(rot if csv is not None else 0), _p(out), c_i64(S),
                           c_i64(heads), c_i64(head_dim))
    return out


def attend_qkv(qkv_bf16, heads: int, qw=None, kw=None, do_norm: bool = True, eps: float = 1e-6, cs=None,
               rot: int = 0, flags: int = 0) -> np.ndarray:
    """The DiT's attend (dit.rs:741-757): qk_norm_rope of q and k out of the fused qkv, then attention_qkv with V
    from the qkv rows.  bf16 bits [S, heads, 128]."""
    S = qkv_bf16.shape[0]
    inner = heads * 128
    q = qk_norm_rope(qkv_bf16, 0, heads, 128, qw, eps, do_norm, cs, rot)
    k = qk_norm_rope(qkv_bf16, inner, heads, 128, kw, eps, do_norm, cs, rot)
    block = bool(flags & ATTN_SCALE_BLOCK128)
    km = attn_kmean(k)
    q8, qs = attn_quant_heads(q, None, block)
    k8, ks = attn_quant_heads(k, km, block)
    return attn_forward(q8, qs, k8, ks, np.ascontiguousarray(qkv_bf16), qkv_bf16.shape[1], 2 * inner,
                        bool(flags & ATTN_PV_BF16))


def make_rope_inputs(seed: int, S: int, H: int, D: int = 128, rot: int = 96):
    """DiT-like inputs of the attention step: a fused qkv bf16 [S, 3 H D] ~N(0, 1) with per-token magnitudes in
    [1, 4], norm weights bf16 ~1 + N(0, 0.2), and a rope table [2, S, rot/2] of cos / sin of angles in [0, 100)
    rounded through bf16 (as the DiT stores it, dit.rs:803-819)."""
    rng = np.random.default_rng(seed)
    qkv = rng.standard_normal((S, 3 * H * D)).astype(np.float32) * (1 + 3 * rng.random((S, 1), dtype=np.float32))
    qw = (1.0 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    kw = (1.0 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    ang = (100.0 * rng.random((S, rot // 2))).astype(np.float32)
    cs = np.stack([np.cos(ang), np.sin(ang)]).astype(np.float32)
    cs = bf16_bits_to_f32(f32_to_bf16_bits(cs)).reshape(2, S, rot // 2)
    return f32_to_bf16_bits(qkv), f32_to_bf16_bits(qw), f32_to_bf16_bits(kw), np.ascontiguousarray(cs)


def make_modulate_inputs(seed: int, S: int, C: int, R: int = 3):
    """DiT-like inputs of rms_modulate: x bf16 ~N(0, 1) with 8 outlier channels x20, norm weight bf16 ~1 + N(0, 0.1),
    adaLN scale / shift tables f32 ~N(0, 0.5) with R rows, idx u32 [S] in [0, R)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((S, C)).astype(np.float32)
    x[:, rng.choice(C, 8, replace=False)] *= 20.0
    w = (1.0 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    scale = (0.5 * rng.standard_normal((R, C))).astype(np.float32)
    shift = (0.5 * rng.standard_normal((R, C))).astype(np.float32)
    idx = rng.integers(0, R, S).astype(np.uint32)
    return f32_to_bf16_bits(x), f32_to_bf16_bits(w), scale, shift, idx


# ----------------------------------------------------------------------------- LoRA merge (weights.rs:692-761)

def _lora_ptrs(loras):
    """(a [r, k], b [n, r], scale) with f32 (or bf16-widened) factors -> the C oracle's pointer arrays."""
    m = max(len(loras), 1)
    pa, pb = (c_vp * m)(), (c_vp * m)()
    ranks, scales = np.zeros(m, dtype=np.int64), np.zeros(m, dtype=np.float64)
    keep = []
    for i, (a, b, s) in enumerate(loras):
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        keep += [a, b]
        pa[i], pb[i] = a.ctypes.data, b.ctypes.data
        ranks[i], scales[i] = a.shape[0], float(s)
    return pa, pb, ranks, scales, keep


def lora_merge_i8(q: np.ndarray, scale: np.ndarray, loras, convrot: int = 256):
    """QLinear::merge_loras for an int8 layer (weights.rs:716-757): dequantize, rotate back, add the deltas,
    rotate, requantize per row.  loras: (a f32 [r, k], b f32 [n, r], scale).  Returns (q' int8 [n, k],
    s' f32 [n]); with no LoRA the inputs come back (weights.rs:693-695)."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    n, k = q.shape
    scale = np.ascontiguousarray(scale, dtype=np.float32).reshape(-1)
    if not loras:
        return q, scale
    pa, pb, ranks, scales, keep = _lora_ptrs(loras)
    qo = np.empty((n, k), dtype=np.int8)
    so = np.empty(n, dtype=np.float32)
    rc = lib().h3o_lora_merge_i8(_p(q), _p(scale), c_int(1 if scale.size == n else 0), c_int(convrot),
                                 c_int(len(loras)), pa, pb, _p(ranks), _p(scales), _p(qo), _p(so), c_i64(n), c_i64(k))
    if rc != 0:
        raise ValueError("unsupported LoRA merge arguments")
    del keep
    return qo, so


def lora_merge_dense(w: np.ndarray, loras) -> np.ndarray:
    """QLinear::merge_loras for a dense layer before the cast back (weights.rs:710-715): f32(w) + deltas."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    pa, pb, ranks, scales, keep = _lora_ptrs(loras)
    out = np.empty((n, k), dtype=np.float32)
    lib().h3o_lora_merge_dense(_p(w), c_int(len(loras)), pa, pb, _p(ranks), _p(scales), _p(out), c_i64(n), c_i64(k))
    del keep
    return out


def lora_merge_i8_f64(q: np.ndarray, scale: np.ndarray, loras, convrot: int = 256):
    """The same merge in f64 with the exact rotation (x @ H), no rounding until the codes: an order-free
    restatement of weights.rs:716-757 for checking the f32 oracle.  Returns (codes int8, scales f64)."""
    q = np.asarray(q, dtype=np.int8)
    n, k = q.shape
    scale = np.asarray(scale, dtype=np.float32).reshape(-1)
    s = scale.astype(np.float64) if scale.size == n else np.full(n, float(scale[0]))
    w = q.astype(np.float64) * s[:, None]
    H = hadamard(256).astype(np.float64) if convrot else None
    rot = (lambda x: (x.reshape(-1, 256) @ H).reshape(x.shape)) if convrot else (lambda x: x)
    w = rot(w)
    for a, b, sc in loras:
        w = w + float(np.float32(sc)) * (np.asarray(b, np.float64) @ np.asarray(a, np.float64))
    w = rot(w)
    m = np.abs(w).max(axis=1)
    so = np.maximum(m / 127.0, 1e-30)
    r = w / so[:, None]
    codes = np.clip(np.sign(r) * np.floor(np.abs(r) + 0.5), -128, 127).astype(np.int8)
    return codes, so
