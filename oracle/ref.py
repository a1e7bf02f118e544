"""TEST INFRASTRUCTURE ONLY -- the reference's own CUDA C kernels (kernels.rs / attn8.rs raw strings),
compiled for sm_100a into oracle/_ref/libh3ref.so by `make -C oracle ref`, launched exactly as the
reference's host code launches them.  Used by GPU tests to pin the CPU oracle and the h3q kernels to the
reference's actual device results.  Takes torch CUDA tensors.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def path() -> str:
    return os.path.join(_HERE, "_ref", "libh3ref.so")


def available() -> bool:
    return os.path.exists(path())


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(path())
        for name in ("h3ref_quant_rows", "h3ref_quant_rows_linear", "h3ref_int8_epilogue", "h3ref_dequant_i8",
                     "h3ref_dequant_nvfp4", "h3ref_gate_add", "h3ref_gemm_s8", "h3ref_col_sum",
                     "h3ref_quant_heads", "h3ref_v_to_f16", "h3ref_attn_qk8", "h3ref_rms_modulate", "h3ref_qk_norm_rope"):
            getattr(_LIB, name).restype = ctypes.c_int
    return _LIB


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what}: CUDA error {rc}")


def quant_rows(x, kind: int, rotate: bool, linear_path: bool = False):
    """quant_rows_raw (kernels.rs:1133-1161) or, with linear_path, Int8Linear's quantizer (kernels.rs:979-991)."""
    import torch
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    fn = lib().h3ref_quant_rows_linear if linear_path else lib().h3ref_quant_rows
    _check(fn(_ptr(x), kind, _ptr(q), _ptr(s), M, K, int(rotate), _stream()), "ref quant_rows")
    return q, s


def gemm_s8(a, b, xs, ws, bias, swiglu: bool):
    """The gemm_s8 kernel (attn8.rs:258-344) on pre-quantized rows; bf16 out as int16 view."""
    import torch
    M, K = a.shape
    N = b.shape[0]
    out = torch.empty((M, N // 2 if swiglu else N), dtype=torch.bfloat16, device=a.device)
    per_row = int(ws.numel() == N and N > 1)
    _check(lib().h3ref_gemm_s8(_ptr(a), _ptr(b), _ptr(xs), _ptr(ws), per_row, _ptr(bias), int(bias is not None),
                               _ptr(out), M, N, K, int(swiglu), _stream()), "ref gemm_s8")
    return out


def int8_epilogue(acc, xs, ws, bias, out_dtype, swiglu: bool):
    import torch
    M, Nacc = acc.shape
    n_out = Nacc // 2 if swiglu else Nacc
    out = torch.empty((M, n_out), dtype=out_dtype, device=acc.device)
    okind = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[out_dtype]
    per_row = int(ws.numel() == Nacc and Nacc > 1)
    _check(lib().h3ref_int8_epilogue(_ptr(acc), _ptr(xs), _ptr(ws), per_row, _ptr(bias), int(bias is not None),
                                     _ptr(out), okind, ctypes.c_ulonglong(M), ctypes.c_ulonglong(n_out), int(swiglu),
                                     _stream()), "ref int8_epilogue")
    return out


def dequant_nvfp4(q, bs, g, out_dtype):
    import torch
    rows, kp = q.shape
    out = torch.empty((rows, 2 * kp), dtype=out_dtype, device=q.device)
    okind = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[out_dtype]
    _check(lib().h3ref_dequant_nvfp4(_ptr(q), _ptr(bs), _ptr(g), _ptr(out), ctypes.c_ulonglong(rows),
                                     ctypes.c_ulonglong(2 * kp), okind, _stream()), "ref dequant_nvfp4")
    return out


def col_mean(k):
    """ColMean then / S (attn8.rs:429-455, :622), with the reference's atomicAdd chunk sums: f32 [H, 128]."""
    import torch
    S, H, _ = k.shape
    acc = torch.zeros(H * 128, dtype=torch.float32, device=k.device)
    _check(lib().h3ref_col_sum(_ptr(k), _ptr(acc), S, H * 128, _stream()), "ref col_sum")
    return (acc * torch.tensor(1.0 / S, dtype=torch.float64).to(torch.float32).item()).reshape(H, 128)


def quant_heads(x, mean=None):
    """QuantHeads (attn8.rs:395-427): codes int8 [H, S, 128] and scales f32 [H, S]."""
    import torch
    S, H, _ = x.shape
    codes = torch.empty((H, S, 128), dtype=torch.int8, device=x.device)
    scales = torch.empty((H, S), dtype=torch.float32, device=x.device)
    _check(lib().h3ref_quant_heads(_ptr(x), _ptr(mean), _ptr(codes), _ptr(scales), S, H, _stream()), "ref quant_heads")
    return codes, scales


def v_to_f16(src, row_stride: int, col_off: int, S: int, H: int):
    """VToF16 (attn8.rs:457-486): [H, S, 128] f16."""
    import torch
    out = torch.empty((H, S, 128), dtype=torch.float16, device=src.device)
    _check(lib().h3ref_v_to_f16(_ptr(src), ctypes.c_ulonglong(row_stride), ctypes.c_ulonglong(col_off), _ptr(out), S,
                                H, _stream()), "ref v_to_f16")
    return out


def attn_qk8(q8, qs, k8, ks, v16, scale_log2: float):
    """attn_qk8 (attn8.rs:107-246): codes [H, S, 128], scales [H, S], V f16 [H, S, 128] -> bf16 [S, H, 128]."""
    import torch
    H, S, _ = q8.shape
    out = torch.empty((S, H, 128), dtype=torch.bfloat16, device=q8.device)
    _check(lib().h3ref_attn_qk8(_ptr(q8), _ptr(qs), _ptr(k8), _ptr(ks), _ptr(v16), _ptr(out), S, H,
                                ctypes.c_float(scale_log2), _stream()), "ref attn_qk8")
    return out


def rms_modulate(x, w, eps: float, scale, shift, idx):
    """rms_modulate (kernels.rs:376-401), the reference's launch: bf16 [S, C]."""
    import torch
    S, C = x.shape
    out = torch.empty_like(x)
    _check(lib().h3ref_rms_modulate(_ptr(x), 2, _ptr(w), ctypes.c_float(eps), _ptr(scale), _ptr(shift), _ptr(idx),
                                    _ptr(out), S, C, _stream()), "ref rms_modulate")
    return out


def qk_norm_rope(x, col_off: int, head_stride: int, H: int, D: int, w, eps: float, do_norm: bool, cs, rot: int):
    """qk_norm_rope (kernels.rs:86-126), the reference's launch: x bf16 [S, width] -> bf16 [S, H, D]; w bf16 [D] or
    None; cs f32 [2, S, rot/2] or None (rot is then 0)."""
    import torch
    S, width = x.shape
    out = torch.empty((S, H, D), dtype=torch.bfloat16, device=x.device)
    if cs is None:
        rot = 0
    _check(lib().h3ref_qk_norm_rope(_ptr(x), 2, ctypes.c_ulonglong(width), ctypes.c_ulonglong(col_off),
                                    ctypes.c_ulonglong(head_stride), _ptr(w), 2, int(w is not None), int(do_norm),
                                    ctypes.c_float(eps), _ptr(cs), rot, _ptr(out), 2, S, H, D, _stream()),
           "ref qk_norm_rope")
    return out
