"""h3q -- Python binding of the B200 quantized-linear library (lib/libh3q.so, C ABI in include/h3q.h).

The functions mirror h3-rs's op API (attn8::gemm_s8, kernels::int8_linear_ex, kernels::dequant_i8, ...): they
take torch CUDA tensors, allocate outputs and workspaces with torch's allocator, and call the C ABI on the
current stream.  There is no fallback: if libh3q.so is missing or the device is not sm_100, calls raise.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libh3q.so")
_LIB = None

OK, ERR_ARG, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_NCCL, ERR_WORKSPACE = range(7)
EPI_LINEAR, EPI_SWIGLU_PAIRS, EPI_SWIGLU_HALVES, EPI_GELU_TANH, EPI_GATE_RESID, EPI_ACC_I32 = range(6)

_vp, _i64, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t

class QLinearDesc(ctypes.Structure):
    """h3q_qlinear: an int8 layer as weights.rs's QLinear holds it."""
    _fields_ = [("format", ctypes.c_int), ("convrot", ctypes.c_int), ("interleaved", ctypes.c_int),
                ("n_loras", ctypes.c_int), ("out_features", ctypes.c_int64), ("in_features", ctypes.c_int64),
                ("weight", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("scale_numel", ctypes.c_int64),
                ("bias", ctypes.c_void_p)]


class Switches(ctypes.Structure):
    """h3q_switches: H3_INT8, H3_GEMM, H3_ROT, H3_FUSED_ROT as explicit flags."""
    _fields_ = [("int8", ctypes.c_int), ("gemm_fused", ctypes.c_int), ("rot_fused", ctypes.c_int),
                ("fused_rot_linear", ctypes.c_int)]


class LoraDesc(ctypes.Structure):
    """h3q_lora: one low-rank delta scale * (b @ a) (weights.rs LoraDelta)."""
    _fields_ = [("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("rank", ctypes.c_int64), ("dtype", ctypes.c_int),
                ("scale", ctypes.c_double)]


class HostLinear(ctypes.Structure):
    """h3q_host_linear: one linear of a host-pipeline batch (the arguments of h3q_host_pipeline_gemm_s8)."""
    _fields_ = [("x_host", ctypes.c_void_p), ("w", ctypes.c_void_p), ("ws", ctypes.c_void_p), ("ws_numel", ctypes.c_int64),
                ("bias", ctypes.c_void_p), ("out_host", ctypes.c_void_p), ("m", ctypes.c_int64), ("n", ctypes.c_int64),
                ("k", ctypes.c_int64), ("swiglu", ctypes.c_int), ("rotate", ctypes.c_int)]


FMT_DENSE, FMT_INT8, FMT_NVFP4 = 0, 1, 2
ATTN_SCALE_TOKEN, ATTN_SCALE_BLOCK128, ATTN_PV_F16, ATTN_PV_BF16 = 0, 1, 0, 2
PATH_GEMM_S8, PATH_INT8_LINEAR, PATH_ROTATE_FUSED, PATH_ROTATE_SEPARATE, PATH_SWIGLU_FUSED, PATH_SWIGLU_AFTER = (
    1, 2, 4, 8, 16, 32)


# name -> (restype, argtypes) of every symbol include/h3q.h declares
SIGNATURES = {
    "h3q_last_error": (ctypes.c_char_p, []),
    "h3q_host_pipeline_create": (_int, [_i64, _i64, _i64, ctypes.POINTER(_vp)]),
    "h3q_host_pipeline_create_ex": (_int, [_i64, _i64, _i64, _int, _int, ctypes.POINTER(_vp)]),
    "h3q_host_pipeline_destroy": (None, [_vp]),
    "h3q_host_pipeline_gemm_s8": (_int, [_vp, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp]),
    "h3q_host_pipeline_run": (_int, [_vp, _vp, _int, _vp]),
    "h3q_streamer_create": (_int, [_sz, _int, ctypes.POINTER(_vp)]),
    "h3q_streamer_destroy": (None, [_vp]),
    "h3q_streamer_slot_bytes": (_sz, [_vp]),
    "h3q_streamer_fetch": (_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_sz), _int, _vp, ctypes.POINTER(_int),
                                  ctypes.POINTER(_vp)]),
    "h3q_streamer_release": (_int, [_vp, _int, _vp]),
    "h3q_checkpoint_open": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "h3q_checkpoint_close": (None, [_vp]),
    "h3q_checkpoint_count": (_i64, [_vp]),
    "h3q_checkpoint_name": (ctypes.c_char_p, [_vp, _i64]),
    "h3q_checkpoint_has": (_int, [_vp, ctypes.c_char_p]),
    "h3q_checkpoint_metadata": (ctypes.c_char_p, [_vp, ctypes.c_char_p]),
    "h3q_checkpoint_info": (_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_int), ctypes.POINTER(_int),
                                   ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_uint64)]),
    "h3q_checkpoint_read": (_int, [_vp, ctypes.c_char_p, _vp, ctypes.c_uint64]),
    "h3q_checkpoint_upload": (_int, [_vp, ctypes.c_char_p, _vp, ctypes.c_uint64, _int, _vp]),
    "h3q_checkpoint_qlinear": (_int, [_vp, ctypes.c_char_p, _vp]),
    "h3q_lora_merge_i8_workspace_size": (_sz, [_i64, _i64]),
    "h3q_lora_merge_i8": (_int, [_vp, _vp, _i64, _int, ctypes.POINTER(LoraDesc), _int, _vp, _vp, _i64, _i64, _vp,
                                 _sz, _vp]),
    "h3q_lora_merge_dense": (_int, [_vp, _int, ctypes.POINTER(LoraDesc), _int, _vp, _i64, _i64, _vp]),
    "h3q_version": (ctypes.c_char_p, []),
    "h3q_available_arch": (_int, [_int]),
    "h3q_init": (_int, [_int]),
    "h3q_rotate_activation": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "h3q_swiglu": (_int, [_vp, _vp, _int, _i64, _i64, _int, _vp]),
    "h3q_can_fuse_rotation": (_int, [_sz, _sz]),
    "h3q_device_status": (_int, [_int, ctypes.POINTER(_int)]),
    "h3q_quant_rows_i8": (_int, [_vp, _int, _vp, _vp, _i64, _i64, _int, _vp]),
    "h3q_gemm_s8_workspace_size": (_sz, [_i64, _i64]),
    "h3q_gemm_s8": (_int, [_vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp, _sz, _vp]),
    "h3q_int8_linear_workspace_size": (_sz, [_i64, _i64]),
    "h3q_int8_linear_ex": (_int, [_vp, _int, _vp, _vp, _i64, _vp, _vp, _int, _i64, _i64, _i64, _int, _int, _vp, _sz,
                                  _vp]),
    "h3q_gemm_s8_quantized": (_int, [_vp, _vp, _vp, _vp, _i64, _vp, _vp, _int, _i64, _i64, _i64, _int, _vp, _vp, _vp,
                                     _vp]),
    "h3q_gemm_s8_acc": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "h3q_dequant_i8": (_int, [_vp, _vp, _i64, _vp, _int, _i64, _i64, _vp]),
    "h3q_dequant_nvfp4": (_int, [_vp, _vp, _vp, _vp, _int, _i64, _i64, _vp]),
    "h3q_gate_add": (_int, [_vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _vp]),
    "h3q_gemm_s8_static": (_int, [_vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp]),
    "h3q_gemm_s8_static_status": (_int, [_int, ctypes.POINTER(_int)]),
    "h3q_comm_unique_id": (_int, [_vp]),
    "h3q_comm_init": (_int, [_int, _int, _vp, ctypes.POINTER(_vp)]),
    "h3q_comm_destroy": (_int, [_vp]),
    "h3q_comm_rank": (_int, [_vp]),
    "h3q_comm_size": (_int, [_vp]),
    "h3q_comm_allgather": (_int, [_vp, _vp, _vp, _sz, _vp]),
    "h3q_comm_barrier": (_int, [_vp, _vp]),
    "h3q_nsplit_range": (None, [_i64, _int, _int, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "h3q_gemm_s8_nsplit_workspace_size": (_sz, [_i64, _i64, _int, _int]),
    "h3q_gemm_s8_nsplit": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _i64, _vp, ctypes.POINTER(_vp), _i64, _i64, _i64, _vp,
                                  _sz, _vp]),
    "h3q_selftest_wait_timeout": (_int, [_int, ctypes.c_uint64, _vp, _vp]),
    "h3q_nvfp4_linear_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "h3q_nvfp4_linear": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "h3q_default_switches": (Switches, []),
    "h3q_qlinear_plan": (_int, [ctypes.POINTER(QLinearDesc), _int, _i64, _int, ctypes.POINTER(Switches)]),
    "h3q_qlinear_workspace_size": (_sz, [ctypes.POINTER(QLinearDesc), _int, _i64, _int, ctypes.POINTER(Switches)]),
    "h3q_qlinear_forward": (_int, [ctypes.POINTER(QLinearDesc), _vp, _int, _i64, _int, _vp, _vp, _sz,
                                   ctypes.POINTER(Switches), _vp]),
    "h3q_rms_modulate": (_int, [_vp, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "h3q_rms_modulate_quant": (_int, [_vp, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "h3q_attention_available": (_int, [_i64, _int, _int]),
    "h3q_attention_workspace_size": (_sz, [_i64, _i64, _int]),
    "h3q_attention": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _int, _vp, _sz, _vp]),
    "h3q_attention_qkv": (_int, [_vp, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _int, _vp, _sz, _vp]),
    "h3q_qk_norm_rope": (_int, [_vp, _i64, _i64, _i64, _vp, _int, ctypes.c_float, _vp, _int, _vp, _i64, _i64, _i64,
                                _vp]),
    "h3q_attend_qkv": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _vp, _int, ctypes.c_float, _vp, _int, _vp, _i64, _i64,
                              _int, _vp, _sz, _vp]),
    "h3q_attention_rows_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "h3q_attention_rows": (_int, [_vp, _i64, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _int, _vp, _sz, _vp]),
    "h3q_attn_kmean_workspace_size": (_sz, [_i64, _i64]),
    "h3q_peer_buffer_alloc": (_int, [_sz, ctypes.POINTER(_vp), _vp]),
    "h3q_peer_buffer_open": (_int, [_vp, ctypes.POINTER(_vp)]),
    "h3q_peer_buffer_close": (_int, [_vp]),
    "h3q_peer_buffer_free": (_int, [_vp]),
    "h3q_gemm_s8_allgather": (_int, [_vp, _vp, _vp, _vp, _i64, _vp, ctypes.POINTER(_vp), _int, _i64, _i64, _i64,
                                     _i64, _i64, _vp]),
    "h3q_attn_kmean": (_int, [_vp, _i64, _i64, _vp, _vp, _sz, _vp]),
    "h3q_attn_quant_heads": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _int, _vp]),
    "h3q_attn_v_layout": (_int, [_vp, _i64, _i64, _vp, _i64, _i64, _int, _vp]),
    "h3q_attention_core": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _vp, _vp]),
}


class H3QError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[h3q status {status}] {msg}")
        self.status = status


def lib() -> ctypes.CDLL:
    """The loaded libh3q.so (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"h3q native library not built: {LIB_PATH} (run `make -C h3-rs_b200`)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def last_error() -> str:
    return lib().h3q_last_error().decode()


def check(status: int) -> None:
    if status != OK:
        raise H3QError(status, last_error())


def _kind(dtype) -> int:
    import torch
    return {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]


def _p(t) -> int:
    return None if t is None else t.data_ptr()


def _stream(dev=None) -> int:
    import torch
    return torch.cuda.current_stream(dev).cuda_stream


def _cuda(*ts) -> None:
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("h3q: expected contiguous CUDA tensors")


def rotate_activation(x):
    """weights::rotate_activation(x, 256) for bf16 x [M, K]: bf16 [M, K]."""
    import torch
    _cuda(x)
    y = torch.empty_like(x)
    check(lib().h3q_rotate_activation(_p(x), _p(y), x.shape[0], x.shape[1], _stream(x.device)))
    return y


def swiglu(y, interleaved: bool = True):
    """swiglu_interleaved / ops::swiglu on y [rows, 2F] (f32, f16 or bf16): [rows, F]."""
    import torch
    _cuda(y)
    rows, n = y.shape
    out = torch.empty((rows, n // 2), dtype=y.dtype, device=y.device)
    check(lib().h3q_swiglu(_p(y), _p(out), _kind(y.dtype), rows, n // 2, int(interleaved), _stream(y.device)))
    return out


def init(device: int = 0) -> None:
    """h3q_init: the per-device set-up, done up front instead of on the first call."""
    check(lib().h3q_init(device))


def available_arch(device: int = 0) -> bool:
    """attn8::available_arch (attn8.rs:584-589) for this build: an sm_100 device."""
    return bool(lib().h3q_available_arch(device))


def can_fuse_rotation(k: int, group: int) -> bool:
    """kernels::can_fuse_rotation (kernels.rs:1081-1085)."""
    return bool(lib().h3q_can_fuse_rotation(k, group))


def device_status(device: int = 0) -> int:
    code = _int(0)
    lib().h3q_device_status(device, ctypes.byref(code))
    return code.value


def quant_rows(x, rotate: bool):
    """kernels::quant_rows_raw (kernels.rs:1133-1161): (int8 codes [M,K], f32 scales [M])."""
    import torch
    _cuda(x)
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    check(lib().h3q_quant_rows_i8(_p(x), _kind(x.dtype), _p(q), _p(s), M, K, int(rotate), _stream(x.device)))
    return q, s


def gemm_s8(x, w, ws, bias=None, swiglu: bool = False, rotate: bool = False, workspace=None):
    """attn8::gemm_s8 (attn8.rs:570-581): bf16 x [M,K] (quantized per row on the fly), int8 w [N,K] (int8 or
    uint8 bytes), f32 ws ([N] or scalar), f32 bias [N] or None -> bf16 [M,N] (or [M,N/2] with swiglu)."""
    import torch
    if x.dtype != torch.bfloat16:
        raise H3QError(ERR_ARG, "gemm_s8: bf16 input with K % 64 == 0 required")
    ws = ws.to(torch.float32).reshape(-1).contiguous()
    bias = None if bias is None else bias.to(torch.float32).contiguous()
    _cuda(x, w, ws, bias)
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty((M, N // 2 if swiglu else N), dtype=torch.bfloat16, device=x.device)
    need = lib().h3q_gemm_s8_workspace_size(M, K)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    check(lib().h3q_gemm_s8(_p(x), _p(w), _p(ws), ws.numel(), _p(bias), _p(out), M, N, K, int(swiglu), int(rotate),
                            _p(workspace), workspace.numel(), _stream(x.device)))
    return out


def int8_linear_ex(x, w, scale, bias=None, out_dtype=None, swiglu: bool = False, rotate: bool = False,
                   workspace=None):
    """kernels::int8_linear_ex (kernels.rs:1088-1097)."""
    import torch
    out_dtype = out_dtype or x.dtype
    scale = scale.to(torch.float32).reshape(-1).contiguous()
    bias = None if bias is None else bias.to(torch.float32).contiguous()
    _cuda(x, w, scale, bias)
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty((M, N // 2 if swiglu else N), dtype=out_dtype, device=x.device)
    need = lib().h3q_int8_linear_workspace_size(M, K)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    check(lib().h3q_int8_linear_ex(_p(x), _kind(x.dtype), _p(w), _p(scale), scale.numel(), _p(bias), _p(out),
                                   _kind(out_dtype), M, N, K, int(swiglu), int(rotate), _p(workspace),
                                   workspace.numel(), _stream(x.device)))
    return out


def int8_linear(x, w, scale, bias=None, out_dtype=None):
    """kernels::int8_linear (kernels.rs:1074-1076)."""
    return int8_linear_ex(x, w, scale, bias, out_dtype, False, False)


def gemm_s8_quantized(a, xs, w, ws, bias=None, epilogue: int = EPI_LINEAR, out_dtype=None, gate=None,
                      gate_idx=None, resid=None, out=None):
    """The tcgen05 GEMM on pre-quantized rows with a chosen epilogue (include/h3q.h)."""
    import torch
    ws = ws.to(torch.float32).reshape(-1).contiguous()
    _cuda(a, xs, w, ws, bias, gate, gate_idx, resid)
    M, K = a.shape
    N = w.shape[0]
    if epilogue == EPI_ACC_I32:
        dt, n_out = torch.int32, N
    elif epilogue in (EPI_SWIGLU_PAIRS, EPI_SWIGLU_HALVES):
        dt, n_out = (torch.bfloat16 if epilogue == EPI_SWIGLU_PAIRS else (out_dtype or torch.bfloat16)), N // 2
    elif epilogue == EPI_LINEAR:
        dt, n_out = out_dtype or torch.bfloat16, N
    else:
        dt, n_out = torch.bfloat16, N
    if out is None:
        out = torch.empty((M, n_out), dtype=dt, device=a.device)
    okind = _kind(dt) if dt != torch.int32 else 0
    check(lib().h3q_gemm_s8_quantized(_p(a), _p(xs), _p(w), _p(ws), ws.numel(), _p(bias), _p(out), okind, M, N, K,
                                      epilogue, _p(gate), _p(gate_idx), _p(resid), _stream(a.device)))
    return out


def gemm_s8_acc(a, w):
    """Raw int32 accumulators of a [M,K] x w [N,K]^T."""
    import torch
    _cuda(a, w)
    M, K = a.shape
    N = w.shape[0]
    acc = torch.empty((M, N), dtype=torch.int32, device=a.device)
    check(lib().h3q_gemm_s8_acc(_p(a), _p(w), _p(acc), M, N, K, _stream(a.device)))
    return acc


def dequant_i8(q, scale, out_dtype):
    """kernels::dequant_i8 (kernels.rs:636-638)."""
    import torch
    scale = scale.to(torch.float32).reshape(-1).contiguous()
    _cuda(q, scale)
    rows, cols = q.shape
    out = torch.empty((rows, cols), dtype=out_dtype, device=q.device)
    check(lib().h3q_dequant_i8(_p(q), _p(scale), scale.numel(), _p(out), _kind(out_dtype), rows, cols,
                               _stream(q.device)))
    return out


def dequant_nvfp4(q, block_scale, global_scale, out_dtype):
    """kernels::dequant_nvfp4 (kernels.rs:677-680)."""
    import torch
    g = global_scale.to(torch.float32).reshape(1).contiguous()
    _cuda(q, block_scale, g)
    rows, kp = q.shape
    out = torch.empty((rows, 2 * kp), dtype=out_dtype, device=q.device)
    check(lib().h3q_dequant_nvfp4(_p(q), _p(block_scale), _p(g), _p(out), _kind(out_dtype), rows, 2 * kp,
                                  _stream(q.device)))
    return out


def nvfp4_linear(x, q, block_scale, global_scale, pre_quant_scale=None, bias=None):
    """QLinear::apply for an NVFP4 layer (weights.rs:612-635), fused: bf16 x [M,K] -> bf16 [M,N]."""
    import torch
    g = global_scale.to(torch.float32).reshape(1).contiguous()
    pqs = None if pre_quant_scale is None else pre_quant_scale.to(torch.bfloat16).contiguous()
    bias = None if bias is None else bias.to(torch.float32).contiguous()
    _cuda(x, q, block_scale, g, pqs, bias)
    M, K = x.shape
    N = q.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    need = lib().h3q_nvfp4_linear_workspace_size(M, N, K, int(pqs is not None))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    check(lib().h3q_nvfp4_linear(_p(x), _p(pqs), _p(q), _p(block_scale), _p(g), _p(bias), _p(out), M, N, K, _p(ws),
                                 ws.numel(), _stream(x.device)))
    return out


def gate_add(x, y, gate, idx):
    """kernels::gate_add (kernels.rs:879-883)."""
    import torch
    y = y.to(x.dtype).contiguous()
    _cuda(x, y, gate, idx)
    S, C = x.shape
    out = torch.empty_like(x)
    check(lib().h3q_gate_add(_p(x), _p(y), _kind(x.dtype), _p(gate), _p(idx), _p(out), S, C, _stream(x.device)))
    return out


def rms_modulate(x, w, eps: float, scale, shift, idx):
    """kernels::rms_modulate (kernels.rs:1201-1204) for bf16 x [S, C]: bf16 [S, C]."""
    import torch
    w = w.to(torch.bfloat16).contiguous()
    _cuda(x, w, scale, shift, idx)
    S, C = x.shape
    out = torch.empty_like(x)
    check(lib().h3q_rms_modulate(_p(x), _p(w), eps, _p(scale), _p(shift), _p(idx), _p(out), S, C, _stream(x.device)))
    return out


def rms_modulate_quant(x, w, eps: float, scale, shift, idx):
    """rms_modulate fused with the rotated per-row int8 quantizer: (codes int8 [S, C], row scales f32 [S])."""
    import torch
    w = w.to(torch.bfloat16).contiguous()
    _cuda(x, w, scale, shift, idx)
    S, C = x.shape
    q = torch.empty((S, C), dtype=torch.int8, device=x.device)
    xs = torch.empty(S, dtype=torch.float32, device=x.device)
    check(lib().h3q_rms_modulate_quant(_p(x), _p(w), eps, _p(scale), _p(shift), _p(idx), _p(q), _p(xs), S, C,
                                       _stream(x.device)))
    return q, xs


def attention_available(q) -> bool:
    """attn8::available (attn8.rs:592-602): head_dim 128, bf16, an sm_100 device."""
    import torch
    if not q.is_cuda:
        return False
    return bool(lib().h3q_attention_available(q.shape[-1], _kind(q.dtype) if q.dtype in (
        torch.float32, torch.float16, torch.bfloat16) else -1, q.device.index or 0))


def attention(q, k, v, flags: int = 0):
    """attn8::attention (attn8.rs:611-615): q, k, v bf16 [S, H, 128] -> bf16 [S, H, 128]."""
    import torch
    _cuda(q, k, v)
    S, H, _ = q.shape
    out = torch.empty_like(q)
    need = lib().h3q_attention_workspace_size(S, H, flags)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    check(lib().h3q_attention(_p(q), _p(k), _p(v), _p(out), S, H, flags, _p(ws), ws.numel(), _stream(q.device)))
    return out


def attention_qkv(q, k, qkv, v_col: int, flags: int = 0):
    """attn8::attention_qkv (attn8.rs:604-609): V read from the fused qkv [S, W] at column v_col."""
    import torch
    _cuda(q, k, qkv)
    S, H, _ = q.shape
    out = torch.empty_like(q)
    need = lib().h3q_attention_workspace_size(S, H, flags)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    check(lib().h3q_attention_qkv(_p(q), _p(k), _p(qkv), qkv.shape[1], v_col, _p(out), S, H, flags, _p(ws),
                                  ws.numel(), _stream(q.device)))
    return out


def qk_norm_rope(x, col_off: int, heads: int, head_dim: int, norm=None, table=None, rot: int = 0,
                 head_stride: int | None = None):
    """kernels::qk_norm_rope(_strided) (kernels.rs:745-800) for bf16 x [S, width]: norm = (weight or None, eps) or
    None; table = f32 [2, S, rot/2] cos / sin or None.  Returns bf16 [S, heads, head_dim]."""
    import torch
    S, width = x.shape
    do_norm, w, eps = (0, None, 0.0) if norm is None else (1, norm[0], float(norm[1]))
    if w is not None:
        w = w.to(torch.bfloat16).contiguous()
    if table is not None:
        table = table.to(torch.float32).contiguous()
    _cuda(x, w, table)
    out = torch.empty((S, heads, head_dim), dtype=torch.bfloat16, device=x.device)
    check(lib().h3q_qk_norm_rope(_p(x), width, col_off, head_dim if head_stride is None else head_stride, _p(w),
                                 do_norm, eps, _p(table), rot if table is not None else 0, _p(out), S, heads,
                                 head_dim, _stream(x.device)))
    return out


def attend_qkv(qkv, heads: int, norms=None, eps: float = 1e-6, rope=None, rot: int = 0, flags: int = 0):
    """The DiT's attention step (dit.rs:741-757) on a fused qkv [S, 3 * heads * 128]: q/k RMSNorm (norms = (q weight,
    k weight) or None) and RoPE (rope = f32 [2, S, rot/2] or None) fused into the int8 attention's front end.
    Returns bf16 [S, heads * 128]."""
    import torch
    S, width = qkv.shape
    inner = heads * 128
    qw, kw = (None, None) if norms is None else (norms[0].to(torch.bfloat16).contiguous(),
                                                 norms[1].to(torch.bfloat16).contiguous())
    if rope is not None:
        rope = rope.to(torch.float32).contiguous()
    _cuda(qkv, qw, kw, rope)
    out = torch.empty((S, inner), dtype=torch.bfloat16, device=qkv.device)
    need = lib().h3q_attention_workspace_size(S, heads, flags)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=qkv.device)
    check(lib().h3q_attend_qkv(_p(qkv), width, 0, inner, 2 * inner, _p(qw), _p(kw), int(norms is not None), eps,
                               _p(rope), rot if rope is not None else 0, _p(out), S, heads, flags, _p(ws), ws.numel(),
                               _stream(qkv.device)))
    return out


def attention_rows(q, k, v_src, v_row_stride: int, v_col: int, flags: int = 0):
    """Attention of the query rows q [Sq, H, 128] against all keys k [S, H, 128] (V from rows of v_src [S, W] at
    column v_col): the rows of attention() on the whole sequence that q covers."""
    import torch
    _cuda(q, k, v_src)
    Sq, H, _ = q.shape
    S = k.shape[0]
    out = torch.empty_like(q)
    need = lib().h3q_attention_rows_workspace_size(Sq, S, H, flags)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    check(lib().h3q_attention_rows(_p(q), Sq, _p(k), _p(v_src), v_row_stride, v_col, _p(out), S, H, flags, _p(ws),
                                   ws.numel(), _stream(q.device)))
    return out


def attn_kmean(k):
    """ColMean / S (attn8.rs:429-455, :622) in a fixed summation order: f32 [H, 128]."""
    import torch
    _cuda(k)
    S, H, _ = k.shape
    out = torch.empty((H, 128), dtype=torch.float32, device=k.device)
    need = lib().h3q_attn_kmean_workspace_size(S, H)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=k.device)
    check(lib().h3q_attn_kmean(_p(k), S, H, _p(out), _p(ws), ws.numel(), _stream(k.device)))
    return out


def attn_quant_heads(x, mean=None, flags: int = 0):
    """QuantHeads (attn8.rs:395-427): codes int8 [H, S, 128], scales f32 [H, roundup(S, 128)]."""
    import torch
    _cuda(x, mean)
    S, H, _ = x.shape
    Sp = (S + 127) // 128 * 128
    codes = torch.empty((H, S, 128), dtype=torch.int8, device=x.device)
    scales = torch.empty((H, Sp), dtype=torch.float32, device=x.device)
    check(lib().h3q_attn_quant_heads(_p(x), _p(mean), _p(codes), _p(scales), S, H, flags, _stream(x.device)))
    return codes, scales


def attn_v_layout(src, row_stride: int, col_off: int, S: int, H: int, flags: int = 0):
    """VToF16 (attn8.rs:457-486), transposed: V^T [H, 128, roundup(S, 128)] in f16 (or bf16)."""
    import torch
    _cuda(src)
    Sp = (S + 127) // 128 * 128
    dt = torch.bfloat16 if flags & ATTN_PV_BF16 else torch.float16
    vt = torch.empty((H, 128, Sp), dtype=dt, device=src.device)
    check(lib().h3q_attn_v_layout(_p(src), row_stride, col_off, _p(vt), S, H, flags, _stream(src.device)))
    return vt


def attention_core(q8, qs, k8, ks, vt, flags: int = 0, scores: bool = False):
    """Attn (attn8.rs:488-520) on prepared stages -> bf16 [S, H, 128] (and the int32 Q.K^T [H, S, S] if scores)."""
    import torch
    _cuda(q8, qs, k8, ks, vt)
    H, S, _ = q8.shape
    out = torch.empty((S, H, 128), dtype=torch.bfloat16, device=q8.device)
    sc = torch.empty((H, S, S), dtype=torch.int32, device=q8.device) if scores else None
    check(lib().h3q_attention_core(_p(q8), _p(qs), _p(k8), _p(ks), _p(vt), _p(out), S, H, flags, _p(sc),
                                   _stream(q8.device)))
    return (out, sc) if scores else out


class HostPipeline:
    """gemm_s8 on pinned host activations with the copies in, the GEMMs and the copies out overlapped
    (h3q_host_pipeline_*)."""

    def __init__(self, chunk_rows: int, max_k: int, max_n: int, device=None, in_slots: int = 2, out_slots: int = 2):
        import torch
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib().h3q_host_pipeline_create_ex(chunk_rows, max_k, max_n, in_slots, out_slots, ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if self._h:
            lib().h3q_host_pipeline_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def gemm_s8(self, x_host, w, ws, bias=None, swiglu: bool = False, rotate: bool = False, out=None):
        """x_host bf16 [M, K] (pinned host) -> bf16 [M, N] (or [M, N/2]) in pinned host memory; stream-ordered on
        the current stream (synchronize before reading the result)."""
        import torch
        ws = ws.to(torch.float32).contiguous()
        m, k = x_host.shape
        n = w.shape[0]
        if out is None:
            out = torch.empty((m, n // 2 if swiglu else n), dtype=torch.bfloat16, pin_memory=True)
        check(lib().h3q_host_pipeline_gemm_s8(self._h, _p(x_host), _p(w), _p(ws), ws.numel(), _p(bias), _p(out), m, n,
                                              k, int(swiglu), int(rotate), _stream(self.device)))
        return out

    def run(self, linears):
        """Several linears as one pipelined sequence (h3q_host_pipeline_run): each item is
        (x_host, w, ws, bias, out_host, swiglu, rotate) with pinned host x_host / out_host; an item may read an
        earlier item's out_host.  Stream-ordered on the current stream, like gemm_s8."""
        import torch
        items = (HostLinear * max(len(linears), 1))()
        keep = []
        for i, (x_host, w, ws, bias, out_host, swiglu, rotate) in enumerate(linears):
            ws = ws.to(torch.float32).contiguous()
            keep.append(ws)
            m, k = x_host.shape
            items[i] = HostLinear(_p(x_host), _p(w), _p(ws), ws.numel(), _p(bias), _p(out_host), m, w.shape[0], k,
                                  int(swiglu), int(rotate))
        check(lib().h3q_host_pipeline_run(self._h, items, len(linears), _stream(self.device)))
        del keep


def _lora_descs(loras, n: int, k: int, device):
    """(a [r, k], b [n, r], scale) device tensors -> an h3q_lora array (and the tensors it points into)."""
    import torch
    descs = (LoraDesc * max(len(loras), 1))()
    keep = []
    for i, (a, b, scale) in enumerate(loras):
        a, b = a.contiguous(), b.contiguous()
        if a.dim() != 2 or b.dim() != 2 or a.shape[1] != k or b.shape[0] != n or b.shape[1] != a.shape[0]:
            raise ValueError(f"LoRA {i}: a {tuple(a.shape)} and b {tuple(b.shape)} do not fit a [{n}, {k}] weight")
        if a.dtype != b.dtype or a.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError(f"LoRA {i}: factors must share one of f32 / f16 / bf16")
        if a.device != torch.device(device) or b.device != torch.device(device):
            raise ValueError(f"LoRA {i}: factors must be on {device}")
        keep += [a, b]
        descs[i] = LoraDesc(a.data_ptr(), b.data_ptr(), a.shape[0], _kind(a.dtype), float(scale))
    return descs, keep


def lora_merge_i8(w, scale, loras, convrot: int = 256, out=None, out_scale=None):
    """QLinear::merge_loras for an int8 layer (weights.rs:716-757): returns (w' int8 [n, k], s' f32 [n]).  loras is
    a sequence of (a [r, k], b [n, r], scale) with scale = alpha / rank * strength.  With no LoRA the inputs come
    back unchanged (the reference's early return)."""
    import torch
    _cuda(w, scale)
    n, k = w.shape
    if not loras:
        return w, scale
    descs, keep = _lora_descs(loras, n, k, w.device)
    scale = scale.to(torch.float32).reshape(-1).contiguous()
    out = torch.empty_like(w) if out is None else out
    out_scale = torch.empty(n, dtype=torch.float32, device=w.device) if out_scale is None else out_scale
    ws = torch.empty(max(lib().h3q_lora_merge_i8_workspace_size(n, k), 1), dtype=torch.uint8, device=w.device)
    check(lib().h3q_lora_merge_i8(_p(w), _p(scale), scale.numel(), convrot, descs, len(loras), _p(out),
                                  _p(out_scale), n, k, _p(ws), ws.numel(), _stream(w.device)))
    del keep
    return out, out_scale


def lora_merge_dense(w, loras, out=None):
    """QLinear::merge_loras for a dense layer (weights.rs:710-715): dtype(f32(w) + sum of the deltas)."""
    import torch
    _cuda(w)
    n, k = w.shape
    if not loras:
        return w
    descs, keep = _lora_descs(loras, n, k, w.device)
    out = torch.empty_like(w) if out is None else out
    check(lib().h3q_lora_merge_dense(_p(w), _kind(w.dtype), descs, len(loras), _p(out), n, k, _stream(w.device)))
    del keep
    return out


def default_switches() -> Switches:
    return lib().h3q_default_switches()


class QLinear:
    """weights.rs QLinear for an int8 layer: forward_raw / run and run_swiglu through h3q_qlinear_forward."""

    def __init__(self, weight, scale, bias=None, convrot: int = 256, interleaved: bool = False, n_loras: int = 0,
                 fmt: int = FMT_INT8):
        import torch
        self.weight = weight
        self.scale = scale.to(torch.float32).reshape(-1).contiguous()
        self.bias = None if bias is None else bias.to(torch.float32).contiguous()
        self.desc = QLinearDesc(fmt, convrot, int(interleaved), n_loras, weight.shape[0], weight.shape[1],
                                weight.data_ptr(), self.scale.data_ptr(), self.scale.numel(),
                                None if self.bias is None else self.bias.data_ptr())

    def plan(self, x_kind: int, swiglu: bool = False, switches: Switches | None = None) -> int:
        sw = switches or default_switches()
        return lib().h3q_qlinear_plan(ctypes.byref(self.desc), x_kind, self.desc.in_features, int(swiglu),
                                      ctypes.byref(sw))

    def forward(self, x, swiglu: bool = False, switches: Switches | None = None):
        import torch
        sw = switches or default_switches()
        _cuda(x)
        rows = x.shape[0]
        kind = _kind(x.dtype)
        n = self.desc.out_features // 2 if swiglu else self.desc.out_features
        out = torch.empty((rows, n), dtype=x.dtype, device=x.device)
        need = lib().h3q_qlinear_workspace_size(ctypes.byref(self.desc), kind, rows, int(swiglu), ctypes.byref(sw))
        ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        check(lib().h3q_qlinear_forward(ctypes.byref(self.desc), _p(x), kind, rows, int(swiglu), _p(out), _p(ws),
                                        ws.numel(), ctypes.byref(sw), _stream(x.device)))
        return out

    run = forward

    def run_swiglu(self, x, switches: Switches | None = None):
        return self.forward(x, swiglu=True, switches=switches)

    def merge_loras(self, loras) -> None:
        """QLinear::merge_loras (weights.rs:692-761): fold (a, b, scale) deltas into the int8 weight and per-row
        scales.  Interleaved (SwiGLU-paired) layers are left alone, as in the reference: merge before
        interleaving."""
        if not loras or self.desc.interleaved:
            return
        self.weight, self.scale = lora_merge_i8(self.weight, self.scale, loras, convrot=self.desc.convrot)
        self.desc.weight = self.weight.data_ptr()
        self.desc.scale = self.scale.data_ptr()
        self.desc.scale_numel = self.scale.numel()
