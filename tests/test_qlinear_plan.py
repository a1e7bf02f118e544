"""CPU tests of the QLinear dispatch mirror (weights.rs:833-947): the path h3q_qlinear_plan picks for each layer,
activation and switch setting, case by case against the reference's branches.  Host logic only."""
import ctypes

import pytest

import h3q

BF16, F16, F32 = 2, 1, 0
G, I, RF, RS, SF, SA = (h3q.PATH_GEMM_S8, h3q.PATH_INT8_LINEAR, h3q.PATH_ROTATE_FUSED, h3q.PATH_ROTATE_SEPARATE,
                        h3q.PATH_SWIGLU_FUSED, h3q.PATH_SWIGLU_AFTER)


def layer(k=5120, n=15360, convrot=256, interleaved=False, n_loras=0, fmt=h3q.FMT_INT8):
    return h3q.QLinearDesc(fmt, convrot, int(interleaved), n_loras, n, k, None, None, n, None)


def sw(**kw):
    s = h3q.default_switches()
    for k, v in kw.items():
        setattr(s, k, v)
    return s


def plan(l, kind=BF16, swiglu=False, s=None):
    return h3q.lib().h3q_qlinear_plan(ctypes.byref(l), kind, l.in_features, int(swiglu), ctypes.byref(s or sw()))


def test_default_switches_are_the_reference_defaults():
    s = h3q.default_switches()
    assert (s.int8, s.gemm_fused, s.rot_fused, s.fused_rot_linear) == (1, 1, 1, 0)


def test_dit_linears_take_the_fused_gemm_with_fused_rotation():
    """try_gemm_s8 (weights.rs:889-909): bf16, K % 64, N % 128, convrot 256 with K/256 <= 56."""
    assert plan(layer(5120, 15360)) == G | RF
    assert plan(layer(13824, 5120)) == G | RF           # 54 groups
    assert plan(layer(14336, 5120)) == G | RF           # 56 groups: the rot2 limit
    assert plan(layer(14592, 5120)) == G | RS           # 57 groups: rotate_activation first (weights.rs:899-903)


def test_switches_redirect_like_the_environment():
    assert plan(layer(), s=sw(rot_fused=0)) == G | RS                  # H3_ROT=gemm
    assert plan(layer(), s=sw(gemm_fused=0)) == I | RS                 # H3_GEMM=cublaslt, H3_FUSED_ROT unset
    assert plan(layer(), s=sw(gemm_fused=0, fused_rot_linear=1)) == I | RF
    assert plan(layer(), s=sw(int8=0)) == -h3q.ERR_UNSUPPORTED         # H3_INT8=0: dequantise-then-matmul


def test_gemm_gates_fall_back_to_int8_linear():
    assert plan(layer(5120, 1000)) == I | RS       # out_features % 128 != 0
    assert plan(layer(), kind=F16) == I | RS       # non-bf16 activations
    assert plan(layer(5120, 1024, convrot=0)) == G  # no ConvRot: no rotation at all
    assert plan(layer(5120, 1000, convrot=0)) == I


def test_run_swiglu_paths():
    """run_swiglu (weights.rs:860-886)."""
    assert plan(layer(5120, 27648, interleaved=True), swiglu=True) == G | RF | SF
    assert plan(layer(5120, 27648, interleaved=False), swiglu=True) == I | RS | SF
    assert plan(layer(5120, 27648, interleaved=False), swiglu=True, s=sw(fused_rot_linear=1)) == I | RF | SF
    assert plan(layer(5120, 27648, interleaved=True), swiglu=True, s=sw(gemm_fused=0)) == I | RS | SA


def test_layers_outside_the_int8_fast_path_are_refused():
    assert plan(layer(n_loras=1)) == -h3q.ERR_UNSUPPORTED
    assert plan(layer(fmt=h3q.FMT_DENSE)) == -h3q.ERR_UNSUPPORTED
    assert plan(layer(fmt=h3q.FMT_NVFP4)) == -h3q.ERR_UNSUPPORTED
    assert plan(layer(), kind=7) == -h3q.ERR_ARG


def test_workspace_grows_with_separate_passes():
    L = h3q.lib()
    l = layer(5120, 1024)
    base = L.h3q_qlinear_workspace_size(ctypes.byref(l), BF16, 64, 0, ctypes.byref(sw()))
    sep = L.h3q_qlinear_workspace_size(ctypes.byref(l), BF16, 64, 0, ctypes.byref(sw(rot_fused=0)))
    assert base == L.h3q_gemm_s8_workspace_size(64, 5120)
    assert sep == base + 64 * 5120 * 2
