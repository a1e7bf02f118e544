"""GPU parity of the QLinear dispatch: each path h3q_qlinear_forward can take, against the oracle composed the
same way the reference composes it."""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from tests.gpu_util import bf16_bits, bf16_tensor, t

pytestmark = pytest.mark.gpu


def _layer(seed, M, K, N, cuda, interleaved=False, convrot=256):
    x, w, ws, bias = O.make_linear_inputs(seed, M, K, N)
    ql = h3q.QLinear(t(w, cuda), t(ws, cuda), t(bias, cuda), convrot=convrot, interleaved=interleaved)
    return (x, w, ws, bias), ql


def _sw(**kw):
    s = h3q.default_switches()
    for k, v in kw.items():
        setattr(s, k, v)
    return s


def test_fused_path_equals_gemm_s8(cuda):
    (x, w, ws, bias), ql = _layer(1, 200, 5120, 1024, cuda)
    assert ql.plan(2) == h3q.PATH_GEMM_S8 | h3q.PATH_ROTATE_FUSED
    out = bf16_bits(ql.run(bf16_tensor(x, cuda)))
    want, _, _, _ = O.gemm_s8(x, w, ws, bias, swiglu=False, rotate=True)
    assert np.array_equal(out, want)


def test_separate_rotation_path(cuda):
    """H3_ROT=gemm: rotate_activation to bf16, then gemm_s8 without rotation (weights.rs:899-905)."""
    (x, w, ws, bias), ql = _layer(2, 130, 1024, 512, cuda)
    s = _sw(rot_fused=0)
    assert ql.plan(2, switches=s) == h3q.PATH_GEMM_S8 | h3q.PATH_ROTATE_SEPARATE
    out = bf16_bits(ql.run(bf16_tensor(x, cuda), switches=s))
    xr = O.rotate_bf16(x)
    want, _, _, _ = O.gemm_s8(xr, w, ws, bias, swiglu=False, rotate=False)
    assert np.array_equal(out, want)


def test_int8_linear_path_with_separate_rotation(cuda):
    """H3_GEMM=cublaslt: rotate_activation, then int8_linear_ex unrotated (weights.rs:925-935)."""
    (x, w, ws, bias), ql = _layer(3, 77, 1024, 512, cuda)
    s = _sw(gemm_fused=0)
    out = bf16_bits(ql.run(bf16_tensor(x, cuda), switches=s))
    xr = O.rotate_bf16(x)
    q, xs = O.quant_rows(xr, 2, O.QUANT_PLAIN)
    want = O.int8_epilogue(O.gemm_s8_acc(q, w), xs, ws, bias, 2, False)
    assert np.array_equal(out, want)


def test_swiglu_paths(cuda):
    M, K, N = 96, 1024, 768
    (x, w, ws, bias), ql = _layer(4, M, K, N, cuda, interleaved=True)
    xd = bf16_tensor(x, cuda)
    fused = O.bf16_bits_to_f32(bf16_bits(ql.run_swiglu(xd)))
    after = O.bf16_bits_to_f32(bf16_bits(ql.run_swiglu(xd, switches=_sw(gemm_fused=0))))
    want_f, _, _, _ = O.gemm_s8(x, w, ws, bias, swiglu=True, rotate=True)
    xr = O.rotate_bf16(x)
    q, xs = O.quant_rows(xr, 2, O.QUANT_PLAIN)
    lin = O.int8_epilogue(O.gemm_s8_acc(q, w), xs, ws, bias, 2, False)
    want_a = O.swiglu_bf16(lin, interleaved=True)
    assert O.max_abs_rel(fused, O.bf16_bits_to_f32(want_f)) < 1e-2
    assert O.max_abs_rel(after, O.bf16_bits_to_f32(want_a)) < 1e-2
    # non-interleaved layer: split-half SwiGLU inside int8_linear_ex (weights.rs:868-883)
    (x2, w2, ws2, b2), ql2 = _layer(5, M, K, N, cuda, interleaved=False)
    out2 = O.bf16_bits_to_f32(bf16_bits(ql2.run_swiglu(bf16_tensor(x2, cuda))))
    xr2 = O.rotate_bf16(x2)
    q2, xs2 = O.quant_rows(xr2, 2, O.QUANT_PLAIN)
    want2 = O.int8_epilogue(O.gemm_s8_acc(q2, w2), xs2, ws2, b2, 2, True)
    assert O.max_abs_rel(out2, O.bf16_bits_to_f32(want2)) < 1e-2


def test_rotation_kernel_matches_exact_rotation(cuda):
    x, _, _, _ = O.make_linear_inputs(6, 33, 5120, 1)
    (_, w, ws, bias), ql = _layer(6, 33, 5120, 256, cuda)
    s = _sw(rot_fused=0)
    # the separate-rotation path must equal the oracle's bf16 rotation exactly (same butterfly order)
    out = bf16_bits(ql.run(bf16_tensor(x, cuda), switches=s))
    want, _, _, _ = O.gemm_s8(O.rotate_bf16(x), w, ws, bias, swiglu=False, rotate=False)
    assert np.array_equal(out, want)
    exact = O.rotate_f64(O.bf16_bits_to_f32(x))
    assert O.max_abs_rel(O.bf16_bits_to_f32(O.rotate_bf16(x)), exact) < 1e-2


def test_unsupported_layers_raise(cuda):
    (x, _, _, _), ql = _layer(7, 8, 1024, 256, cuda)
    ql.desc.n_loras = 1
    with pytest.raises(h3q.H3QError) as e:
        ql.run(bf16_tensor(x, cuda))
    assert e.value.status == h3q.ERR_UNSUPPORTED
