"""CPU checks of the oracle's qk_norm_rope (kernels.rs:86-126) and of the DiT attention step built on it.

Pinned on the reference's own known-answer test (portable/kernels.rs:357-380: zero angles rotate nothing) and on
the float semantics of its portable restatement (portable/kernels.rs:92-135), in float64.
"""
import numpy as np
import pytest

from oracle import oracle as O


def test_reference_known_answer_zero_angles():
    """portable_modulation_rope_and_resize_run_on_metal: x [[1, 2], [3, 4]], one head of 2 dims, no norm, a table of
    zero angles (cos 1, sin 0) over rot = 2 -> x unchanged."""
    x = O.f32_to_bf16_bits(np.array([[1.0, 2.0], [3.0, 4.0]], dtype=np.float32))
    cs = np.stack([np.cos(np.zeros((2, 1))), np.sin(np.zeros((2, 1)))]).astype(np.float32)
    y = O.qk_norm_rope(x, 0, 1, 2, None, 0.0, False, cs, 2)
    np.testing.assert_array_equal(O.bf16_bits_to_f32(y).reshape(-1), [1.0, 2.0, 3.0, 4.0])


def test_no_norm_no_table_is_identity():
    rng = np.random.default_rng(1)
    x = O.f32_to_bf16_bits(rng.standard_normal((7, 3 * 64)).astype(np.float32))
    y = O.qk_norm_rope(x, 64, 2, 64, None, 0.0, False, None, 0)
    np.testing.assert_array_equal(y.reshape(7, 128), x[:, 64:192])


def _float64_reference(x_bits, col, H, D, w_bits, eps, do_norm, cs, rot):
    """portable qk_norm_rope_strided's arithmetic in float64: y / sqrt(mean(y^2) + eps) * w, then split-half
    rotation over the first rot dims."""
    S = x_bits.shape[0]
    y = O.bf16_bits_to_f32(x_bits)[:, col:col + H * D].reshape(S, H, D).astype(np.float64)
    if do_norm:
        y = y / np.sqrt((y * y).mean(axis=2, keepdims=True) + eps)
        if w_bits is not None:
            y = y * O.bf16_bits_to_f32(w_bits).astype(np.float64)
    if cs is not None and rot:
        half = rot // 2
        a, b = y[:, :, :half].copy(), y[:, :, half:rot].copy()
        c, sn = cs[0][:, None, :].astype(np.float64), cs[1][:, None, :].astype(np.float64)
        y[:, :, :half] = a * c - b * sn
        y[:, :, half:rot] = a * sn + b * c
    return y


@pytest.mark.parametrize("D,rot,use_w", [(128, 96, True), (128, 128, False), (64, 48, True), (80, 32, True),
                                         (256, 0, True)])
def test_matches_float_semantics(D, rot, use_w):
    S, H = 40, 3
    rng = np.random.default_rng(D + rot)
    x = O.f32_to_bf16_bits((rng.standard_normal((S, 2 * H * D)) * 3).astype(np.float32))
    w = O.f32_to_bf16_bits((1 + 0.2 * rng.standard_normal(D)).astype(np.float32)) if use_w else None
    cs = None
    if rot:
        ang = rng.random((S, rot // 2)) * 50
        cs = np.stack([np.cos(ang), np.sin(ang)]).astype(np.float32)
    got = O.bf16_bits_to_f32(O.qk_norm_rope(x, H * D, H, D, w, 1e-6, True, cs, rot)).astype(np.float64)
    want = _float64_reference(x, H * D, H, D, w, 1e-6, True, cs, rot)
    # one bf16 rounding of the output (2^-9 relative) plus f32 arithmetic
    assert np.max(np.abs(got - want) / np.maximum(np.abs(want), 1e-3)) <= 2 ** -8


def test_rotation_preserves_row_norm():
    S, H, D, rot = 16, 2, 128, 128
    rng = np.random.default_rng(5)
    x = O.f32_to_bf16_bits(rng.standard_normal((S, H * D)).astype(np.float32))
    ang = rng.random((S, rot // 2)) * 50
    cs = np.stack([np.cos(ang), np.sin(ang)]).astype(np.float32)
    y = O.bf16_bits_to_f32(O.qk_norm_rope(x, 0, H, D, None, 0.0, False, cs, rot)).astype(np.float64)
    x0 = O.bf16_bits_to_f32(x).reshape(S, H, D).astype(np.float64)
    np.testing.assert_allclose(np.linalg.norm(y, axis=2), np.linalg.norm(x0, axis=2), rtol=1e-2)


def test_attend_qkv_oracle_is_the_composition():
    """O.attend_qkv is qk_norm_rope on q and k followed by attention_qkv's stages; against exact softmax attention
    on the normalised, rotated q / k it stays within the int8 approximation's error."""
    S, H, rot = 96, 2, 96
    qkv, qw, kw, cs = O.make_rope_inputs(3, S, H, 128, rot)
    out = O.attend_qkv(qkv, H, qw, kw, True, 1e-6, cs, rot)
    q = O.qk_norm_rope(qkv, 0, H, 128, qw, 1e-6, True, cs, rot)
    k = O.qk_norm_rope(qkv, H * 128, H, 128, kw, 1e-6, True, cs, rot)
    v = np.ascontiguousarray(qkv[:, 2 * H * 128:]).reshape(S, H, 128)
    ex = O.attention_exact(q, k, v)
    assert O.max_abs_rel(O.bf16_bits_to_f32(out), ex) <= 5e-2
