"""CPU checks of the attention oracle (attn8.rs restated in oracle/h3q_oracle.c) and of the attention C ABI's
host-side argument checks.  No GPU calls."""
import numpy as np
import pytest

import h3q
from oracle import oracle as O


def test_kmean_is_the_column_mean():
    q, k, v = O.make_attn_inputs(3, 333, 2, 3.0)
    km = O.attn_kmean(k)
    exact = O.bf16_bits_to_f32(k).astype(np.float64).mean(axis=0)
    np.testing.assert_allclose(km, exact, rtol=1e-5, atol=1e-6)


def test_kmean_chunk_order():
    """S = 300 -> chunks of ceil(300 / 128) = 3 rows, 100 of them; the sum order is chunk by chunk."""
    S, H = 300, 1
    k = O.f32_to_bf16_bits(np.random.default_rng(0).standard_normal((S, H, 128)).astype(np.float32))
    x = O.bf16_bits_to_f32(k).reshape(S, 128)
    want = np.zeros(128, dtype=np.float32)
    for r0 in range(0, S, 3):
        s = np.zeros(128, dtype=np.float32)
        for r in range(r0, min(S, r0 + 3)):
            s = (s + x[r]).astype(np.float32)
        want = (want + s).astype(np.float32)
    want = (want * np.float32(1.0 / S)).astype(np.float32)
    np.testing.assert_array_equal(O.attn_kmean(k).reshape(-1), want)


def test_quant_heads_formula():
    """sc = max(max|v| / 127, 1e-20); q = clamp(rint(v / sc), -127, 127) per (token, head) row."""
    q, k, v = O.make_attn_inputs(4, 70, 3)
    codes, scales = O.attn_quant_heads(q)
    x = O.bf16_bits_to_f32(q)
    for s in (0, 17, 69):
        for h in range(3):
            m = np.max(np.abs(x[s, h]))
            sc = np.float32(max(np.float32(m) / np.float32(127.0), np.float32(1e-20)))
            assert scales[h, s] == sc
            inv = np.float32(1.0) / sc
            want = np.clip(np.rint((x[s, h] * inv).astype(np.float32)), -127, 127).astype(np.int8)
            np.testing.assert_array_equal(codes[h, s], want)
    assert np.all(scales[:, 70:] == 0)
    assert codes.min() >= -127


def test_quant_heads_block_mode_shares_one_scale():
    q, k, v = O.make_attn_inputs(5, 300, 2)
    codes, scales = O.attn_quant_heads(q, None, True)
    for h in range(2):
        for b0 in (0, 128, 256):
            blk = scales[h, b0:min(300, b0 + 128)]
            assert np.all(blk == blk[0])
            m = np.max(np.abs(O.bf16_bits_to_f32(q)[b0:b0 + 128, h]))
            assert blk[0] == np.float32(max(np.float32(m) / np.float32(127.0), np.float32(1e-20)))


def test_scores_are_integer_dot_products():
    q, k, v = O.make_attn_inputs(6, 50, 2)
    q8, _ = O.attn_quant_heads(q)
    k8, _ = O.attn_quant_heads(k)
    sc = O.attn_scores(q8, k8)
    want = np.einsum("hsd,htd->hst", q8.astype(np.int64), k8.astype(np.int64))
    np.testing.assert_array_equal(sc, want)


def test_scale_log2():
    want = np.float32(np.float32(1.0) / np.sqrt(np.float32(128.0))) * np.float32(np.log2(np.e))
    assert O.attn_scale_log2() == np.float32(want)


@pytest.mark.parametrize("flags", [0, 1, 2, 3])
def test_oracle_attention_tracks_exact_softmax(flags):
    """The int8 attention approximates float softmax attention: SageAttention's quantisation error only."""
    q, k, v = O.make_attn_inputs(7, 256, 2, 3.0)
    y = O.bf16_bits_to_f32(O.attention(q, k, v, flags))
    ex = O.attention_exact(q, k, v)
    assert O.max_abs_rel(y, ex) < 3e-2
    assert np.abs(y - ex).mean() / np.abs(ex).mean() < 2e-2


def test_oracle_attention_smoothing_matters():
    """Without the K mean the per-token K scale covers the channel offsets and the error grows."""
    q, k, v = O.make_attn_inputs(8, 256, 1, 8.0)
    q8, qs = O.attn_quant_heads(q)
    k8n, ksn = O.attn_quant_heads(k, None)
    y_plain = O.bf16_bits_to_f32(O.attn_forward(q8, qs, k8n, ksn, v.reshape(256, 128), 128, 0))
    y_smooth = O.bf16_bits_to_f32(O.attention(q, k, v))
    ex = O.attention_exact(q, k, v)
    assert O.max_abs_rel(y_smooth, ex) < O.max_abs_rel(y_plain, ex)


def test_attention_cabi_argument_checks():
    L = h3q.lib()
    assert L.h3q_attention_workspace_size(0, 4, 0) == 0
    assert L.h3q_attention_workspace_size(32760, 40, 0) > 32760 * 40 * 128 * 4
    # S == 0: nothing to do
    assert L.h3q_attention(None, None, None, None, 0, 4, 0, None, 0, None) == h3q.OK
    assert L.h3q_attention(None, None, None, None, 16, 4, 8, None, 0, None) == h3q.ERR_ARG
    assert L.h3q_attention(None, None, None, None, 16, 4, 0, None, 0, None) == h3q.ERR_ARG
    assert L.h3q_attention_qkv(None, None, None, 100, 0, None, 16, 1, 0, None, 0, None) == h3q.ERR_ARG
    assert "outside a qkv row" in h3q.last_error()
    assert L.h3q_attn_v_layout(None, 64, 0, None, 16, 1, 0, None) == h3q.ERR_ARG
    assert L.h3q_attention_core(None, None, None, None, None, None, -1, 1, 0, None, None) == h3q.ERR_ARG
    assert L.h3q_attention_available(64, 2, 0) == 0
    assert L.h3q_attention_available(128, 1, 0) == 0


def test_rms_modulate_oracle_formula():
    """The oracle's rms_modulate against the formula in f64 (one bf16 unit of rounding slack)."""
    x, w, sc, sh, idx = O.make_modulate_inputs(1, 40, 1024)
    got = O.bf16_bits_to_f32(O.rms_modulate(x, w, 1e-6, sc, sh, idx)).astype(np.float64)
    xf = O.bf16_bits_to_f32(x).astype(np.float64)
    inv = 1.0 / np.sqrt((xf ** 2).mean(axis=1, keepdims=True) + 1e-6)
    n = O.bf16_round((xf * inv * O.bf16_bits_to_f32(w)[None, :]).astype(np.float32)).astype(np.float64)
    want = n * (1.0 + O.bf16_round(sc[idx]).astype(np.float64)) + O.bf16_round(sh[idx]).astype(np.float64)
    assert np.max(np.abs(got - want) / (np.abs(want) + 1e-3)) < 2e-2
