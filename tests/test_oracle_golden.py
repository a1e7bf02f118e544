"""CPU tests: pin the oracle (oracle/h3q_oracle.c) against the reference's known-answer tests, against
torch's generator, and against exact arithmetic.  No GPU."""
import math
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_nvfp4_kat_high_nibble_and_swizzled_block_scales():
    """portable/kernels.rs:334-355: q = 0x12 everywhere, e4m3 scale 1 (0x38) for rows < 32 and 2 (0x40) otherwise,
    global 3 -> even columns (high nibble 1 -> 0.5) and odd columns (low nibble 2 -> 1.0) times row scale times 3."""
    q = np.full((128, 32), 0x12, dtype=np.uint8)
    scales = np.zeros(512, dtype=np.uint8)
    for r in range(128):
        for block in range(4):
            scales[(r % 32) * 16 + (r // 32) * 4 + block] = 0x38 if r < 32 else 0x40
    y = O.dequant_nvfp4(q, scales, 3.0, 0)
    for r in range(128):
        for c in range(64):
            expected = (0.5 if c % 2 == 0 else 1.0) * (1.0 if r < 32 else 2.0) * 3.0
            assert y[r, c] == expected


def test_nvfp4_scale_offset_matches_reference_formula():
    """kernels.rs:76-78: off = (r/128*ncb + b/4)*512 + (r%32)*16 + (r%128/32)*4 + b%4."""
    k = 5120
    ncb = (k // 16 + 3) // 4
    rng = np.random.default_rng(0)
    for _ in range(200):
        r, b = int(rng.integers(0, 1000)), int(rng.integers(0, k // 16))
        off = (r // 128 * ncb + b // 4) * 512 + (r % 32) * 16 + (r % 128 // 32) * 4 + b % 4
        assert O.nvfp4_scale_offset(r, b, k) == off


def test_fp8e4m3_decode():
    assert O.fp8e4m3(0x38) == 1.0 and O.fp8e4m3(0x40) == 2.0 and O.fp8e4m3(0xB8) == -1.0
    assert O.fp8e4m3(0x7E) == 448.0 and math.isnan(O.fp8e4m3(0x7F)) and O.fp8e4m3(0x01) == 2.0 ** -9


def test_int8_linear_pattern_row_scales():
    """apple.rs:177-196 pattern: w[i] = (i as i8) * 3 wrapping, per-row scales {0.125, 0.25}, x[i] = sin(0.13 i);
    the dequantised linear must equal x . (q * s_row)^T within 1e-3 (pins per-row scale semantics)."""
    w = np.array([np.int8(np.int16(i) * 3 & 0xFF if (i * 3) & 0xFF < 128 else ((i * 3) & 0xFF) - 256)
                  for i in range(128)], dtype=np.int8).reshape(2, 64)
    assert w[0, 1] == 3 and w[0, 43] == np.int8(-127)
    scales = np.array([0.125, 0.25], dtype=np.float32)
    x = np.sin(np.arange(192, dtype=np.float32) * np.float32(0.13)).reshape(3, 64).astype(np.float32)
    wd = O.dequant_i8(w, scales, 0)
    got = x @ wd.T
    want = np.array([[sum(float(x[m, k]) * float(w[n, k]) * float(scales[n]) for k in range(64)) for n in range(2)]
                     for m in range(3)])
    assert np.max(np.abs(got - want)) < 1e-3
    # scalar scale: one entry applies to every row
    assert np.array_equal(O.dequant_i8(w, scales[:1], 0)[1], w[1].astype(np.float32) * np.float32(0.125))


def test_torchgen_matches_committed_torch_randn():
    """rng.rs TorchGen vs torch.randn(generator=manual_seed(seed)) values recorded by tests/golden/gen_golden.py."""
    d = np.load(os.path.join(GOLDEN, "torch_randn.npz"))
    for key in d.files:
        seed, n = (int(v) for v in key.split("_")[1:])
        got = O.TorchGen(seed).randn(n)
        assert np.allclose(got, d[key], rtol=1e-5, atol=1e-6), key


def test_torchgen_u32_stream_is_mt19937():
    """The first tempered outputs of mt19937 seeded with 5489 (the generator's published test vector)."""
    g = O.TorchGen(5489)
    assert [g.next_u32() for _ in range(3)] == [3499211612, 581869302, 3890346734]


def test_hadamard_orthonormal_and_symmetric():
    h = O.hadamard(256).astype(np.float64)
    assert np.allclose(h, h.T)
    assert np.allclose(h @ h, np.eye(256), atol=1e-6)
    assert np.all(np.abs(np.abs(h) - 1.0 / 16) < 1e-9)
    with pytest.raises(ValueError):
        O.hadamard(128)


@pytest.mark.parametrize("mode", [O.QUANT_ROT, O.QUANT_ROT2])
def test_butterflies_equal_exact_rotation(mode):
    """Both butterfly orders compute x . H256 up to fp32 rounding (weights.rs:482-489)."""
    x, _, _, _ = O.make_linear_inputs(3, 16, 1024, 16)
    xf = O.bf16_bits_to_f32(x)
    exact = O.rotate_f64(xf)
    q, s = O.quant_rows(x, 2, mode)
    # dequantised codes reproduce the rotation within half a quantization step
    assert np.all(np.abs(q.astype(np.float64) * s[:, None] - exact) <= 0.5 * s[:, None] * (1 + 1e-4) + 1e-6)
    assert np.allclose(s, np.max(np.abs(exact), axis=1) / 127, rtol=1e-5)


def test_rot_orders_agree_up_to_one_code():
    x, _, _, _ = O.make_linear_inputs(4, 64, 5120, 16)
    q1, s1 = O.quant_rows(x, 2, O.QUANT_ROT)
    q2, s2 = O.quant_rows(x, 2, O.QUANT_ROT2)
    d = np.abs(q1.astype(np.int32) - q2.astype(np.int32))
    assert d.max() <= 1
    assert np.allclose(s1, s2, rtol=1e-6)


def test_quant_edge_values():
    # all-zero row: scale floors at 1e-30, codes 0 (kernels.rs:278)
    z = np.zeros((2, 256), dtype=np.uint16)
    q, s = O.quant_rows(z, 2, O.QUANT_ROT2)
    assert np.all(q == 0) and np.all(s == np.float32(1e-30))
    # the row maximum maps to +-127
    x = np.zeros((1, 256), dtype=np.float32)
    x[0, 5] = -3.0
    x[0, 7] = 1.5
    q, s = O.quant_rows(x, 0, O.QUANT_PLAIN)
    assert q[0, 5] == -127 and q[0, 7] == 64 and s[0] == np.float32(3.0) / np.float32(127.0)
    # round half to even: 0.5 -> 0, 1.5 -> 2 (codes of v*inv exactly at .5)
    x = np.array([[127.0, 0.5, 1.5, 2.5, -0.5]], dtype=np.float32)
    q, s = O.quant_rows(x, 0, O.QUANT_PLAIN)
    assert list(q[0]) == [127, 0, 2, 2, 0]


def test_epilogue_matches_formula():
    rng = np.random.default_rng(1)
    acc = rng.integers(-2 ** 20, 2 ** 20, size=(4, 32), dtype=np.int32)
    xs = rng.random(4, dtype=np.float32) * 0.01
    ws = rng.random(32, dtype=np.float32) * 0.01
    bias = rng.standard_normal(32).astype(np.float32)
    out = O.bf16_bits_to_f32(O.gemm_s8_epilogue(acc, xs, ws, bias))
    want = (acc.astype(np.float64) * xs[:, None] * ws[None, :] + bias[None, :])
    assert O.max_abs_rel(out, want) < 1e-2
    pairs = O.bf16_bits_to_f32(O.gemm_s8_epilogue(acc, xs, ws, bias, O.EPI_SWIGLU_PAIRS))
    g, u = want[:, 0::2], want[:, 1::2]
    assert O.max_abs_rel(pairs, g / (1 + np.exp(-g)) * u) < 2e-2


def test_cpu_path_tracks_w8a8_oracle():
    """The reference's CPU path (no activation quantization) and the W8A8 path agree to quantization noise."""
    x, w, ws, bias = O.make_linear_inputs(7, 64, 1024, 256)
    ref = O.bf16_bits_to_f32(O.cpu_int8_linear(x, w, ws, bias, rotate=True))
    out, _, _, _ = O.gemm_s8(x, w, ws, bias, swiglu=False, rotate=True)
    assert O.max_abs_rel(O.bf16_bits_to_f32(out), ref) < 1e-2


def test_nvfp4_activation_quantizer_rounding():
    """The W4A4 activation quantizer's building blocks: e2m1 round-to-nearest-even with saturation at 6, the
    e4m3 value table (max 448), and a block whose values sit on the e2m1 grid coming back unchanged."""
    r = O._round_to_table(np.array([0.25, 0.75, 1.25, 2.5, 5.0, 7.0, -0.3]), O._E2M1_VALUES)
    np.testing.assert_array_equal(r, [0.0, 1.0, 1.0, 2.0, 4.0, 6.0, -0.5])
    t = O._e4m3_values()
    assert t[0] == 0.0 and t[1] == 2.0 ** -9 and t[-1] == 448.0 and np.all(np.diff(t) > 0)
    x = np.array([[6.0, -3.0, 1.5, 0.5] * 4], dtype=np.float64)
    np.testing.assert_allclose(O.nvfp4_quantize_activation(x), x, rtol=0, atol=0)


@pytest.mark.parametrize("K", [5120, 25600])
def test_nvfp4_w4a4_exceeds_the_nvfp4_contract(K):
    """Why the NVFP4 linear keeps bf16 activations (W4A16): quantizing the AWQ-scaled activations to NVFP4 as well
    (what a kind::mxf4nvf4 W4A4 GEMM needs) moves the c3 layer's output by ~9% of its largest magnitude against the
    reference's bf16-activation result (weights.rs:612-635), over four times the 2e-2 tolerance of the NVFP4 path.
    c3's K with fewer output rows (the error is per output element, set by K and the distributions)."""
    x, q, bs, g, pqs, b = O.make_nvfp4_inputs(3, 64, K, 1024)
    ref = O.bf16_bits_to_f32(O.nvfp4_linear(x, q, bs, g, pqs, b))
    w4 = O.bf16_bits_to_f32(O.nvfp4_linear_w4a4(x, q, bs, g, pqs, b))
    err = O.max_abs_rel(w4, ref)
    assert 0.05 < err < 0.2, err
