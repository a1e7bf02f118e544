"""GPU parity of the fused NVFP4+AWQ linear (weights.rs:612-635): the in-kernel fp4 decode is checked bit for bit
against the reference's dequant (one-hot activations make the output the weight itself); full linears are checked
at max-abs-rel 2e-2, the NVFP4 tolerance of the parity contract."""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from tests.gpu_util import bf16_bits, bf16_tensor, t

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _run(x, q, bs, g, pqs, bias, cuda):
    return h3q.nvfp4_linear(bf16_tensor(x, cuda), t(q, cuda), t(bs, cuda), torch.tensor([g], device=cuda),
                            None if pqs is None else bf16_tensor(pqs, cuda), None if bias is None else t(bias, cuda))


def test_decode_is_bit_exact_with_one_hot_rows(cuda):
    K, N = 128, 256
    _, q, bs, g, _, _ = O.make_nvfp4_inputs(1, 1, K, N)
    x = O.f32_to_bf16_bits(np.eye(K, dtype=np.float32))          # row m selects weight column m
    y = bf16_bits(_run(x, q, bs, g, None, None, cuda))           # y[m, n] = W[n, m]
    w = np.ascontiguousarray(O.dequant_nvfp4(q, bs, float(g), 2).T)  # the reference's bf16 weight
    # code 0x8 decodes to -0.0; a matmul sums it with +0 products, so the output zero is +0
    w[w == 0x8000] = 0
    assert np.array_equal(y, w)


def test_kat_weights_through_the_linear(cuda):
    """portable/kernels.rs:334-355 codes and scales, read through the fused linear with one-hot rows."""
    K, N = 64, 128
    q = np.full((N, K // 2), 0x12, dtype=np.uint8)
    bs = np.zeros(512, dtype=np.uint8)
    for r in range(128):
        for blk in range(4):
            bs[(r % 32) * 16 + (r // 32) * 4 + blk] = 0x38 if r < 32 else 0x40
    x = O.f32_to_bf16_bits(np.eye(K, dtype=np.float32))
    y = O.bf16_bits_to_f32(bf16_bits(_run(x, q, bs, np.float32(3.0), None, None, cuda)))
    for c in (0, 1, 62, 63):
        for r in (0, 31, 32, 127):
            assert y[c, r] == (0.5 if c % 2 == 0 else 1.0) * (1.0 if r < 32 else 2.0) * 3.0


@pytest.mark.parametrize("M,K,N,awq,bias", [(300, 1024, 1024, True, True), (77, 512, 384, False, True),
                                            (512, 4096, 512, True, False), (1, 256, 256, True, True),
                                            (300, 2048, 384, True, True), (512, 2048, 384, True, False)])
def test_linear_matches_reference_composition(cuda, M, K, N, awq, bias):
    x, q, bs, g, pqs, b = O.make_nvfp4_inputs(M + N, M, K, N)
    y = O.bf16_bits_to_f32(bf16_bits(_run(x, q, bs, g, pqs if awq else None, b if bias else None, cuda)))
    want = O.bf16_bits_to_f32(O.nvfp4_linear(x, q, bs, g, pqs if awq else None, b if bias else None))
    assert O.max_abs_rel(y, want) < TOL


@pytest.mark.parametrize("K,N", [(5120, 25600), (25600, 5120)])
def test_text_encoder_shapes_sampled_rows(cuda, K, N):
    """BASELINE config 3 (M = 512 prompt tokens): every row computed on the device, sampled rows checked."""
    M = 512
    x, q, bs, g, pqs, b = O.make_nvfp4_inputs(K, M, K, N)
    y = O.bf16_bits_to_f32(bf16_bits(_run(x, q, bs, g, pqs, None, cuda)))
    rows = np.r_[0:4, 255:258, 508:512]
    want = O.bf16_bits_to_f32(O.nvfp4_linear(x, q, bs, g, pqs, None, rows=rows))
    assert O.max_abs_rel(y[rows], want) < TOL
    assert np.isfinite(y).all()
