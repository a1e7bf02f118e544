"""GPU parity: the fused rotate + quantize kernel against the oracle and against the reference's own kernels
(compiled from their CUDA C text).  Codes and scales must be bit-identical."""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from oracle import ref as R
from tests.gpu_util import bf16_tensor, t

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1), (3, 4), (129, 20), (64, 21), (17, 54), (8, 56), (5, 57), (4, 64), (300, 20)]


@pytest.mark.parametrize("M,G", SHAPES)
@pytest.mark.parametrize("rotate", [True, False])
def test_quant_rows_bf16_bit_exact(cuda, M, G, rotate):
    K = 256 * G
    x, _, _, _ = O.make_linear_inputs(M * 1000 + G, M, K, 1)
    q, s = h3q.quant_rows(bf16_tensor(x, cuda), rotate)
    qo, so = O.quant_rows(x, 2, O.reference_quant_mode(2, K, rotate))
    assert np.array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), qo)


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("rotate", [True, False])
def test_quant_rows_f32_f16_bit_exact(cuda, kind, rotate):
    M, K = 37, 1024
    rng = np.random.default_rng(kind + 2 * rotate)
    xf = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    if kind == 0:
        x_host, x_dev = xf, t(xf, cuda)
    else:
        x_host = xf.astype(np.float16).view(np.uint16)
        x_dev = t(xf.astype(np.float16), cuda)
    q, s = h3q.quant_rows(x_dev, rotate)
    qo, so = O.quant_rows(x_host, kind, O.reference_quant_mode(kind, K, rotate))
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy(), so)


def test_quant_rows_unrotated_any_k(cuda):
    """quant_rows_i8 handles any K (kernels.rs:296-318)."""
    M, K = 5, 1000
    x, _, _, _ = O.make_linear_inputs(9, M, K, 1)
    q, s = h3q.quant_rows(bf16_tensor(x, cuda), False)
    qo, so = O.quant_rows(x, 2, O.QUANT_PLAIN)
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(s.cpu().numpy(), so)


def test_quant_rows_zero_and_nonfinite_rows(cuda):
    K = 512
    x = np.zeros((4, K), dtype=np.float32)
    x[1, 3] = np.inf
    x[2, 7] = np.nan
    x[2, 8] = 1.0
    x[3, :] = 1e-35
    bits = O.f32_to_bf16_bits(x)
    for rotate in (True, False):
        q, s = h3q.quant_rows(bf16_tensor(bits, cuda), rotate)
        qo, so = O.quant_rows(bits, 2, O.reference_quant_mode(2, K, rotate))
        assert np.array_equal(q.cpu().numpy(), qo)
        assert np.array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))


@pytest.mark.skipif(not R.available(), reason="reference comparator not built")
@pytest.mark.parametrize("M,G", [(7, 4), (130, 20), (33, 54), (9, 56), (6, 60)])
def test_quant_rows_match_reference_kernels(cuda, M, G):
    """The reference's quant_rows_i8_rot2 / quant_rows_i8_rot, run on this GPU, equal both the oracle and h3q."""
    K = 256 * G
    x, _, _, _ = O.make_linear_inputs(G, M, K, 1)
    xd = bf16_tensor(x, cuda)
    for rotate in (True, False):
        qr, sr = R.quant_rows(xd, 2, rotate)
        qh, sh = h3q.quant_rows(xd, rotate)
        qo, so = O.quant_rows(x, 2, O.reference_quant_mode(2, K, rotate))
        assert np.array_equal(qr.cpu().numpy(), qo), "oracle differs from the reference kernel"
        assert np.array_equal(sr.cpu().numpy(), so)
        assert torch.equal(qr, qh) and torch.equal(sr, sh)


@pytest.mark.skipif(not R.available(), reason="reference comparator not built")
def test_linear_path_quantizer_matches_reference(cuda):
    """int8_linear_ex quantizes with quant_rows_i8_rot (kernels.rs:979-991), also for bf16 input."""
    M, K = 65, 5120
    x, _, _, _ = O.make_linear_inputs(11, M, K, 1)
    xd = bf16_tensor(x, cuda)
    qr, sr = R.quant_rows(xd, 2, True, linear_path=True)
    qo, so = O.quant_rows(x, 2, O.QUANT_ROT)
    assert np.array_equal(qr.cpu().numpy(), qo) and np.array_equal(sr.cpu().numpy(), so)
