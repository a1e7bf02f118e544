"""GPU tests of the standalone ConvRot rotation (h3q_rotate_activation, weights.rs:482-489) and SwiGLU (h3q_swiglu,
weights.rs:806-816 / ops.rs:39-44): the rotation bit-exact against the oracle's butterfly and within one bf16
rounding of the exact f64 rotation; SwiGLU against the oracle (device __expf vs host expf: over 99% of outputs
identical, all within 1e-2) in both column layouts."""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from tests.gpu_util import bf16_bits, bf16_tensor

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K", [(300, 5120), (64, 13824), (5, 256), (1000, 16384), (1, 1024)])
def test_rotate_activation(cuda, M, K):
    rng = np.random.default_rng(M + K)
    x = O.f32_to_bf16_bits((rng.standard_normal((M, K)) * 3).astype(np.float32))
    got = bf16_bits(h3q.rotate_activation(bf16_tensor(x, cuda)))
    np.testing.assert_array_equal(got, O.rotate_bf16(x))
    exact = O.rotate_f64(O.bf16_bits_to_f32(x).astype(np.float64))
    g = O.bf16_bits_to_f32(got).astype(np.float64)
    # one bf16 rounding (half an ulp, 2^-9 relative) plus the f32 butterfly's own rounding, tiny against the row
    assert np.all(np.abs(g - exact) <= 2.0 ** -8 * np.abs(exact) + 1e-5 * np.abs(exact).max())


def test_rotate_activation_rejects_bad_widths(cuda):
    with pytest.raises(h3q.H3QError, match="does not divide"):
        h3q.rotate_activation(torch.zeros((4, 300), dtype=torch.bfloat16, device=cuda))
    with pytest.raises(h3q.H3QError):
        h3q.rotate_activation(torch.zeros((4, 256 * 65), dtype=torch.bfloat16, device=cuda))


@pytest.mark.parametrize("interleaved", [True, False])
@pytest.mark.parametrize("rows,F", [(300, 6912), (7, 64), (1024, 13824)])
def test_swiglu(cuda, interleaved, rows, F):
    rng = np.random.default_rng(rows + F)
    y = O.f32_to_bf16_bits((rng.standard_normal((rows, 2 * F)) * 4).astype(np.float32))
    got = bf16_bits(h3q.swiglu(bf16_tensor(y, cuda), interleaved))
    want = O.swiglu_bf16(y, interleaved)
    assert (got == want).mean() > 0.99
    assert O.max_abs_rel(O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(want)) <= 1e-2
    assert h3q.device_status() == 0
