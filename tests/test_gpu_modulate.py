"""GPU parity of RMSNorm + adaLN modulate (kernels.rs:376-401), alone and fused into the rotated int8 quantizer.

Against the reference's own rms_modulate kernel compiled for sm_100a: bit-exact (same reduction order, same
hardware rsqrtf).  The fused kernel's codes and row scales equal h3q's quantizer applied to the modulated rows, bit
for bit.  Against the CPU oracle (1/sqrtf for rsqrtf): over 99% of the bf16 outputs identical, all within 1e-2.
"""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from oracle import ref as R
from tests.gpu_util import bf16_bits, bf16_tensor, t

pytestmark = pytest.mark.gpu

SHAPES = [(1, 256), (77, 1024), (300, 5120), (64, 13824), (5, 16384)]
EPS = 1e-6


def _inputs(seed, S, C, dev):
    x, w, sc, sh, idx = O.make_modulate_inputs(seed, S, C)
    return (x, w, sc, sh, idx), (bf16_tensor(x, dev), bf16_tensor(w, dev), t(sc, dev), t(sh, dev), t(idx, dev))


@pytest.mark.skipif(not R.available(), reason="reference kernels not built (make -C oracle ref)")
@pytest.mark.parametrize("S,C", SHAPES)
def test_rms_modulate_matches_reference_kernel(cuda, S, C):
    _, (x, w, sc, sh, idx) = _inputs(S + C, S, C, cuda)
    got = h3q.rms_modulate(x, w, EPS, sc, sh, idx)
    want = R.rms_modulate(x, w, EPS, sc, sh, idx)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("S,C", SHAPES)
def test_rms_modulate_vs_oracle(cuda, S, C):
    (xn, wn, scn, shn, idxn), (x, w, sc, sh, idx) = _inputs(S + 2 * C, S, C, cuda)
    got = bf16_bits(h3q.rms_modulate(x, w, EPS, sc, sh, idx))
    want = O.rms_modulate(xn, wn, EPS, scn, shn, idxn)
    # rsqrtf and 1/sqrtf may differ in the last bit of inv; that moves n by at most one bf16 unit, which the
    # modulation can turn into a few units of a nearly cancelled output
    assert (got == want).mean() > 0.99
    assert O.max_abs_rel(O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(want)) <= 1e-2


@pytest.mark.parametrize("S,C", SHAPES)
def test_fused_quant_equals_quant_of_modulated_rows(cuda, S, C):
    _, (x, w, sc, sh, idx) = _inputs(3 * S + C, S, C, cuda)
    q, xs = h3q.rms_modulate_quant(x, w, EPS, sc, sh, idx)
    q2, xs2 = h3q.quant_rows(h3q.rms_modulate(x, w, EPS, sc, sh, idx), True)
    assert torch.equal(q, q2)
    assert torch.equal(xs.view(torch.int32), xs2.view(torch.int32))
    if R.available():
        q3, xs3 = R.quant_rows(R.rms_modulate(x, w, EPS, sc, sh, idx), 2, True)
        assert torch.equal(q, q3)
        assert torch.equal(xs.view(torch.int32), xs3.view(torch.int32))


def test_fused_quant_feeds_the_gemm(cuda):
    """The fused pass plus the quantized GEMM equals rms_modulate then gemm_s8 (the DiT's qkv step)."""
    S, C, N = 300, 5120, 1024
    _, (x, w, sc, sh, idx) = _inputs(7, S, C, cuda)
    g = torch.Generator(device=cuda).manual_seed(3)
    wt = torch.randint(-127, 128, (N, C), generator=g, device=cuda, dtype=torch.int8)
    ws = torch.rand(N, generator=g, device=cuda) * 9e-3 + 1e-3
    b = torch.randn(N, generator=g, device=cuda) * 0.02
    q, xs = h3q.rms_modulate_quant(x, w, EPS, sc, sh, idx)
    y = h3q.gemm_s8_quantized(q, xs, wt, ws, b)
    y2 = h3q.gemm_s8(h3q.rms_modulate(x, w, EPS, sc, sh, idx), wt, ws, b, rotate=True)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    assert h3q.device_status() == 0


@pytest.mark.parametrize("S,C", [(6000, 1024), (4000, 5120), (1500, 16384)])
@pytest.mark.parametrize("blocked", [False, True])
def test_many_rows_per_cta(cuda, S, C, blocked):
    """Enough rows that every CTA works through a block of them (the next row's sums are formed under the current
    row's barrier, the table slice is reloaded when the index changes): per-row random table rows, and table rows
    that change every 700 tokens (a latent frame)."""
    _, (x, w, sc, sh, idx) = _inputs(S ^ C, S, C, cuda)
    if blocked:
        idx = ((torch.arange(S, device=cuda) // 700) % sc.shape[0]).to(torch.int32)
    y = h3q.rms_modulate(x, w, EPS, sc, sh, idx)
    q, xs = h3q.rms_modulate_quant(x, w, EPS, sc, sh, idx)
    q2, xs2 = h3q.quant_rows(y, True)
    assert torch.equal(q, q2)
    assert torch.equal(xs.view(torch.int32), xs2.view(torch.int32))
    if R.available():
        assert torch.equal(y.view(torch.int16), R.rms_modulate(x, w, EPS, sc, sh, idx).view(torch.int16))
    else:
        want = O.rms_modulate(bf16_bits(x), bf16_bits(w), EPS, sc.cpu().numpy(), sh.cpu().numpy(),
                              idx.cpu().numpy().astype(np.uint32))
        assert (bf16_bits(y) == want).mean() > 0.99
    assert h3q.device_status() == 0
