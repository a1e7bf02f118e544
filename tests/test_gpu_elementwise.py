"""GPU parity of the weight-decode and gated-residual kernels (bit-exact)."""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from oracle import ref as R
from tests.gpu_util import bf16_bits, bf16_tensor, t

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols,per_row", [(64, 256, True), (7, 100, True), (33, 48, False), (1, 16, True)])
@pytest.mark.parametrize("okind,dtype", [(0, torch.float32), (1, torch.float16), (2, torch.bfloat16)])
def test_dequant_i8(cuda, rows, cols, per_row, okind, dtype):
    rng = np.random.default_rng(rows * cols)
    q = rng.integers(-128, 128, size=(rows, cols), dtype=np.int8)
    s = (rng.random(rows if per_row else 1, dtype=np.float32) * 0.01).astype(np.float32)
    out = h3q.dequant_i8(t(q, cuda), t(s, cuda), dtype)
    want = O.dequant_i8(q, s, okind)
    got = out.cpu().numpy() if okind == 0 else out.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, want)


def test_dequant_nvfp4_kat(cuda):
    """portable/kernels.rs:334-355 on the device."""
    q = np.full((128, 32), 0x12, dtype=np.uint8)
    scales = np.zeros(512, dtype=np.uint8)
    for r in range(128):
        for block in range(4):
            scales[(r % 32) * 16 + (r // 32) * 4 + block] = 0x38 if r < 32 else 0x40
    y = h3q.dequant_nvfp4(t(q, cuda), t(scales, cuda), torch.tensor([3.0], device=cuda), torch.float32).cpu().numpy()
    for r in (0, 31, 32, 127):
        for c in range(64):
            assert y[r, c] == (0.5 if c % 2 == 0 else 1.0) * (1.0 if r < 32 else 2.0) * 3.0


@pytest.mark.parametrize("rows,k", [(256, 5120), (130, 64), (1, 16)])
def test_dequant_nvfp4_random(cuda, rows, k):
    rng = np.random.default_rng(rows + k)
    q = rng.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
    ncb = (k // 16 + 3) // 4
    nbytes = ((rows + 127) // 128) * ncb * 512
    bs = rng.integers(0x30, 0x50, size=nbytes, dtype=np.uint8)
    g = np.float32(1.0 / 448)
    for okind, dtype in ((0, torch.float32), (2, torch.bfloat16)):
        out = h3q.dequant_nvfp4(t(q, cuda), t(bs, cuda), torch.tensor([g], device=cuda), dtype)
        want = O.dequant_nvfp4(q, bs, float(g), okind)
        got = out.cpu().numpy() if okind == 0 else out.view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got, want)
        if R.available():
            ref = R.dequant_nvfp4(t(q, cuda), t(bs, cuda), torch.tensor([g], device=cuda), dtype)
            assert torch.equal(ref, out)


def test_gate_add(cuda):
    S, C = 100, 384
    rng = np.random.default_rng(5)
    x = O.f32_to_bf16_bits(rng.standard_normal((S, C)).astype(np.float32))
    y = O.f32_to_bf16_bits(rng.standard_normal((S, C)).astype(np.float32))
    gate = rng.random((4, C), dtype=np.float32)
    idx = rng.integers(0, 4, size=S).astype(np.uint32)
    out = h3q.gate_add(bf16_tensor(x, cuda), bf16_tensor(y, cuda), t(gate, cuda), t(idx, cuda))
    assert np.array_equal(bf16_bits(out), O.gate_add(x, y, 2, gate, idx))
