"""GPU test of the per-device set-up (h3q_init): succeeds, can be repeated, and leaves the current device as it
was; calls after it work as before."""
import pytest
import torch

import h3q

pytestmark = pytest.mark.gpu


def test_init_then_call(cuda):
    before = torch.cuda.current_device()
    for d in range(torch.cuda.device_count()):
        h3q.init(d)
        h3q.init(d)
    assert torch.cuda.current_device() == before
    x = torch.randn((64, 256), device=cuda).to(torch.bfloat16)
    w = torch.randint(-127, 128, (128, 256), device=cuda, dtype=torch.int8)
    ws = torch.full((128,), 1e-2, device=cuda)
    y = h3q.gemm_s8(x, w, ws, None, rotate=True)
    torch.cuda.synchronize()
    assert y.shape == (64, 128) and torch.isfinite(y.float()).all()
    assert h3q.device_status() == 0
