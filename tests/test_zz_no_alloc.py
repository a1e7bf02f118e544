"""GPU test of h3q_gemm_s8_static, the gemm_s8 entry point for callers that cannot allocate device memory.

Such callers (a plugin in a host that has reserved all GPU memory for its own pool, or code that cannot afford
cudaMalloc's synchronisation) get the quantized-activation scratch from a fixed array inside the library instead
of a workspace they allocate.  The test calls it through the C ABI, twice in a row with different inputs (the
second call reuses the array the first one filled), and checks each result against h3q_gemm_s8, the entry point
with a caller-allocated workspace, bit for bit (the tolerance the other linear-epilogue tests use).  It also
checks that a problem too large for the fixed array is refused.  This file sorts last so that a run stopping at
the first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from tests.gpu_util import bf16_tensor, t

pytestmark = pytest.mark.gpu

CALLS = [  # (seed, M, K, N, swiglu, rotate)
    (101, 300, 5120, 1024, False, True),
    (202, 129, 1024, 768, True, True),
]


def _static_call(x, w, ws, bias, swiglu, rotate):
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty((M, N // 2 if swiglu else N), dtype=torch.bfloat16, device=x.device)
    st = h3q.lib().h3q_gemm_s8_static(x.data_ptr(), w.data_ptr(), ws.data_ptr(), ws.numel(), bias.data_ptr(),
                                      out.data_ptr(), M, N, K, int(swiglu), int(rotate),
                                      torch.cuda.current_stream().cuda_stream)
    h3q.check(st)
    return out


def test_static_scratch_matches_workspace_entry_point(cuda):
    outs = []
    for seed, M, K, N, swiglu, rotate in CALLS:
        x, w, ws, bias = O.make_linear_inputs(seed, M, K, N)
        xd, wd, wsd, bd = bf16_tensor(x, cuda), t(w, cuda), t(ws, cuda), t(bias, cuda)
        got = _static_call(xd, wd, wsd, bd, swiglu, rotate)
        want = h3q.gemm_s8(xd, wd, wsd, bd, swiglu=swiglu, rotate=rotate)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
        outs.append(got)
    assert h3q.device_status(0) == 0
    assert outs[0].shape != outs[1].shape


def test_static_scratch_rejects_oversized_problem(cuda):
    M, K, N = 32760, 5120, 256  # 168 MB of codes: more than the fixed array holds
    x = torch.zeros((M, K), dtype=torch.bfloat16, device=cuda)
    w = torch.zeros((N, K), dtype=torch.int8, device=cuda)
    ws = torch.ones(N, device=cuda)
    b = torch.zeros(N, device=cuda)
    with pytest.raises(h3q.H3QError) as e:
        _static_call(x, w, ws, b, False, True)
    assert e.value.status == h3q.ERR_ARG and "fixed" in str(e.value)
