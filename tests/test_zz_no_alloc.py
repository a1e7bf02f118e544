"""GPU test of h3q_gemm_s8_static, the gemm_s8 entry point for callers that cannot allocate device memory.

Such callers (a plugin in a host that has reserved all GPU memory for its own pool, or code that cannot afford
cudaMalloc's synchronisation) get the quantized-activation scratch from a fixed array inside the library instead
of a workspace they allocate.  The test calls it through the C ABI, twice in a row with different inputs (the
second call reuses the array the first one filled), and checks each result against h3q_gemm_s8, the entry point
with a caller-allocated workspace, bit for bit (the tolerance the other linear-epilogue tests use).  It checks
that calls after the first on a device change neither torch's allocation count nor the device's free memory,
that a problem too large for the fixed array is refused, and that a kernel time-out on this path is reported by
h3q_gemm_s8_static_status (sticky until read) and not by h3q_device_status.  This file sorts last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes

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
SELFTEST_CODE = 10  # kDevTimeoutSelftest (ptx.cuh)


def _static_call(x, w, ws, bias, swiglu, rotate, out=None):
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N // 2 if swiglu else N), dtype=torch.bfloat16, device=x.device)
    st = h3q.lib().h3q_gemm_s8_static(x.data_ptr(), w.data_ptr(), ws.data_ptr(), ws.numel(), bias.data_ptr(),
                                      out.data_ptr(), M, N, K, int(swiglu), int(rotate),
                                      torch.cuda.current_stream().cuda_stream)
    h3q.check(st)
    return out


def _static_status(dev: int = 0):
    code = ctypes.c_int(0)
    st = h3q.lib().h3q_gemm_s8_static_status(dev, ctypes.byref(code))
    return st, code.value


def _inputs(dev):
    res = []
    for seed, M, K, N, swiglu, rotate in CALLS:
        x, w, ws, bias = O.make_linear_inputs(seed, M, K, N)
        res.append(((bf16_tensor(x, dev), t(w, dev), t(ws, dev), t(bias, dev)), swiglu, rotate))
    return res


def test_static_scratch_matches_workspace_entry_point(cuda):
    outs = []
    for (xd, wd, wsd, bd), swiglu, rotate in _inputs(cuda):
        got = _static_call(xd, wd, wsd, bd, swiglu, rotate)
        want = h3q.gemm_s8(xd, wd, wsd, bd, swiglu=swiglu, rotate=rotate)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
        outs.append(got)
    assert _static_status(0) == (h3q.OK, 0)
    assert outs[0].shape != outs[1].shape


def test_static_scratch_allocates_nothing(cuda):
    cases = _inputs(cuda)
    outs = []
    for (xd, wd, wsd, bd), swiglu, rotate in cases:
        M, N = xd.shape[0], wd.shape[0]
        outs.append(torch.empty((M, N // 2 if swiglu else N), dtype=torch.bfloat16, device=cuda))
    # the first calls on a device may reserve the array and load the kernels' code; later ones allocate nothing
    for ((xd, wd, wsd, bd), swiglu, rotate), out in zip(cases, outs):
        _static_call(xd, wd, wsd, bd, swiglu, rotate, out)
    torch.cuda.synchronize()
    torch_before = torch.cuda.memory_allocated(cuda)
    free_before = torch.cuda.mem_get_info(cuda)[0]
    for _ in range(2):
        for ((xd, wd, wsd, bd), swiglu, rotate), out in zip(cases, outs):
            _static_call(xd, wd, wsd, bd, swiglu, rotate, out)
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(cuda) == torch_before
    assert torch.cuda.mem_get_info(cuda)[0] == free_before


def test_static_status_reports_a_timeout(cuda):
    assert _static_status(0) == (h3q.OK, 0)
    assert h3q.device_status(0) == 0
    done = torch.zeros(1, dtype=torch.int32, device=cuda)
    # a bounded wait made to run out (1 ms) on this path's status word
    h3q.check(h3q.lib().h3q_selftest_wait_timeout(1, 1_000_000, done.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(done.item()) == 3
    assert h3q.device_status(0) == 0, "the static path's time-outs stay out of the device error word"
    # a call made after the time-out does not clear it: the word is sticky until read
    (xd, wd, wsd, bd), swiglu, rotate = _inputs(cuda)[0]
    got = _static_call(xd, wd, wsd, bd, swiglu, rotate)
    st, code = _static_status(0)
    assert st == h3q.ERR_TIMEOUT and code == SELFTEST_CODE
    assert _static_status(0) == (h3q.OK, 0), "reading the status clears it"
    want = h3q.gemm_s8(xd, wd, wsd, bd, swiglu=swiglu, rotate=rotate)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_static_scratch_rejects_oversized_problem(cuda):
    M, K, N = 32760, 5120, 256  # 168 MB of codes: more than the fixed array holds
    x = torch.zeros((M, K), dtype=torch.bfloat16, device=cuda)
    w = torch.zeros((N, K), dtype=torch.int8, device=cuda)
    ws = torch.ones(N, device=cuda)
    b = torch.zeros(N, device=cuda)
    with pytest.raises(h3q.H3QError) as e:
        _static_call(x, w, ws, b, False, True)
    assert e.value.status == h3q.ERR_ARG and "fixed" in str(e.value)
    # rows so many that m * k would wrap a 64-bit product: refused before any size arithmetic
    L = h3q.lib()
    st = L.h3q_gemm_s8_static(x.data_ptr(), w.data_ptr(), ws.data_ptr(), 1, None, x.data_ptr(), 1 << 60, 256, 1024,
                              0, 0, None)
    assert st == h3q.ERR_ARG and "fixed" in h3q.last_error()
