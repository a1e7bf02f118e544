"""GPU tests of the bounded-wait failure path: a kernel wait that runs out returns an error status the host reads,
and the context stays usable.

No wait of the library's kernels runs out in normal operation, so h3q_selftest_wait_timeout makes one run out: a
CTA with a pipeline kernel's roles waits on a barrier nothing completes, its producer gives up after a 1 ms limit
through the same bounded-wait code every kernel uses, the other roles leave on the abort flag, TMEM is freed and
the kernel returns.  The host then reads H3Q_ERR_TIMEOUT from h3q_device_status, and the next GEMM (which takes
TMEM on every SM) still runs and matches the oracle bit for bit.  Nothing here faults, traps or spins forever.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

import h3q
from oracle import oracle as O
from tests.gpu_util import bf16_bits, linear_inputs

pytestmark = pytest.mark.gpu

SELFTEST_CODE = 10  # kDevTimeoutSelftest (ptx.cuh)


def _selftest(target: int, limit_ns: int, dev):
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    h3q.check(h3q.lib().h3q_selftest_wait_timeout(target, limit_ns, done.data_ptr(),
                                                  torch.cuda.current_stream(dev).cuda_stream))
    t0 = time.perf_counter()
    torch.cuda.synchronize(dev)
    return int(done.item()), time.perf_counter() - t0


def test_bounded_wait_times_out_and_reports(cuda):
    assert h3q.device_status(0) == 0  # clears anything left by earlier tests
    done, secs = _selftest(0, 1_000_000, cuda)
    assert done == 3, "the CTA must reach its exit path and its producer's wait must give up"
    assert secs < 5.0, f"a 1 ms wait limit took {secs:.2f} s to end the kernel"
    code = ctypes.c_int(0)
    st = h3q.lib().h3q_device_status(0, ctypes.byref(code))
    assert st == h3q.ERR_TIMEOUT and code.value == SELFTEST_CODE
    assert "gave up waiting" in h3q.last_error()
    assert h3q.device_status(0) == 0, "reading the status clears it"


def test_context_usable_after_timeouts(cuda):
    for _ in range(3):
        done, _ = _selftest(0, 1_000_000, cuda)
        assert done == 3
        assert h3q.device_status(0) == SELFTEST_CODE
    (x, w, ws, bias), (xd, wd, wsd, bd) = linear_inputs(5, 300, 1024, 768, cuda)
    y = h3q.gemm_s8(xd, wd, wsd, bd, swiglu=False, rotate=True)
    torch.cuda.synchronize()
    want = O.gemm_s8(x, w, ws, bias, swiglu=False, rotate=True)[0]
    np.testing.assert_array_equal(bf16_bits(y), want)
    assert h3q.device_status(0) == 0


def test_selftest_rejects_bad_arguments(cuda):
    L = h3q.lib()
    assert L.h3q_selftest_wait_timeout(0, 0, None, None) == h3q.ERR_ARG
    assert L.h3q_selftest_wait_timeout(0, 2_000_000_000, None, None) == h3q.ERR_ARG
    assert L.h3q_selftest_wait_timeout(7, 1000, None, None) == h3q.ERR_ARG
