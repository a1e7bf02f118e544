"""GPU tests of gemm_s8 on host activations (h3q_host_pipeline_*): the chunked, overlapped copies in and out give
the bits of h3q_gemm_s8 on device tensors, for ragged last chunks, SwiGLU, and two calls chained through host
memory.
"""
import pytest
import torch

import h3q

pytestmark = pytest.mark.gpu


def _layer(N, K, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    w = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
    ws = torch.rand(N, generator=g, device=dev) * 9e-3 + 1e-3
    b = torch.randn(N, generator=g, device=dev) * 0.02
    return w, ws, b


@pytest.mark.parametrize("M,chunk", [(1000, 256), (4096, 1024), (77, 1024), (3000, 1000)])
def test_host_gemm_equals_device_gemm(cuda, M, chunk):
    K, N = 1024, 768
    w, ws, b = _layer(N, K, M, cuda)
    x = (torch.randn((M, K), device=cuda) * 2).to(torch.bfloat16)
    want = h3q.gemm_s8(x, w, ws, b, rotate=True).cpu()
    pipe = h3q.HostPipeline(chunk, K, N, cuda)
    xh = x.cpu().pin_memory()
    got = pipe.gemm_s8(xh, w, ws, b, rotate=True)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    # SwiGLU epilogue (interleaved rows), output half as wide
    want2 = h3q.gemm_s8(x, w, ws, b, swiglu=True, rotate=True).cpu()
    got2 = pipe.gemm_s8(xh, w, ws, b, swiglu=True, rotate=True)
    torch.cuda.synchronize()
    assert torch.equal(got2.view(torch.int16), want2.view(torch.int16))
    pipe.close()
    assert h3q.device_status() == 0


def test_chained_calls_through_host_memory(cuda):
    """Layer 2 reads layer 1's host output: the second call starts after the first one's last copy out."""
    M, K = 2048, 1024
    w1, s1, b1 = _layer(K, K, 1, cuda)
    w2, s2, b2 = _layer(K, K, 2, cuda)
    x = (torch.randn((M, K), device=cuda) * 2).to(torch.bfloat16)
    want = h3q.gemm_s8(h3q.gemm_s8(x, w1, s1, b1, rotate=True), w2, s2, b2, rotate=True).cpu()
    pipe = h3q.HostPipeline(512, K, K, cuda)
    mid = torch.empty((M, K), dtype=torch.bfloat16, pin_memory=True)
    out = torch.empty((M, K), dtype=torch.bfloat16, pin_memory=True)
    for _ in range(2):  # the second pass reuses every buffer and event
        pipe.gemm_s8(x.cpu().pin_memory(), w1, s1, b1, rotate=True, out=mid)
        pipe.gemm_s8(mid, w2, s2, b2, rotate=True, out=out)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    with pytest.raises(h3q.H3QError, match="exceed"):
        pipe.gemm_s8(torch.zeros((8, 2048), dtype=torch.bfloat16), w1, s1, b1)
    pipe.close()
