"""GPU tests of gemm_s8 on host activations (h3q_host_pipeline_*).

* The chunked, overlapped copies in and out give the bits of h3q_gemm_s8 on device tensors. This holds for ragged
  last chunks, SwiGLU, and two calls chained through host memory.
* A batch (h3q_host_pipeline_run) of independent linears gives the bits of separate calls.
* A batch whose later linear reads an earlier linear's host output gives the bits of the device chain.
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


def test_batch_equals_separate_calls(cuda):
    """Three independent linears of different shapes (one SwiGLU) as one batch, twice, with chunks that straddle
    the linears (the buffer hand-over runs on across them)."""
    M = 1500
    shapes = [(1024, 768, False), (512, 1024, True), (768, 512, False)]
    layers = [(_layer(N, K, 10 + i, cuda), K, N, sw) for i, (K, N, sw) in enumerate(shapes)]
    xs = [(torch.randn((M, K), device=cuda) * 2).to(torch.bfloat16) for _, K, _, _ in layers]
    want = [h3q.gemm_s8(x, w, ws, b, swiglu=sw, rotate=True).cpu() for x, ((w, ws, b), _, _, sw) in zip(xs, layers)]
    pipe = h3q.HostPipeline(400, 1024, 1024, cuda)
    xh = [x.cpu().pin_memory() for x in xs]
    outs = [torch.empty(wt.shape, dtype=torch.bfloat16, pin_memory=True) for wt in want]
    for _ in range(2):
        for o in outs:
            o.zero_()
        pipe.run([(x, w, ws, b, o, sw, True) for x, ((w, ws, b), _, _, sw), o in zip(xh, layers, outs)])
        torch.cuda.synchronize()
        for o, wt in zip(outs, want):
            assert torch.equal(o.view(torch.int16), wt.view(torch.int16))
    pipe.close()
    assert h3q.device_status() == 0


@pytest.mark.parametrize("in_slots,out_slots", [(5, 3), (2, 7)])
def test_batch_with_more_chunk_buffers(cuda, in_slots, out_slots):
    """Copies in running up to in_slots chunks ahead (and GEMMs up to out_slots ahead of the copies out) give the
    same bits, including an item that reads an earlier item's output."""
    M, K = 2500, 1024
    (w1, s1, b1), (w2, s2, b2) = _layer(K, K, 31, cuda), _layer(512, K, 32, cuda)
    x = (torch.randn((M, K), device=cuda) * 2).to(torch.bfloat16)
    y1 = h3q.gemm_s8(x, w1, s1, b1, rotate=True)
    want = [y1.cpu(), h3q.gemm_s8(y1, w2, s2, b2, rotate=True).cpu(), h3q.gemm_s8(x, w2, s2, b2, rotate=True).cpu()]
    pipe = h3q.HostPipeline(300, K, K, cuda, in_slots=in_slots, out_slots=out_slots)
    xh = x.cpu().pin_memory()
    outs = [torch.empty(wt.shape, dtype=torch.bfloat16, pin_memory=True) for wt in want]
    for _ in range(2):
        pipe.run([(xh, w1, s1, b1, outs[0], False, True), (outs[0], w2, s2, b2, outs[1], False, True),
                  (xh, w2, s2, b2, outs[2], False, True)])
        torch.cuda.synchronize()
        for o, wt in zip(outs, want):
            assert torch.equal(o.view(torch.int16), wt.view(torch.int16))
    pipe.close()
    assert h3q.device_status() == 0


def test_batch_chains_through_host_memory(cuda):
    """Linear 2 reads linear 1's host output and linear 3 reads a row slice of linear 2's, in one batch."""
    M, K = 2048, 1024
    (w1, s1, b1), (w2, s2, b2), (w3, s3, b3) = (_layer(K, K, 20 + i, cuda) for i in range(3))
    x = (torch.randn((M, K), device=cuda) * 2).to(torch.bfloat16)
    y1 = h3q.gemm_s8(x, w1, s1, b1, rotate=True)
    y2 = h3q.gemm_s8(y1, w2, s2, b2, rotate=True)
    want = h3q.gemm_s8(y2[700:1900].contiguous(), w3, s3, b3, rotate=True).cpu()
    pipe = h3q.HostPipeline(512, K, K, cuda)
    xh = x.cpu().pin_memory()
    mid1 = torch.empty((M, K), dtype=torch.bfloat16, pin_memory=True)
    mid2 = torch.empty((M, K), dtype=torch.bfloat16, pin_memory=True)
    out = torch.empty((1200, K), dtype=torch.bfloat16, pin_memory=True)
    pipe.run([(xh, w1, s1, b1, mid1, False, True), (mid1, w2, s2, b2, mid2, False, True),
              (mid2[700:1900], w3, s3, b3, out, False, True)])
    torch.cuda.synchronize()
    assert torch.equal(mid2.view(torch.int16), y2.cpu().view(torch.int16))
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    # an item that does not fit fails before anything is enqueued: the outputs keep their bits
    out.zero_()
    with pytest.raises(h3q.H3QError, match="item 1"):
        pipe.run([(xh[:8], w1, s1, b1, out[:8], False, True),
                  (torch.zeros((8, 2048), dtype=torch.bfloat16), w1, s1, b1, out, False, True)])
    torch.cuda.synchronize()
    assert not bool(out.view(torch.int16).any())
    pipe.close()
