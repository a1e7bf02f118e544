"""GPU tests of weight streaming (h3q_streamer_*; the reference's copy-stream uploads, weights.rs:185-273, and its
per-block fetch, dit.rs:1160-1186): layers whose weights stay in pinned host memory and reach the GPU through a
2-slot ring give the bits of the same layers with resident weights, and the ring refuses a slot that is still
held.
"""
import pytest
import torch

import h3q
from h3q.streaming import WeightStreamer

pytestmark = pytest.mark.gpu


def _layers(n, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).pin_memory()
        s = (torch.rand(N, generator=g) * 9e-3 + 1e-3).pin_memory()
        b = (torch.randn(N, generator=g) * 0.02).pin_memory()
        out.append((w, s, b))
    return out


@pytest.mark.parametrize("slots", [1, 2, 3])
def test_streamed_layers_equal_resident_layers(cuda, slots):
    N, K, M = 1024, 1024, 512
    layers = _layers(7, N, K, slots)
    x = (torch.randn((M, K), device=cuda) * 2).to(torch.bfloat16)
    want = [h3q.gemm_s8(x, w.to(cuda), s.to(cuda), b.to(cuda), rotate=True) for w, s, b in layers]
    ws = WeightStreamer(N * K + 2 * 4 * N + 512, slots, cuda)
    got, pending = [], []
    # up to `slots` layers resident; each layer's kernels are enqueued before the next fetch, so the copy of the
    # next layer overlaps them
    for i in range(min(slots, len(layers))):
        pending.append(ws.fetch(list(layers[i])))
    for i in range(len(layers)):
        (w, s, b), slot = pending.pop(0)
        got.append(h3q.gemm_s8(x, w, s, b, rotate=True))
        ws.release(slot)
        if i + slots < len(layers):
            pending.append(ws.fetch(list(layers[i + slots])))
    torch.cuda.synchronize()
    for a, b in zip(got, want):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    ws.close()
    assert h3q.device_status() == 0


def test_held_slot_and_oversized_fetch_are_refused(cuda):
    ws = WeightStreamer(4096, 1, cuda)
    t = torch.zeros(1024, dtype=torch.float32).pin_memory()
    views, slot = ws.fetch([t])
    with pytest.raises(h3q.H3QError, match="still held"):
        ws.fetch([t])
    ws.release(slot)
    with pytest.raises(h3q.H3QError, match="not held"):
        ws.release(slot)
    with pytest.raises(h3q.H3QError, match="exceed the slot size"):
        ws.fetch([torch.zeros(2048, dtype=torch.float32).pin_memory()])
    views, slot = ws.fetch([t])
    ws.release(slot)
    torch.cuda.synchronize()
    assert torch.count_nonzero(views[0]).item() == 0
    ws.close()
