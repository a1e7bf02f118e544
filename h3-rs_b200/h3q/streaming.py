"""h3q.streaming -- weights kept in host memory and streamed to the GPU layer by layer (h3q_streamer_*; the
reference's copy-stream uploads, weights.rs:185-273, and its per-block fetch, dit.rs:1160-1186).

    ws = WeightStreamer(slot_bytes, slots=2, device=dev)
    views, slot = ws.fetch([w_host, scale_host])   # enqueued on the copy stream; the current stream waits for it
    ... enqueue the kernels that read `views` on the current stream ...
    ws.release(slot)                               # after the slot's last reader is enqueued
"""
from __future__ import annotations

import ctypes

from . import _stream, check, lib


class _CudaView:
    """A device region seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


_TYPESTR = {"torch.int8": "|i1", "torch.uint8": "|u1", "torch.float32": "<f4", "torch.float16": "<f2",
            "torch.bfloat16": "<i2", "torch.int32": "<i4", "torch.int64": "<i8"}


class WeightStreamer:
    """A ring of `slots` device slots of slot_bytes each, filled from host tensors on a copy stream."""

    def __init__(self, slot_bytes: int, slots: int = 2, device=None):
        import torch
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib().h3q_streamer_create(slot_bytes, slots, ctypes.byref(h)))
        self._h = h
        self.slots = slots

    def close(self) -> None:
        if self._h:
            lib().h3q_streamer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def fetch(self, host_tensors):
        """Enqueue the copies of the (contiguous, ideally pinned) host tensors into the next slot; returns their
        device views (same shapes and dtypes) and the slot index."""
        import torch
        n = len(host_tensors)
        src = (ctypes.c_void_p * n)(*[t.data_ptr() for t in host_tensors])
        nb = (ctypes.c_size_t * n)(*[t.numel() * t.element_size() for t in host_tensors])
        dst = (ctypes.c_void_p * n)()
        slot = ctypes.c_int()
        check(lib().h3q_streamer_fetch(self._h, src, nb, n, _stream(self.device), ctypes.byref(slot), dst))
        views = []
        for t, p in zip(host_tensors, dst):
            v = torch.as_tensor(_CudaView(p, t.shape, _TYPESTR[str(t.dtype)]), device=self.device)
            views.append(v.view(torch.bfloat16) if t.dtype == torch.bfloat16 else v)
        return views, slot.value

    def release(self, slot: int) -> None:
        check(lib().h3q_streamer_release(self._h, slot, _stream(self.device)))


__all__ = ["WeightStreamer"]
