"""h3q.parallel -- the quantized linear and the int8 attention across the GPUs of one node, one process per GPU.

The reference runs on a single GPU; partitioning follows the data:

* Token (M) sharding, weights replicated: rank r owns rows row_range(M, world, r) of every activation.  The linear
  needs no collective (per-row quantisation, per-row scales); gather_rows() assembles a full [M, ...] tensor on
  every rank when a caller needs one.
* N-split linear: rank r holds the weight rows (output columns) nsplit_range(N, world, r) and the full activation;
  NSplitLinear writes each rank's column block into every rank's output inside the GEMM (peer memory over
  NVLink, h3q_gemm_s8_allgather), or computes locally and all-gathers through NCCL; by default the faster of the
  two for the number of ranks.
* Query-sharded attention: rank r owns query rows row_range(S, world, r); K and V rows are gathered from all ranks
  and each rank attends its queries against every key (h3q_attention_rows).  Its rows equal the single-GPU
  result's (per-token scales).

Collectives go through torch.distributed: NCCL between GPUs, gloo in the CPU tests.  The operators are parameters
so the host logic can be exercised on CPU with the oracle; on GPUs they default to this library's kernels.
"""
from __future__ import annotations

import ctypes

from . import H3QError, _p, _stream, check, lib
from . import attention_rows as _attention_rows
from . import gemm_s8_quantized as _gemm_s8_quantized
from . import quant_rows as _quant_rows


def row_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [floor(r total / g), floor((r + 1) total / g)) of rank r."""
    return total * rank // world, total * (rank + 1) // world


def nsplit_range(n: int, world: int, rank: int, align: int = 256) -> tuple[int, int]:
    """Output columns of rank r in the N split: whole `align`-column GEMM tiles, as evenly as possible, so every
    block but the last is tile aligned (and a multiple of 8, as the peer stores need)."""
    tiles = -(-n // align)
    t0, t1 = tiles * rank // world, tiles * (rank + 1) // world
    return min(n, t0 * align), min(n, t1 * align)


def _dist():
    import torch.distributed as dist
    return dist


def gather_rows(local, total: int, group=None):
    """Every rank's row block (row_range order) -> the full [total, ...] tensor on every rank.  Blocks may differ
    by a row; they are padded to the largest for the collective and trimmed after."""
    import torch
    dist = _dist()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    ranges = [row_range(total, world, r) for r in range(world)]
    if local.shape[0] != ranges[rank][1] - ranges[rank][0]:
        raise ValueError(f"gather_rows: rank {rank} holds {local.shape[0]} rows, expected {ranges[rank]}")
    width = max(hi - lo for lo, hi in ranges)
    buf = local.new_zeros((width,) + tuple(local.shape[1:]))
    buf[: local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([parts[r][: hi - lo] for r, (lo, hi) in enumerate(ranges)], dim=0)


def gather_columns(local, n: int, group=None, align: int = 256):
    """Every rank's column block (nsplit_range order) of an [M, n_r] output -> [M, n] on every rank (the NCCL
    all-gather plus relayout that the fused N-split GEMM makes unnecessary)."""
    import torch
    dist = _dist()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    ranges = [nsplit_range(n, world, r, align) for r in range(world)]
    width = max(hi - lo for lo, hi in ranges)
    buf = local.new_zeros((local.shape[0], width))
    buf[:, : local.shape[1]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf.contiguous(), group=group)
    return torch.cat([parts[r][:, : hi - lo] for r, (lo, hi) in enumerate(ranges)], dim=1)


class _CudaArray:
    """A raw device allocation seen by torch through __cuda_array_interface__ (int16 elements)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffers:
    """One [rows, cols] bf16 buffer per rank, every rank's mapped into every process (CUDA IPC), so a kernel on
    any GPU can write any rank's copy.  Set-up allocates; use it for as long as the shape stays."""

    def __init__(self, rows: int, cols: int, device, group=None):
        import torch
        dist = _dist()
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.rows, self.cols = rows, cols
        nbytes = rows * cols * 2
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        with torch.cuda.device(device):
            check(lib().h3q_peer_buffer_alloc(nbytes, ctypes.byref(own), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.ptrs = []
        self._opened = []
        with torch.cuda.device(device):
            for r in range(self.world):
                if r == self.rank:
                    self.ptrs.append(own.value)
                    continue
                p = ctypes.c_void_p()
                hb = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
                check(lib().h3q_peer_buffer_open(hb, ctypes.byref(p)))
                self.ptrs.append(p.value)
                self._opened.append(p.value)
        self._own = own.value
        self.local = torch.as_tensor(_CudaArray(self._own, (rows, cols)), device=device).view(torch.bfloat16)
        self.device = device

    def close(self) -> None:
        import torch
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            for p in self._opened:
                lib().h3q_peer_buffer_close(ctypes.c_void_p(p))
            self._opened = []
            if self._own:
                self.local = None
                lib().h3q_peer_buffer_free(ctypes.c_void_p(self._own))
                self._own = None


class NSplitLinear:
    """attn8::gemm_s8 (linear epilogue, bf16 out) with the weight rows split over the ranks.  Every rank passes the
    full activation x [M, K] and receives the full output [M, N]; rank r stores the columns nsplit_range(N, g, r).

    fused=True: one kernel per rank computes its columns and writes them into every rank's output buffer over
    NVLink; a one-element all-reduce after it is the barrier that makes the output complete.  fused=False: local
    GEMM, then gather_columns (NCCL all-gather + relayout).  fused=None (the default) picks the faster one as
    measured on B200 for the DiT linears: the fused kernel up to FUSED_MAX_RANKS ranks (2 GPUs: 4.6 ms against
    8.8 ms for the four c1 linears), NCCL beyond (8 GPUs: 10.2 ms against 27.1 ms, where every output box becomes
    seven small remote stores)."""

    FUSED_MAX_RANKS = 2

    def __init__(self, w, ws, bias, group=None, fused: bool | None = None, rotate: bool = True):
        import torch
        dist = _dist()
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.n = w.shape[0]
        self.n0, self.n1 = nsplit_range(self.n, self.world, self.rank)
        self.w = w[self.n0:self.n1].contiguous()
        ws = ws.to(torch.float32).reshape(-1)
        self.ws = (ws[self.n0:self.n1] if ws.numel() == self.n and self.n > 1 else ws[:1]).contiguous()
        self.bias = None if bias is None else bias.to(torch.float32)[self.n0:self.n1].contiguous()
        self.fused = (self.world <= self.FUSED_MAX_RANKS) if fused is None else bool(fused)
        self.rotate = rotate
        self.bufs = None
        self._flag = None

    def _buffers(self, m: int, device):
        if self.bufs is None or self.bufs.rows != m:
            if self.bufs is not None:
                self.bufs.close()
            self.bufs = PeerBuffers(m, self.n, device, self.group)
        return self.bufs

    def forward(self, x):
        import torch
        dist = _dist()
        q, xs = _quant_rows(x, self.rotate)
        if not self.fused:
            y = _gemm_s8_quantized(q, xs, self.w, self.ws, self.bias)
            return gather_columns(y, self.n, self.group)
        m, k = q.shape
        bufs = self._buffers(m, x.device)
        outs = (ctypes.c_void_p * self.world)(*bufs.ptrs)
        check(lib().h3q_gemm_s8_allgather(_p(q), _p(xs), _p(self.w), _p(self.ws), self.ws.numel(), _p(self.bias),
                                          outs, self.world, m, self.n, self.n0, self.n1 - self.n0, k,
                                          _stream(x.device)))
        if self._flag is None:
            self._flag = torch.zeros(1, device=x.device)
        dist.all_reduce(self._flag, group=self.group)  # every rank's stores are complete past this point
        return bufs.local

    def close(self) -> None:
        if self.bufs is not None:
            self.bufs.close()
            self.bufs = None


def gather_full(local, total: int, group=None):
    """gather_rows without the staging copies when every rank holds the same number of rows (total divisible by
    the world size): one all-gather straight into the full [total, ...] tensor, rank blocks in rank order."""
    dist = _dist()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if total % world != 0:
        return gather_rows(local, total, group)
    lo, hi = row_range(total, world, rank)
    if local.shape[0] != hi - lo:
        raise ValueError(f"gather_full: rank {rank} holds {local.shape[0]} rows, expected {(lo, hi)}")
    out = local.new_empty((total,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def sharded_attention(q_local, k_local, v_local, total: int, group=None, flags: int = 0, rows_op=None):
    """Query-sharded attention: this rank's rows q_local, k_local, v_local ([s_r, H, 128], row_range order) ->
    its output rows [s_r, H, 128], attending over the keys and values of every rank.  K and V are each gathered
    straight into full tensors (gather_full).  rows_op(q, k, v, flags) defaults to h3q.attention_rows."""
    k_full = gather_full(k_local, total, group)
    v_full = gather_full(v_local, total, group)
    if rows_op is None:
        H = q_local.shape[1]
        return _attention_rows(q_local, k_full, v_full.reshape(total, H * 128), H * 128, 0, flags)
    return rows_op(q_local, k_full, v_full, flags)


class RankLeft(RuntimeError):
    """A rank announced that it left the job (RankMonitor.leave)."""

    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank} left the job: {reason}")
        self.rank = rank


class RankLost(RuntimeError):
    """A rank did not reach a step within the monitor's time limit and did not say why."""

    def __init__(self, ranks, step: int, timeout: float):
        super().__init__(f"rank(s) {list(ranks)} did not reach step {step} within {timeout:.1f} s")
        self.ranks = list(ranks)


class JobCancelled(RuntimeError):
    """Some rank cancelled the job (RankMonitor.cancel_all)."""


class RankMonitor:
    """Between-step failure detection for one multi-GPU job, on the host only.

    The reference runs on one GPU and checks for cancellation between steps and blocks (progress::check,
    progress.rs:102-107, called per block at dit.rs:1164; cancel_all bumps a generation, progress.rs:87-89).  With
    several ranks a step's collectives would wait for a rank that has gone, so before issuing a step's kernels and
    collectives every rank calls ready(step):

      * it publishes its own heartbeat (the step number) in the job's key-value store (torch.distributed's store:
        TCPStore between processes);
      * it raises JobCancelled if any rank called cancel_all() since this monitor was made;
      * it raises RankLeft if a rank called leave();
      * it waits until every rank has published a heartbeat of at least `step`, and raises RankLost for the ranks
        still missing after `timeout` seconds.

    cancel_all() and leave() are called between steps, before the caller's next ready(); since every rank waits
    for every heartbeat of a step and then looks once more, all ranks raise at the same step.

    Every surviving rank therefore learns of a departure before its next launch, with no kernel or collective of
    that step in flight.  A rank leaves only between steps.  A rank that dies inside a step is caught by the
    process group's own (short) timeout in the collective it left behind."""

    def __init__(self, store, rank: int, world: int, prefix: str = "h3q/monitor", timeout: float = 10.0,
                 poll: float = 0.01):
        self.store, self.rank, self.world = store, rank, world
        self.prefix, self.timeout, self.poll = prefix, float(timeout), float(poll)
        self.gen = int(self.store.add(f"{prefix}/gen", 0))

    def _beat_key(self, r: int) -> str:
        return f"{self.prefix}/beat/{r}"

    def _left_key(self, r: int) -> str:
        return f"{self.prefix}/left/{r}"

    def _raise_if_stopped(self) -> None:
        if int(self.store.add(f"{self.prefix}/gen", 0)) != self.gen:
            raise JobCancelled("the job was cancelled")
        for r in range(self.world):
            if r != self.rank and self.store.check([self._left_key(r)]):
                raise RankLeft(r, self.store.get(self._left_key(r)).decode(errors="replace"))

    def ready(self, step: int) -> None:
        import time
        self.store.set(self._beat_key(self.rank), str(int(step)))
        deadline = time.monotonic() + self.timeout
        missing = [r for r in range(self.world) if r != self.rank]
        while True:
            self._raise_if_stopped()
            missing = [r for r in missing
                       if not (self.store.check([self._beat_key(r)]) and
                               int(self.store.get(self._beat_key(r))) >= step)]
            if not missing:
                # a rank cancels or leaves before it publishes its next heartbeat, so once every heartbeat of this
                # step is visible, one more look sees any cancellation made ahead of it: all ranks agree
                self._raise_if_stopped()
                return
            if time.monotonic() > deadline:
                raise RankLost(missing, step, self.timeout)
            time.sleep(self.poll)

    def leave(self, reason: str = "left") -> None:
        self.store.set(self._left_key(self.rank), reason)

    def cancel_all(self) -> None:
        self.store.add(f"{self.prefix}/gen", 1)


__all__ = ["row_range", "nsplit_range", "gather_rows", "gather_full", "gather_columns", "PeerBuffers", "NSplitLinear",
           "sharded_attention", "H3QError", "RankMonitor", "RankLeft", "RankLost", "JobCancelled"]
