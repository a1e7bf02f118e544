"""h3q.parallel -- the quantized linear and the int8 attention across the GPUs of one node, one process per GPU.

The reference runs on a single GPU; partitioning follows the data:

* Token (M) sharding, weights replicated: rank r owns rows row_range(M, world, r) of every activation.  The linear
  needs no collective (per-row quantisation, per-row scales); gather_rows() assembles a full [M, ...] tensor on
  every rank when a caller needs one.
* N-split linear: rank r holds the weight rows (output columns) nsplit_range(N, world, r) and the full activation;
  NSplitLinear runs h3q_gemm_s8_nsplit (C ABI) in one of its forms: the GEMM storing each output box into every
  rank's buffer (fused), the GEMM in row chunks with the copy engines pushing finished chunks to the peers (push),
  or a local GEMM + ncclAllGather + relayout (nccl).
* Query-sharded attention: rank r owns query rows row_range(S, world, r); K and V rows are gathered from all ranks
  (h3q_comm_allgather) and each rank attends its queries against every key (h3q_attention_rows).  Its rows equal
  the single-GPU result's (per-token scales).

On GPUs the data plane is the library's: a Comm is an NCCL communicator created through the C ABI
(h3q_comm_init), its id handed around over torch.distributed.  torch.distributed also carries the host-side
set-up (ids, IPC handles) and, in the CPU tests, the gloo collectives; the operators are parameters, so the host
logic is exercised on CPU with the oracle.
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


NSPLIT_FUSED, NSPLIT_PUSH, NSPLIT_NCCL, NSPLIT_PEER = 0, 1, 2, 3
NSPLIT_MODES = {"fused": NSPLIT_FUSED, "push": NSPLIT_PUSH, "nccl": NSPLIT_NCCL, "peer": NSPLIT_PEER}


class Comm:
    """An h3q communicator (NCCL, created by h3q_comm_init through the C ABI) over the ranks of a torch.distributed
    group, on `device`.  Rank 0 of the group makes the id; torch.distributed hands it to the others."""

    def __init__(self, device, group=None):
        import torch
        dist = _dist()
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.device = torch.device(device)
        idb = (ctypes.c_uint8 * 128)()
        if self.rank == 0:
            check(lib().h3q_comm_unique_id(idb))
        obj = [bytes(idb) if self.rank == 0 else None]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(obj, src=src, group=group, device=self.device)
        idb = (ctypes.c_uint8 * 128).from_buffer_copy(obj[0])
        self.ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib().h3q_comm_init(self.world, self.rank, idb, ctypes.byref(self.ptr)))

    def allgather(self, send, recv) -> None:
        """recv (world x send's bytes, rank order) = every rank's send; on the current stream."""
        nbytes = send.numel() * send.element_size()
        if recv.numel() * recv.element_size() != self.world * nbytes:
            raise ValueError("Comm.allgather: recv must hold world x send bytes")
        check(lib().h3q_comm_allgather(self.ptr, _p(send), _p(recv), nbytes, _stream(self.device)))

    def barrier(self) -> None:
        check(lib().h3q_comm_barrier(self.ptr, _stream(self.device)))

    def close(self) -> None:
        if self.ptr:
            import torch
            torch.cuda.synchronize(self.device)
            check(lib().h3q_comm_destroy(self.ptr))
            self.ptr = None


class NSplitLinear:
    """attn8::gemm_s8 (linear epilogue, bf16 out) with the weight rows split over the ranks.  Every rank passes the
    full activation x [M, K] and receives the full output [M, N]; rank r computes the columns nsplit_range(N, g, r)
    and h3q_gemm_s8_nsplit all-gathers them in the chosen form:

      "fused"  one GEMM per rank whose epilogue stores every output box into every rank's buffer (peer memory over
               NVLink), so the transfer runs inside the GEMM;
      "push"   the GEMM in row chunks into this rank's buffer, the copy engines pushing each finished chunk into
               the peers' buffers while the next chunk computes;
      "nccl"   local GEMM, ncclAllGather of the column blocks, relayout kernel;
      "peer"   the GEMM into this rank's buffer, then a kernel on every SM storing the column block into every
               peer's buffer.

    mode=None picks the form measured fastest on B200 for the four c1 linears (M = 32760, default_mode): "push" up
    to 2 ranks (2 GPUs: 4.13 ms against 4.47 fused and 7.02 nccl), "peer" up to 4 (4 GPUs: 4.97 ms against 5.98
    fused, 6.52 nccl and 6.62 push; the SM stores deliver ~0.7 TB/s per GPU there), "nccl" beyond (8 GPUs: 7.17 ms
    against 7.53 peer and 9.82 push: with every GPU sending to seven, stores and copies deliver ~0.4 TB/s per GPU
    and NCCL's all-gather ~0.6).
    shard_quant=True quantizes only this rank's row_range of x and all-gathers the int8 codes and row scales
    (M K + 4 M bytes over NVLink) instead of every rank quantizing all rows (needs M % world == 0).
    """

    @staticmethod
    def default_mode(world: int) -> str:
        return "push" if world <= 2 else "peer" if world <= 4 else "nccl"

    def __init__(self, w, ws, bias, comm: Comm, mode: str | None = None, rotate: bool = True,
                 shard_quant: bool = False, group=None):
        import torch
        self.comm, self.group = comm, group
        self.world, self.rank = comm.world, comm.rank
        self.n = w.shape[0]
        self.n0, self.n1 = nsplit_range(self.n, self.world, self.rank)
        self.w = w[self.n0:self.n1].contiguous()
        ws = ws.to(torch.float32).reshape(-1)
        self.ws = (ws[self.n0:self.n1] if ws.numel() == self.n and self.n > 1 else ws[:1]).contiguous()
        self.bias = None if bias is None else bias.to(torch.float32)[self.n0:self.n1].contiguous()
        mode = mode or self.default_mode(self.world)
        if mode not in NSPLIT_MODES:
            raise ValueError(f"NSplitLinear: unknown mode {mode!r}")
        self.mode = mode
        self.rotate = rotate
        self.shard_quant = shard_quant
        self.bufs = None
        self.out = None
        self.ws_buf = None

    def _outputs(self, m: int, device):
        import torch
        if self.mode == "nccl":
            if self.out is None or self.out.shape[0] != m:
                self.out = torch.empty((m, self.n), dtype=torch.bfloat16, device=device)
                nb = lib().h3q_gemm_s8_nsplit_workspace_size(m, self.n, self.world, NSPLIT_NCCL)
                self.ws_buf = torch.empty(max(nb, 1), dtype=torch.uint8, device=device)
            ptrs = [None] * self.world
            ptrs[self.rank] = self.out.data_ptr()
            return self.out, ptrs
        if self.bufs is None or self.bufs.rows != m:
            if self.bufs is not None:
                self.bufs.close()
            self.bufs = PeerBuffers(m, self.n, device, self.group)
        return self.bufs.local, self.bufs.ptrs

    def quantize(self, x):
        """(codes [M, K], scales [M]) of x on every rank: computed whole, or per row block and all-gathered."""
        import torch
        m, k = x.shape
        if not self.shard_quant or self.world == 1 or m % self.world:
            return _quant_rows(x, self.rotate)
        lo, hi = row_range(m, self.world, self.rank)
        ql, sl = _quant_rows(x[lo:hi], self.rotate)
        q = torch.empty((m, k), dtype=torch.int8, device=x.device)
        s = torch.empty(m, dtype=torch.float32, device=x.device)
        self.comm.allgather(ql, q)
        self.comm.allgather(sl, s)
        return q, s

    def forward(self, x, quantized=None):
        import torch
        q, xs = quantized if quantized is not None else self.quantize(x)
        m, k = q.shape
        out, ptrs = self._outputs(m, x.device)
        outs = (ctypes.c_void_p * self.world)(*ptrs)
        wsp = self.ws_buf if self.mode == "nccl" else None
        check(lib().h3q_gemm_s8_nsplit(self.comm.ptr, NSPLIT_MODES[self.mode], _p(q), _p(xs), _p(self.w),
                                       _p(self.ws), self.ws.numel(), _p(self.bias), outs, m, self.n, k, _p(wsp),
                                       0 if wsp is None else wsp.numel(), _stream(x.device)))
        return out

    def close(self) -> None:
        if self.bufs is not None:
            self.bufs.close()
            self.bufs = None
        self.out = self.ws_buf = None


def gather_full(local, total: int, group=None, comm: Comm | None = None):
    """gather_rows without the staging copies when every rank holds the same number of rows (total divisible by
    the world size): one all-gather straight into the full [total, ...] tensor, rank blocks in rank order; through
    the library's communicator when `comm` is given, else torch.distributed."""
    dist = _dist()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if total % world != 0:
        return gather_rows(local, total, group)
    lo, hi = row_range(total, world, rank)
    if local.shape[0] != hi - lo:
        raise ValueError(f"gather_full: rank {rank} holds {local.shape[0]} rows, expected {(lo, hi)}")
    out = local.new_empty((total,) + tuple(local.shape[1:]))
    if comm is not None:
        comm.allgather(local.contiguous(), out)
    else:
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def sharded_attention(q_local, k_local, v_local, total: int, group=None, flags: int = 0, rows_op=None,
                      comm: Comm | None = None):
    """Query-sharded attention: this rank's rows q_local, k_local, v_local ([s_r, H, 128], row_range order) ->
    its output rows [s_r, H, 128], attending over the keys and values of every rank.  K and V are each gathered
    straight into full tensors (gather_full, through `comm` when given).  rows_op(q, k, v, flags) defaults to
    h3q.attention_rows."""
    k_full = gather_full(k_local, total, group, comm)
    v_full = gather_full(v_local, total, group, comm)
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
           "Comm", "NSPLIT_MODES",
           "sharded_attention", "H3QError", "RankMonitor", "RankLeft", "RankLost", "JobCancelled"]
