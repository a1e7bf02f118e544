"""The multi-GPU host logic of h3q.parallel on CPU: two gloo ranks (world size 2) in child processes, with the
oracle as each rank's operator.  Sharded results must equal the single-process oracle bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from h3q import parallel as P
from oracle import oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.numpy().astype(np.uint16)


def _worker(rank: int, world: int, port: int, errors):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # row blocks of uneven size
        x = torch.arange(7 * 3, dtype=torch.float32).reshape(7, 3)
        lo, hi = P.row_range(7, world, rank)
        assert torch.equal(P.gather_rows(x[lo:hi], 7), x)
        assert torch.equal(P.gather_full(x[lo:hi], 7), x)  # uneven blocks: falls back to gather_rows
        x8 = torch.arange(8 * 3, dtype=torch.float32).reshape(8, 3)
        lo8, hi8 = P.row_range(8, world, rank)
        assert torch.equal(P.gather_full(x8[lo8:hi8], 8), x8)  # even blocks: one all-gather into the result

        # N split: each rank's oracle linear on its weight rows, column blocks gathered = the full linear
        M, K, N = 40, 512, 600
        xb, w, ws, bias = O.make_linear_inputs(3, M, K, N)
        n0, n1 = P.nsplit_range(N, world, rank)
        y_local = O.gemm_s8(xb, w[n0:n1], ws[n0:n1], bias[n0:n1], False, True)[0]
        y = P.gather_columns(torch.from_numpy(y_local.astype(np.int32)), N)
        want = O.gemm_s8(xb, w, ws, bias, False, True)[0]
        np.testing.assert_array_equal(_bits(y), want)

        # query-sharded attention: each rank's rows against every key = those rows of the whole attention
        S, H = 300, 2
        q, k, v = O.make_attn_inputs(9, S, H, 3.0)
        lo, hi = P.row_range(S, world, rank)

        def rows_op(ql, kf, vf, flags):
            return torch.from_numpy(O.attention_rows(_bits(ql), _bits(kf), _bits(vf), flags).astype(np.int32))

        ti = lambda a: torch.from_numpy(a.astype(np.int32))
        out = P.sharded_attention(ti(q[lo:hi]), ti(k[lo:hi]), ti(v[lo:hi]), S, rows_op=rows_op)
        np.testing.assert_array_equal(_bits(out), O.attention(q, k, v)[lo:hi])
        # an odd token count: uneven row blocks
        S = 301
        q, k, v = O.make_attn_inputs(10, S, H, 3.0)
        lo, hi = P.row_range(S, world, rank)
        out = P.sharded_attention(ti(q[lo:hi]), ti(k[lo:hi]), ti(v[lo:hi]), S, rows_op=rows_op)
        np.testing.assert_array_equal(_bits(out), O.attention(q, k, v)[lo:hi])
        dist.barrier()
    except Exception as e:  # reported to the parent
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


def test_two_rank_host_logic():
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_ranges_cover_and_align():
    for n, g in ((15360, 8), (5120, 3), (600, 2), (100, 4)):
        ranges = [P.nsplit_range(n, g, r) for r in range(g)]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert all(lo % 256 == 0 for lo, _ in ranges)
    for m, g in ((32760, 8), (7, 2), (5, 8)):
        ranges = [P.row_range(m, g, r) for r in range(g)]
        assert ranges[0][0] == 0 and ranges[-1][1] == m
        assert max(hi - lo for lo, hi in ranges) - min(hi - lo for lo, hi in ranges) <= 1


def test_nsplit_default_form_by_world_size():
    """NSplitLinear's default form is the one measured fastest on B200 for the four c1 linears: the copy-engine
    push up to 2 ranks, the SM peer stores up to 4, NCCL's all-gather beyond; every default is a known form."""
    assert [P.NSplitLinear.default_mode(g) for g in (2, 3, 4, 5, 8)] == ["push", "peer", "peer", "nccl", "nccl"]
    assert all(P.NSplitLinear.default_mode(g) in P.NSPLIT_MODES for g in range(2, 17))
