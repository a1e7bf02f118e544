"""Multi-GPU parity of h3q.parallel (one NCCL rank per GPU in child processes, 2 to 8 GPUs; skipped with fewer than
two): the N-split linear through the C ABI (h3q_gemm_s8_nsplit) in its four forms (fused: every rank's column
block stored into every rank's output by the GEMM; push: row chunks forwarded by the copy engines; nccl:
ncclAllGather + relayout; peer: a kernel on every SM storing the block into the peers), with the activations quantized whole or per row block and all-gathered, the library's
byte all-gather, and query-sharded attention, each bit-identical to the single-GPU result."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, errors):
    import torch.distributed as dist
    import h3q
    from h3q import parallel as P
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    lin = None
    comm = None
    try:
        comm = P.Comm(dev)
        assert (comm.world, comm.rank) == (world, rank)
        # the library's byte all-gather
        mine = torch.full((3, 5), rank, dtype=torch.int32, device=dev)
        allr = torch.empty((world * 3, 5), dtype=torch.int32, device=dev)
        comm.allgather(mine, allr)
        assert torch.equal(allr, torch.arange(world, device=dev, dtype=torch.int32).repeat_interleave(3)[:, None]
                           .expand(world * 3, 5))
        g = torch.Generator(device=dev).manual_seed(5)  # same seed: every rank builds the same full tensors
        K, N = 5120, 15360
        w = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
        ws = torch.rand(N, generator=g, device=dev) * 9e-3 + 1e-3
        b = (torch.randn(N, generator=g, device=dev) * 0.02).float()
        for M in (1000, 1003):
            x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
            want = h3q.gemm_s8(x, w, ws, b, swiglu=False, rotate=True)
            for mode in ("fused", "push", "nccl", "peer"):
                for shard in (False, True):
                    lin = P.NSplitLinear(w, ws, b, comm, mode=mode, shard_quant=shard)
                    for _ in range(2):  # twice: the output buffers are reused
                        y = lin.forward(x)
                        torch.cuda.synchronize()
                        assert torch.equal(y.view(torch.int16), want.view(torch.int16)), (M, mode, shard)
                    lin.close()
                    lin = None
        S, H = 1000, 2
        q = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
        full = h3q.attention(q, k, v)
        lo, hi = P.row_range(S, world, rank)
        for c in (None, comm):
            out = P.sharded_attention(q[lo:hi].contiguous(), k[lo:hi].contiguous(), v[lo:hi].contiguous(), S,
                                      comm=c)
            assert torch.equal(out.view(torch.int16), full[lo:hi].view(torch.int16))
        assert h3q.device_status(rank) == 0
        dist.barrier()
    except Exception as e:
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        if lin is not None:
            lin.close()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_multi_gpu_nsplit_and_sharded_attention():
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errors)) for r in range(world)]
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
