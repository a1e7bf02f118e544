"""Multi-GPU parity of h3q.parallel (one NCCL rank per GPU in child processes, 2 to 8 GPUs; skipped with fewer than
two): the fused N-split GEMM (every rank's column block written into every rank's output over NVLink), the NCCL
all-gather form of it, and query-sharded attention, each bit-identical to the single-GPU result."""
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
    try:
        g = torch.Generator(device=dev).manual_seed(5)  # same seed: every rank builds the same full tensors
        M, K, N = 1000, 5120, 15360
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        w = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
        ws = torch.rand(N, generator=g, device=dev) * 9e-3 + 1e-3
        b = (torch.randn(N, generator=g, device=dev) * 0.02).float()
        want = h3q.gemm_s8(x, w, ws, b, swiglu=False, rotate=True)
        for fused in (True, False):
            lin = P.NSplitLinear(w, ws, b, fused=fused)
            for _ in range(2):  # twice: the peer buffers are reused
                y = lin.forward(x)
                assert torch.equal(y.view(torch.int16), want.view(torch.int16)), f"fused={fused}"
            lin.close()
            lin = None
        S, H = 1000, 2
        q = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
        full = h3q.attention(q, k, v)
        lo, hi = P.row_range(S, world, rank)
        out = P.sharded_attention(q[lo:hi].contiguous(), k[lo:hi].contiguous(), v[lo:hi].contiguous(), S)
        assert torch.equal(out.view(torch.int16), full[lo:hi].view(torch.int16))
        assert h3q.device_status(rank) == 0
        dist.barrier()
    except Exception as e:
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        if lin is not None:
            lin.close()
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
