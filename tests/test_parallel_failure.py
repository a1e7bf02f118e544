"""Host-side failure detection of a multi-rank job (h3q.parallel.RankMonitor) on CPU: three gloo ranks in child
processes run steps of a collective, and one of them stops between steps.  No GPU is involved.

Scenarios (the survivors must end with the named error, not hang):
  leave    rank 2 announces that it leaves after step 1            -> RankLeft at the survivors' ready(2)
  vanish   rank 2 exits after step 1 without a word                -> RankLost at ready(2), after the time limit
  cancel   rank 0 cancels the job after step 1 (progress::cancel_all) -> JobCancelled at every rank's ready(2)
  collect  survivors skip the check and start step 2's collective  -> the process group's short timeout raises
"""
import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

from h3q import parallel as P

WORLD = 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _step(dist, step: int) -> None:
    t = torch.full((4,), float(step))
    dist.all_reduce(t)
    assert torch.equal(t, torch.full((4,), float(step * WORLD)))


def _report(results, item) -> None:
    results.put(item)
    results.close()
    results.join_thread()  # the item reaches the parent before os._exit ends this process


def _finish(store, rank: int) -> None:
    """Rank 0 hosts the store: it stays until every rank has reported, so no survivor loses the store early."""
    store.add("test/finished", 1)
    if rank == 0:
        deadline = time.monotonic() + 30.0
        while int(store.add("test/finished", 0)) < WORLD and time.monotonic() < deadline:
            time.sleep(0.02)


def _worker(rank: int, port: int, scenario: str, results):
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", port, WORLD, rank == 0, timeout=timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=WORLD, timeout=timedelta(seconds=3))
    mon = P.RankMonitor(store, rank, WORLD, timeout=2.0)
    outcome = "finished"
    t0 = time.monotonic()
    try:
        for step in range(4):
            if scenario != "collect" or step < 2:
                mon.ready(step)
            _step(dist, step)
            if step == 1 and rank == 2 and scenario == "leave":
                mon.leave("finished its share early")
                outcome = "left"
                break
            if step == 1 and rank == 2 and scenario in ("vanish", "collect"):
                _report(results, (rank, "vanished", 0.0))
                _finish(store, rank)
                os._exit(0)  # gone between steps, without a word
            if step == 1 and rank == 0 and scenario == "cancel":
                mon.cancel_all()
    except P.RankLeft as e:
        outcome = f"RankLeft:{e.rank}"
    except P.RankLost as e:
        outcome = f"RankLost:{e.ranks}"
    except P.JobCancelled:
        outcome = "JobCancelled"
    except RuntimeError as e:  # gloo's own timeout / closed connection in the collective
        outcome = f"collective:{type(e).__name__}"
    _report(results, (rank, outcome, time.monotonic() - t0))
    _finish(store, rank)
    # the survivors' process group may be unusable now; leave without a collective
    os._exit(0)


def _run(scenario: str) -> dict:
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, scenario, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = {}
    while not results.empty():
        r, outcome, secs = results.get()
        out[r] = (outcome, secs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return out


def test_rank_leaves_between_steps():
    out = _run("leave")
    assert out[2][0] == "left"
    for r in (0, 1):
        assert out[r][0] == "RankLeft:2", out
        assert out[r][1] < 10.0


def test_rank_vanishes_between_steps():
    out = _run("vanish")
    assert out[2][0] == "vanished"
    for r in (0, 1):
        assert out[r][0] == "RankLost:[2]", out


def test_job_cancelled_between_steps():
    out = _run("cancel")
    for r in range(WORLD):
        assert out[r][0] == "JobCancelled", out


def test_collective_without_check_times_out():
    out = _run("collect")
    for r in (0, 1):
        assert out[r][0].startswith("collective:"), out
        assert out[r][1] < 60.0
