"""Host-side failure detection between multi-GPU decode steps
(tqkv.health.StepMonitor), on CPU ranks sharing a TCPStore: healthy ranks
step together; a rank that silently stops is reported by the others after the
deadline; a rank that fails with an exception is reported at once.  No GPU is
touched: the failures are made on the host."""
import datetime
import os
import socket
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STEPS = 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, deadline, out):
    import sys
    sys.path.insert(0, os.path.join(REPO, "parallel-final-project_b200"))
    from tqkv.health import PeerFailure, StepMonitor
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=30))
    mon = StepMonitor(store, rank, world, deadline_s=deadline)
    mon.start()   # set-up (process start) time does not count against the deadline
    result = ("ok", None, None, None, None)
    t_wait = time.monotonic()
    try:
        for step in range(STEPS):
            t_wait = time.monotonic()
            mon.wait_peers(step - 1)
            if scenario == "silent" and rank == world - 1 and step == 2:
                result = ("left", None, None, None, None)
                break                          # stops stepping without a word
            if scenario == "crash" and rank == 1 and step == 3:
                raise ValueError("injected host error")
            time.sleep(0.001 * (rank + 1))     # the step's work
            mon.finished(step)
    except PeerFailure as e:
        result = ("peer_failure", e.rank, e.last_step, time.monotonic() - t_wait, e.reason)
    except ValueError as e:
        mon.failed(f"{type(e).__name__}: {e}")
        result = ("raised", None, None, None, None)
    out.put((rank,) + result)
    # the store lives in rank 0: keep it up until every rank is through
    store.set(f"exit/{rank}", "1")
    if rank == 0:
        end = time.monotonic() + 20
        while time.monotonic() < end and not store.check([f"exit/{r}" for r in range(world)]):
            time.sleep(0.01)


def _run(world, scenario, deadline):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, deadline, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=60) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_healthy_ranks_step_together():
    res = _run(3, "healthy", deadline=10.0)
    assert [r[1] for r in res] == ["ok"] * 3


def test_silent_rank_is_reported_after_the_deadline():
    deadline = 2.0
    res = _run(3, "silent", deadline)
    assert res[2][1] == "left"
    for rank, kind, who, last, waited, reason in res[:2]:
        assert kind == "peer_failure", res
        assert who == 2 and last == 1 and reason is None   # rank 2 finished steps 0, 1 only
        assert deadline <= waited < deadline + 10


def test_crashed_rank_is_reported_at_once():
    deadline = 20.0
    res = _run(3, "crash", deadline)
    assert res[1][1] == "raised"
    for rank, kind, who, last, waited, reason in (res[0], res[2]):
        assert kind == "peer_failure", res
        assert who == 1 and last == 2 and reason == "ValueError: injected host error"
        assert waited < deadline / 4             # well before the deadline


def test_monitor_validates_rank():
    from tqkv.health import StepMonitor
    with pytest.raises(ValueError):
        StepMonitor(None, 3, 3)


def _start_worker(rank, world, port, out):
    import sys
    sys.path.insert(0, os.path.join(REPO, "parallel-final-project_b200"))
    from tqkv.health import PeerFailure, StepMonitor
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=30))
    mon = StepMonitor(store, rank, world)
    res = ("ok", None)
    if rank != world - 1:          # the last rank never starts
        try:
            # long enough that start-up skew between the two live ranks (a
            # loaded host can take a second or more to get a spawned child
            # past the store) is not taken for a missing rank
            mon.start(timeout_s=5.0)
        except PeerFailure as e:
            res = ("peer_failure", e.rank)
    out.put((rank,) + res)
    store.set(f"exit/{rank}", "1")
    if rank == 0:
        end = time.monotonic() + 20
        while time.monotonic() < end and not store.check([f"exit/{r}" for r in range(world)]):
            time.sleep(0.01)


def test_start_reports_a_rank_that_never_arrives():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_start_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=60) for _ in range(3))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1:] == ("peer_failure", 2) and res[1][1:] == ("peer_failure", 2)
    assert res[2][1:] == ("ok", None)
