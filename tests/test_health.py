"""Failure detection on the host (gloo ranks on CPU): a rank that stops heartbeating is named by its peer, a clean
exit is told apart, a non-finite value on one rank makes every rank reject the step, and the hang watch dumps the
stacks of a phase that overruns."""
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from arc_forge_2026_b200.parallel.health import Heartbeat, PeerLost, finite_or_raise
from arc_forge_2026_b200.utils.hang_watch import HangWatch
from arc_forge_2026_b200.utils.timing import Sections


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=30))
    dist.init_process_group("gloo", rank=rank, world_size=world, store=dist.PrefixStore("pg", store))
    hb = Heartbeat(store, rank, world, period_s=0.1, timeout_s=1.0)
    # all-rank rejection: rank 1 holds a NaN
    g = torch.tensor([1.0, float("nan") if rank == 1 else 2.0])
    try:
        finite_or_raise([g])
        rejected = False
    except FloatingPointError:
        rejected = True
    hb.check()  # everyone alive
    dist.barrier()
    if rank == 1:  # dies without a clean stop: heartbeats end, no tombstone
        q.put((rank, rejected, None))
        hb._stop.set()
        time.sleep(4)
        os._exit(0)
    deadline, lost = time.time() + 10, None
    while time.time() < deadline:
        try:
            hb.check()
        except PeerLost as e:
            lost = e.ranks
            break
        time.sleep(0.1)
    q.put((rank, rejected, lost))
    hb.stop()
    os._exit(0)


def test_heartbeat_names_a_silent_rank_and_rejection_is_collective():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        r, rejected, lost = q.get(timeout=60)
        res[r] = (rejected, lost)
    for p in ps:
        p.join(timeout=30)
    assert res[0][0] and res[1][0]          # both ranks rejected the step
    assert res[0][1] == [1]                 # rank 0 named the silent rank


def test_hang_watch_dumps_overrunning_phase(tmp_path):
    w = HangWatch(str(tmp_path), limit_s=0.3, poll_s=0.05, rank=0)
    with w.phase("stuck_collective", step=7):
        time.sleep(1.0)
    with w.phase("fast"):
        pass
    time.sleep(0.2)
    w.close()
    assert len(w.dumps) == 1
    text = open(w.dumps[0]).read()
    assert "stuck_collective" in text and "step" in text and "test_hang_watch_dumps_overrunning_phase" in text


def test_sections_accumulate():
    s = Sections()
    for _ in range(3):
        with s.section("a"):
            sum(range(1000))
    r = s.report()
    assert r["a"]["calls"] == 3 and r["a"]["ms"] >= 0


def _ep_worker(rank, world, port, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from arc_forge_2026_b200.parallel.ep import ExpertParallel
    try:  # rank 1 asks for a different capacity: both ranks must refuse before any device memory is touched
        ExpertParallel(world, rank, 80 if rank == 0 else 70, 256, 2, 8, "cpu")
        q.put((rank, "built"))
    except ValueError as e:
        q.put((rank, "refused" if "differ across ranks" in str(e) else f"other: {e}"))
    dist.destroy_process_group()


def test_expert_parallel_refuses_mismatched_shapes():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_ep_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(world))
    for p in ps:
        p.join(timeout=30)
    assert res == {0: "refused", 1: "refused"}


def _host_check_worker(rank, world, port, out):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from arc_forge_2026_b200.parallel.guard import host_check
    host_check([1, 2, 3])
    try:
        host_check([1, 2, rank])
        ok = False
    except RuntimeError:
        ok = True
    with open(f"{out}.{rank}", "w") as f:
        f.write("1" if ok else "0")
    dist.destroy_process_group()


def test_host_replica_check_raises_on_every_rank(tmp_path):
    import os
    import torch.multiprocessing as mp
    port = 29700 + os.getpid() % 200
    mp.spawn(_host_check_worker, args=(2, port, str(tmp_path / "r")), nprocs=2, join=True)
    assert (tmp_path / "r.0").read_text() == "1" and (tmp_path / "r.1").read_text() == "1"
