"""Failure detection on the host, with CPU ranks (gloo), no GPU.

Two worker processes share a TCPStore.  Worker 1 beats, then dies between
steps (os._exit, no clean departure).  Worker 0 checks worker 1's heartbeat
before each step's launch and must refuse the first launch after the death
becomes visible; a gloo collective with a short timeout must also fail
instead of hanging.  A clean departure is seen at once.
"""

import os
import time

import pytest
import torch.multiprocessing as mp


def _worker(rank, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    from aegaeon_b200.liveness import Heartbeat, PeerGone

    store = dist.TCPStore("127.0.0.1", port, 2, rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=3))
    hb = Heartbeat(store, rank, interval=0.05)
    dist.barrier()
    if rank == 1:
        for _ in range(5):
            dist.barrier()  # five steps in lock-step with worker 0
        os._exit(0)  # dies between steps: no departure key, no more beats
    launches, refused = 0, None
    for step in range(200):
        try:
            hb.check(1, max_age=0.5)
        except PeerGone as e:
            refused = (step, str(e))
            break
        launches += 1  # stands for queuing a copy that reads the peer's memory
        if step < 5:
            dist.barrier()
        else:
            time.sleep(0.05)
    collective_failed = False
    try:
        t = torch.ones(1)
        dist.all_reduce(t)
    except Exception:  # noqa: BLE001 - the expected timeout / connection error
        collective_failed = True
    q.put({"launches": launches, "refused": refused, "collective_failed": collective_failed})
    q.close()
    q.join_thread()  # flush before leaving without tearing down the broken group
    os._exit(0)


def test_dead_peer_is_detected_before_next_launch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res["refused"] is not None, res
    step, msg = res["refused"]
    assert step >= 5 and "silent" in msg
    # beats every 50 ms, limit 500 ms, steps every 50 ms after the death
    assert res["launches"] <= 5 + 20
    assert res["collective_failed"]


def test_clean_departure_is_seen_immediately():
    import datetime

    import torch.distributed as dist

    from aegaeon_b200.liveness import Heartbeat, PeerGone

    store = dist.HashStore()
    a = Heartbeat(store, 0, interval=0.05)
    b = Heartbeat(store, 1, interval=0.05)
    a.check(1)
    b.depart()
    with pytest.raises(PeerGone, match="left"):
        a.check(1)
    with pytest.raises(PeerGone, match="never"):
        a.check(7)
    a.stop()
    del datetime
