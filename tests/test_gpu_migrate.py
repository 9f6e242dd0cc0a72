"""GPU->GPU block migration (the reference's unimplemented migrate_blocks,
worker.py:2420-2451): same-GPU copies through both kernels, and, with two
GPUs, pull and push over IPC-mapped peer memory."""

import os
import time

import numpy as np
import pytest
import torch

from aegaeon_b200 import _lib, swapper

pytestmark = pytest.mark.gpu


def cache_pages(device, layers, blocks, page, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    return [torch.randint(0, 255, (blocks * page,), generator=g, dtype=torch.uint8,
                          device=device) for _ in range(layers)]


def make(device, pages_per_seg, seg_tensors):
    segments, _ = swapper.make_segments(
        [((f"l{i}",), t.numel()) for i, t in enumerate(seg_tensors)],
        seg_tensors[0].numel() // pages_per_seg)
    return swapper.KVSwapper(device, segments, seg_tensors, [frozenset({0})] * len(seg_tensors), [1])


def expected_after(src_pages, dst_pages, src_ids, dst_ids, page):
    exp = [d.cpu().numpy().copy() for d in dst_pages]
    for s, d in zip(src_pages, exp):
        sv = s.cpu().numpy()
        for a, b in zip(src_ids, dst_ids):
            d[b * page:(b + 1) * page] = sv[a * page:(a + 1) * page]
    return exp


@pytest.mark.parametrize("mode", ["sm", "sm_bulk", "ce"])
def test_same_gpu_migration(cuda, mode):
    page, blocks, layers = 16384, 256, 6
    src = cache_pages(cuda, layers, blocks, page, 1)
    dst = cache_pages(cuda, layers, blocks, page, 2)
    a, b = make(0, page, src), make(0, page, dst)
    g = torch.Generator().manual_seed(3)
    sid = torch.randperm(blocks, generator=g)[:150].tolist()
    did = torch.randperm(blocks, generator=g)[:150].tolist()
    exp = expected_after(src, dst, sid, did, page)
    n = len(sid)
    s_ep, t_ep = a.local_endpoint(), b.local_endpoint()
    stream = torch.cuda.current_stream()
    import ctypes
    arr = swapper._entry_arrays(sid, did, [0] * n, [0] * n, [1] * n)
    _lib.check(_lib.lib().kvx_migrate_blocks(s_ep.handle, t_ep.handle, *arr, _lib.mode_of(mode),
                                             stream.cuda_stream, None, None))
    torch.cuda.synchronize()
    assert _lib.last_mode_name() == {"ce": "ce_extent"}.get(mode, mode)
    for d, e in zip(dst, exp):
        assert np.array_equal(d.cpu().numpy(), e)
    assert _lib.device_status(0) == 0
    a.close()
    b.close()


@pytest.mark.parametrize("mode", ["sm", "sm_bulk"])
def test_copy_blocks_local_overlapping_ids(cuda, mode):
    """Source and target ids overlap inside one cache: bytes equal a
    sequential in-order loop (the planner splits conflicting copies into
    ordered waves)."""
    page, blocks = 32768, 16
    pages = cache_pages(cuda, 2, blocks, page, 4)
    sw = make(0, page, pages)
    src_ids, dst_ids = [0, 1, 2, 3, 4], [1, 2, 3, 4, 5]
    exp = [p.cpu().numpy().copy() for p in pages]
    for e in exp:
        for a, b in zip(src_ids, dst_ids):
            e[b * page:(b + 1) * page] = e[a * page:(a + 1) * page]
    sw.copy_blocks_local(src_ids, dst_ids, mode=mode).synchronize()
    for p, e in zip(pages, exp):
        assert np.array_equal(p.cpu().numpy(), e)
    sw.close()


def plan_ids(blocks, whole):
    """The migrated ids: every block of every segment in order (whole), or
    200 random blocks to 200 random places."""
    if whole:
        return list(range(blocks)), list(range(blocks))
    g = torch.Generator().manual_seed(5)
    return (torch.randperm(blocks, generator=g)[:200].tolist(),
            torch.randperm(blocks, generator=g)[:200].tolist())


def _peer_worker(rank, world, q_out, q_in, page, blocks, layers, direction, mode="auto",
                 whole=False):
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    pages = cache_pages(dev, layers, blocks, page, 100 + rank)
    sw = make(rank, page, pages)
    sid, did = plan_ids(blocks, whole)
    q_out.put(("handles", rank, sw.export_kvcache_mem_handles()))
    _, peer, handles = q_in.get(timeout=120)
    torch.cuda.synchronize()
    if rank == 1:  # the decode side: register prefill's cache and pull
        sw.register_kvcache_mem_handles(0, None, handles)
        src_snapshot = None
        if direction == "pull":
            ev = sw.migrate_blocks([1], 0, sid, did, [None], direction="pull", mode=mode)
            ev.synchronize()
        q_out.put(("done", rank, None))
    else:
        sw.register_kvcache_mem_handles(1, None, handles)
        if direction == "push":
            sw.migrate_blocks([1], 1, sid, did, [None], direction="push",
                              mode=mode).synchronize()
        q_out.put(("done", rank, None))
    q_in.get(timeout=120)  # both finished
    out = [p.cpu().numpy().tobytes() for p in pages] if rank == 1 else None
    q_out.put(("pages", rank, out))
    q_in.get(timeout=120)
    sw.close()


@pytest.mark.multigpu
@pytest.mark.parametrize("direction,mode,whole,blocks", [
    ("pull", "auto", False, 512), ("push", "auto", False, 512),
    # every block of every segment: the copy-engine form must not merge copies
    # across two segments' allocations, even where they sit next to each other
    ("pull", "ce_extent", True, 4096), ("push", "ce_extent", True, 4096),
    ("pull", "sm_bulk", True, 4096), ("push", "sm_bulk", False, 512)])
def test_two_gpu_migration(cuda, direction, mode, whole, blocks):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    page, layers = 16384, 4
    q0, q1, qa, qb = ctx.Queue(), ctx.Queue(), ctx.Queue(), ctx.Queue()
    args = (page, blocks, layers, direction, mode, whole)
    procs = [ctx.Process(target=_peer_worker, args=(0, 2, q0, qa) + args),
             ctx.Process(target=_peer_worker, args=(1, 2, q1, qb) + args)]
    for p in procs:
        p.start()
    try:
        h0 = q0.get(timeout=180)
        h1 = q1.get(timeout=180)
        qa.put(h1)
        qb.put(h0)
        assert q0.get(timeout=180)[0] == "done"
        assert q1.get(timeout=180)[0] == "done"
        qa.put("go")
        qb.put("go")
        q0.get(timeout=180)
        got = q1.get(timeout=180)[2]
        qa.put("end")
        qb.put("end")
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    # expected: rank 1's pages with rank 0's selected blocks copied in
    src = cache_pages(torch.device("cuda", 0), layers, blocks, page, 100)
    dst = cache_pages(torch.device("cuda", 1), layers, blocks, page, 101)
    sid, did = plan_ids(blocks, whole)
    exp = expected_after(src, dst, sid, did, page)
    for e, b in zip(exp, got):
        assert e.tobytes() == b
    assert all(p.exitcode == 0 for p in procs)


def _liveness_worker(rank, port, q_out, q_in, page, blocks, layers):
    """rank 0 = prefill (exports, beats, departs between steps);
    rank 1 = decode (pulls while rank 0 is there, then must refuse)."""
    import datetime

    import torch.distributed as dist

    from aegaeon_b200.liveness import Heartbeat, PeerGone

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    store = dist.TCPStore("127.0.0.1", port, 2, rank == 1, timeout=datetime.timedelta(seconds=60))
    hb = Heartbeat(store, rank, interval=0.05)
    pages = cache_pages(dev, layers, blocks, page, 200 + rank)
    sw = make(rank, page, pages)
    q_out.put(("handles", sw.export_kvcache_mem_handles()))
    if rank == 0:
        q_in.get(timeout=120)  # the decode side finished its pull: leave now
        torch.cuda.synchronize()
        hb.depart()            # announced before the memory goes away
        q_out.put(("left", None))
        q_out.close()
        q_out.join_thread()
        os._exit(0)
    handles = q_in.get(timeout=120)[1]
    sw.register_kvcache_mem_handles(0, None, handles)
    sid, did = list(range(64)), list(range(64, 128))
    sw.migrate_blocks([0], 0, sid, did, None, liveness=hb.guard(0, max_age=2.0)).synchronize()
    expect = cache_pages(torch.device("cuda", 0), 1, blocks, page, 200)[0].view(-1, page)[0:64]
    ok_first = torch.equal(pages[0].view(-1, page)[64:128].cpu(), expect.cpu())
    sw.unregister_kvcache_mem_handles(0)  # unmap the peer before it may go away
    q_out.put(("first", ok_first))
    q_in.get(timeout=120)  # the prefill process has departed and exited
    refused = None
    try:
        sw.migrate_blocks([0], 0, sid, did, None, liveness=hb.guard(0, max_age=2.0))
    except PeerGone as e:
        refused = str(e)
    q_out.put(("refused", refused))
    q_out.close()
    q_out.join_thread()
    os._exit(0)


@pytest.mark.multigpu
def test_departed_prefill_peer_is_never_read(cuda):
    """The decode worker checks the prefill worker's liveness before each
    pull.  Once the prefill process has departed (between steps, nothing in
    flight) the next pull is refused on the host: nothing reads the departed
    peer's memory.  (Silent deaths, found by heartbeat age, are tested on CPU
    ranks in test_liveness_gloo.py.)"""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q0, q1, qa, qb = ctx.Queue(), ctx.Queue(), ctx.Queue(), ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_liveness_worker, args=(0, port, q0, qa, 16384, 256, 2)),
             ctx.Process(target=_liveness_worker, args=(1, port, q1, qb, 16384, 256, 2))]
    for p in procs:
        p.start()
    try:
        h0 = q0.get(timeout=180)
        q1.get(timeout=180)
        qb.put(h0)
        first = q1.get(timeout=180)
        qa.put("leave")
        assert q0.get(timeout=180)[0] == "left"
        procs[0].join(timeout=120)
        assert not procs[0].is_alive()
        qb.put("go")
        refused = q1.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert first == ("first", True)
    assert refused[0] == "refused" and refused[1] is not None and "left" in refused[1]


def _ipc_event_worker(rank, q_out, q_in):
    """rank 0 swaps host data into its cache and ships the (device, handle)
    of the swap's interprocess event at once; rank 1 pulls those blocks after
    waiting on that event."""
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    page, blocks, layers = 262144, 256, 8
    pages = [torch.zeros(blocks * page, dtype=torch.uint8, device=dev) for _ in range(layers)]
    segs, comp = swapper.make_segments([((f"l{i}",), blocks * page) for i in range(layers)], blocks)
    pool = torch.full((blocks * comp,), 0x5A, dtype=torch.uint8).pin_memory() if rank == 0 else None
    sw = swapper.KVSwapper(rank, segs, pages, [frozenset({0})] * layers, [1], kv_swap=pool)
    q_out.put(("handles", sw.export_kvcache_mem_handles()))
    if rank == 0:
        q_in.get(timeout=120)
        ids = list(range(blocks))
        handle = sw.swap_blocks([1], ids, ids, [0] * blocks, [0] * blocks, [1] * blocks, [None],
                                True, return_handle=True)
        q_out.put(("event", handle))  # before the swap-in has finished
        q_in.get(timeout=120)
        torch.cuda.synchronize()
        q_out.put(("bye", None))
        q_out.close()
        q_out.join_thread()
        os._exit(0)
    handles = q_in.get(timeout=120)[1]
    sw.register_kvcache_mem_handles(0, None, handles)
    handle = q_in.get(timeout=120)[1]
    ids = list(range(blocks))
    sw.migrate_blocks([1], 0, ids, ids, [handle]).synchronize()
    ok = all(bool((p == 0x5A).all()) for p in pages)
    sw.unregister_kvcache_mem_handles(0)
    q_out.put(("result", ok))
    q_out.close()
    q_out.join_thread()
    os._exit(0)


@pytest.mark.multigpu
def test_pull_waits_on_producer_ipc_event(cuda):
    """Cross-process ordering with the native event layer: the decode worker
    pulls blocks the prefill worker is still swapping in, after waiting on
    the prefill swap's interprocess event (the reference's reduce/rebuild
    handle format); it must see the swapped-in bytes."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q0, q1, qa, qb = ctx.Queue(), ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_ipc_event_worker, args=(0, q0, qa)),
             ctx.Process(target=_ipc_event_worker, args=(1, q1, qb))]
    for p in procs:
        p.start()
    try:
        h0 = q0.get(timeout=180)
        q1.get(timeout=180)
        qb.put(h0)
        qa.put("go")
        ev = q0.get(timeout=180)
        qb.put(ev)
        result = q1.get(timeout=180)
        qa.put("done")
        assert q0.get(timeout=180)[0] == "bye"
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert result == ("result", True)
