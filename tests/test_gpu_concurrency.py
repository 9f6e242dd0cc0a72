"""Concurrent callers and overrun guards.

* Several host threads, each with its own CUDA stream, swap disjoint blocks
  through one shared KVSwapper at once, in different transfer modes.  This
  exercises the per-device lock, the descriptor ring's event-guarded reuse and
  the per-direction staging areas shared by calls on different streams.
* Guard bytes around every copied extent stay untouched in every mode,
  including partial extents.
"""

import threading

import numpy as np
import pytest
import torch

from aegaeon_b200 import _lib, swapper

pytestmark = pytest.mark.gpu


def make(cuda, layers=8, blocks=256, page=65536, rows=256):
    pages = [torch.randint(0, 255, (blocks * page,), dtype=torch.uint8, device=cuda)
             for _ in range(layers)]
    segs, comp = swapper.make_segments([((f"l{i}",), blocks * page) for i in range(layers)],
                                       blocks)
    pool = torch.zeros(rows * comp, dtype=torch.uint8).pin_memory()
    sw = swapper.KVSwapper(0, segs, pages, [frozenset({0})] * layers, [1], kv_swap=pool)
    return sw, pages, pool, comp


def test_threads_on_separate_streams(cuda):
    sw, pages, pool, comp = make(cuda)
    snapshot = [p.clone() for p in pages]
    torch.cuda.synchronize()  # setup ran on the default stream
    modes = ["ce", "sm", "auto", "ce_extent"]
    errors = []
    per = 256 // len(modes)

    def worker(k):
        try:
            stream = torch.cuda.Stream(cuda)
            ids = list(range(k * per, (k + 1) * per))
            rows = ids[::-1]
            for _ in range(5):
                ev = sw.swap_blocks([k], ids, rows, [0] * per, [0] * per, [1] * per, [None],
                                    False, mode=modes[k], stream=stream)
                with torch.cuda.stream(stream):  # wipe the blocks; swap-in restores them
                    for p in pages:
                        p.view(256, -1)[ids] = 0
                ev = sw.swap_blocks([k], rows, ids, [0] * per, [0] * per, [1] * per, [None],
                                    True, mode=modes[k], stream=stream)
                ev.synchronize()
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=worker, args=(k,)) for k in range(len(modes))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    torch.cuda.synchronize()
    for p, q in zip(pages, snapshot):
        assert torch.equal(p, q)
    # host rows hold every block once: row r = block (reversed within each thread's range)
    rows_view = pool.view(256, -1)
    for k in range(len(modes)):
        for b in (k * per, (k + 1) * per - 1):
            r = (k + 1) * per - 1 - (b - k * per)
            seg0 = rows_view[r, :65536]
            assert torch.equal(seg0.to(cuda), pages[0].view(256, -1)[b])
    assert _lib.device_status(0) == 0
    sw.close()


@pytest.mark.parametrize("mode", ["sm", "ce", "ce_extent", "auto"])
def test_guard_bytes_untouched(cuda, mode):
    """Partial extents (kernel blocks 1..2 of 4) of odd rows: everything else
    in the pool and in the cache keeps its guard pattern."""
    layers, blocks, page, rows = 4, 64, 65536, 64
    pages = [torch.full((blocks * page,), 0xEE, dtype=torch.uint8, device=cuda)
             for _ in range(layers)]
    segs, comp = swapper.make_segments([((f"l{i}",), blocks * page) for i in range(layers)],
                                       blocks)
    pool = torch.full((rows * comp,), 0xEE, dtype=torch.uint8).pin_memory()
    sw = swapper.KVSwapper(0, segs, pages, [frozenset({0})] * layers, [4], kv_swap=pool)
    ids = list(range(1, blocks, 2))
    n = len(ids)
    for p in pages:
        v = p.view(blocks, page)
        v[ids, page // 4: 3 * page // 4] = 0x11
    torch.cuda.synchronize()  # the swap runs on the swapper's own stream
    sw.swap_blocks([0], ids, ids, [0] * n, [1] * n, [2] * n, [None], False, mode=mode).synchronize()
    pv = pool.numpy().reshape(rows, layers, page)
    expect = np.full_like(pv, 0xEE)
    expect[ids, :, page // 4: 3 * page // 4] = 0x11
    assert np.array_equal(pv, expect)
    # back in, to other (even) blocks: only their middle halves change
    dst = list(range(0, blocks, 2))
    sw.swap_blocks([0], ids, dst, [0] * n, [1] * n, [2] * n, [None], True, mode=mode).synchronize()
    for p in pages:
        v = p.view(blocks, page).cpu().numpy()
        assert (v[dst, :page // 4] == 0xEE).all() and (v[dst, 3 * page // 4:] == 0xEE).all()
        assert (v[dst, page // 4: 3 * page // 4] == 0x11).all()
    sw.close()
