"""Full-size checks of the benchmark configurations (size-independent properties).

At the sizes the benchmark moves, a byte-by-byte oracle comparison would take
minutes on the host, so these tests check properties that hold at any size:

* round trip: blocks swapped out and back in to other ids equal the originals
  (compared on the device);
* checksum of checksums: per-segment sums of the host rows written by a
  swap-out equal the sums of the device pages they came from.

The small-size tests compare against the oracle byte for byte.
"""

import pytest
import torch

from aegaeon_b200 import _lib, swapper, workloads

pytestmark = pytest.mark.gpu


def build(shape, num_blocks, rows, dev, seed=0):
    gen = torch.Generator(device=dev).manual_seed(seed)
    pages = []
    for _ in range(shape.num_segments):
        t = torch.empty(num_blocks * shape.page_bytes, dtype=torch.uint8, device=dev)
        workloads.fill_segment(t, shape, gen)
        pages.append(t)
    segs, comp = swapper.make_segments([((f"l{i}",), num_blocks * shape.page_bytes)
                                        for i in range(shape.num_segments)], num_blocks)
    pool = torch.empty(rows * comp, dtype=torch.uint8).pin_memory()
    sw = swapper.KVSwapper(dev.index, segs, pages, [frozenset({0})] * shape.num_segments, [1],
                           kv_swap=pool)
    return sw, pages, pool, comp


def page_view(t, shape):
    return t.view(-1, shape.page_bytes)


def test_cfg2_full_size_round_trip_and_checksums(cuda):
    sh = workloads.CFG2
    n = 1024
    sw, pages, pool, comp = build(sh, sh.num_blocks, n, cuda)
    out_ids, in_ids = workloads.swap_step_ids(sh.num_blocks, n, 0)
    rows = list(range(n))
    z, one = [0] * n, [1] * n
    sw.swap_blocks([0], out_ids, rows, z, z, one, [None], False).synchronize()
    assert sw.last_stats == (n * comp, n * sh.num_segments)
    # checksum of checksums: host rows (segment s at offset s*page) vs device pages
    rows_view = pool.view(n, sh.num_segments, sh.page_bytes)
    idx = torch.tensor(out_ids, device=cuda)
    for s in range(0, sh.num_segments, 7):
        dev_sum = page_view(pages[s], sh)[idx].view(torch.int32).sum(dtype=torch.int64).item()
        host_sum = rows_view[:, s].contiguous().view(torch.int32).sum(dtype=torch.int64).item()
        assert dev_sum == host_sum, s
    # round trip into other blocks
    sw.swap_blocks([0], rows, in_ids, z, z, one, [None], True).synchronize()
    idx_in = torch.tensor(in_ids, device=cuda)
    for s in range(sh.num_segments):
        pv = page_view(pages[s], sh)
        assert torch.equal(pv[idx_in], pv[idx]), s
    assert _lib.device_status(0) == 0
    sw.close()


def test_cfg5_fragmented_full_mapping_round_trip(cuda):
    """All 16,384 entries of the fragmented mapping (half in contiguous runs,
    half isolated), with 4 layers instead of 24 to keep host memory small."""
    import dataclasses

    sh = dataclasses.replace(workloads.CFG5, layers=4)
    n = 16384
    sw, pages, pool, comp = build(sh, sh.num_blocks, n, cuda, seed=5)
    ids, slots = workloads.fragmented_mapping(n, sh.num_blocks, seed=0)
    z, one = [0] * n, [1] * n
    snapshot = [p.clone() for p in pages]
    sw.swap_blocks([0], ids, slots, z, z, one, [None], False).synchronize()
    for p in pages:
        p.zero_()
    sw.swap_blocks([0], slots, ids, z, z, one, [None], True).synchronize()
    idx = torch.tensor(ids, device=cuda)
    for p, q in zip(pages, snapshot):
        assert torch.equal(page_view(p, sh)[idx], page_view(q, sh)[idx])
        # blocks outside the mapping stay zero
        mask = torch.ones(sh.num_blocks, dtype=torch.bool, device=cuda)
        mask[idx] = False
        assert int(page_view(p, sh)[mask].count_nonzero()) == 0
    sw.close()
