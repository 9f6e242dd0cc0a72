"""The opt-in host_bulk form of the SM mode: copies with a host side go
through the TMA bulk kernel (16 KiB bulk copies between shared memory and
the device-mapped host rows).  Swap-out and swap-in of a segmented layout
are compared with the CPU oracle byte for byte."""

import numpy as np
import pytest
import torch

from aegaeon_b200 import _lib, swapper

pytestmark = pytest.mark.gpu


@pytest.fixture
def host_bulk():
    _lib.set_option("host_bulk", 1)
    yield
    _lib.set_option("host_bulk", 0)


def test_host_bulk_swap_round_trip_matches_oracle(cuda, oracle, host_bulk):
    layers, blocks, page, rows = 6, 96, 16384, 80
    g = torch.Generator(device=cuda).manual_seed(71)
    pages = [torch.randint(0, 256, (blocks * page,), generator=g, dtype=torch.uint8, device=cuda)
             for _ in range(layers)]
    segs, comp = swapper.make_segments([((f"l{i}",), blocks * page) for i in range(layers)],
                                       blocks)
    pool = torch.from_numpy(np.random.default_rng(72).integers(
        0, 256, rows * comp, dtype=np.uint8)).pin_memory()
    sw = swapper.KVSwapper(0, segs, pages, [frozenset({0})] * layers, [1], kv_swap=pool)
    cpu = torch.Generator().manual_seed(73)
    n = 64
    out_b = torch.randperm(blocks, generator=cpu)[:n].tolist()
    out_r = torch.randperm(rows, generator=cpu)[:n].tolist()
    seg_np = [p.cpu().numpy().copy() for p in pages]
    pool_np = pool.numpy().copy()
    oracle.swap_blocks(seg_np, [page] * layers, [s.cpu_offset for s in segs], [1] * layers, [1],
                       pool_np, comp, 0, out_b, out_r, [0] * n, [0] * n, [1] * n, False)
    torch.cuda.synchronize()
    sw.swap_blocks([0], out_b, out_r, [0] * n, [0] * n, [1] * n, [None], False,
                   mode="sm").synchronize()
    assert _lib.last_mode_name() == "sm"
    assert np.array_equal(pool.numpy(), pool_np)
    in_r = torch.randperm(rows, generator=cpu)[:n].tolist()
    in_b = torch.randperm(blocks, generator=cpu)[:n].tolist()
    oracle.swap_blocks(seg_np, [page] * layers, [s.cpu_offset for s in segs], [1] * layers, [1],
                       pool_np, comp, 0, in_r, in_b, [0] * n, [0] * n, [1] * n, True)
    sw.swap_blocks([1], in_r, in_b, [0] * n, [0] * n, [1] * n, [None], True,
                   mode="sm").synchronize()
    for p, e in zip(pages, seg_np):
        assert np.array_equal(p.cpu().numpy(), e)
    assert _lib.device_status(0) == 0
    sw.close()
