"""GPU parity of the swap path against the CPU oracle and the reference op.

Bit-exact byte equality throughout (pure copies).  Every test calls the CUDA
path through the C ABI (libkvx.so via aegaeon_b200.ops / .swapper).
"""

import numpy as np
import pytest
import torch

import golden_swap as gs
from aegaeon_b200 import _lib, ops, swapper

pytestmark = pytest.mark.gpu

MODES = ["auto", "sm", "ce", "ce_extent"]


def host_bytes(t: torch.Tensor) -> np.ndarray:
    return t.reshape(-1).view(torch.uint8).numpy()


def rand_cache(shape, dtype, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    if dtype in (torch.bfloat16, torch.float16):
        return torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(dtype)
    return torch.randint(0, 255, shape, generator=g, device=device, dtype=torch.uint8)


def perm(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(n, generator=g)[:k].tolist()


@pytest.mark.parametrize("mode", MODES)
def test_swap_round_trip_matches_oracle(cuda, oracle, mode):
    blocks, slots = 64, 48
    cache = rand_cache((blocks, 16, 8, 128), torch.bfloat16, cuda, 1)
    swap_buf = torch.empty((slots, 16, 8, 128), dtype=torch.bfloat16).pin_memory()
    swap_buf.view(torch.uint8).fill_(0xA5)
    bb = ops.reference_block_bytes(cache)
    src = perm(blocks, 40, 2)
    dst = perm(slots, 40, 3)
    exp_swap = host_bytes(swap_buf).copy()
    cache_host = host_bytes(cache.cpu()).copy()
    oracle.swap(src, dst, False, cache_host, exp_swap, bb)
    ops.swap(src, dst, False, cache, swap_buf, mode=mode)
    torch.cuda.synchronize()
    if mode != "auto":
        assert _lib.last_mode_name() == mode
    assert np.array_equal(host_bytes(swap_buf), exp_swap)
    # swap-in into a zeroed cache at fresh ids
    cache2 = torch.zeros_like(cache)
    back = perm(blocks, 40, 4)
    exp_cache = np.zeros(cache2.numel() * 2, np.uint8)
    oracle.swap(dst, back, True, exp_cache, host_bytes(swap_buf).copy(), bb)
    ops.swap(dst, back, True, cache2, swap_buf, mode=mode)
    torch.cuda.synchronize()
    assert np.array_equal(host_bytes(cache2.cpu()), exp_cache)
    assert torch.equal(cache2[back], cache[src])


def test_swap_matches_reference_op(cuda):
    """The reference's own ops.swap (built from ops/swap.cu into oracle/_ref)
    and ours produce identical buffers on the same inputs."""
    from oracle import build_ref

    ref = build_ref.load_module()
    blocks = 96
    cache = rand_cache((blocks, 16, 8, 128), torch.bfloat16, cuda, 5)
    a = torch.zeros((blocks, 16, 8, 128), dtype=torch.bfloat16).pin_memory()
    b = torch.zeros_like(a).pin_memory()
    src, dst = perm(blocks, 70, 6), perm(blocks, 70, 7)
    ref.swap(src, dst, False, cache, a)
    ops.swap(src, dst, False, cache, b)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    c1, c2 = torch.zeros_like(cache), torch.zeros_like(cache)
    back = perm(blocks, 70, 8)
    ref.swap(dst, back, True, c1, a)
    ops.swap(dst, back, True, c2, b)
    torch.cuda.synchronize()
    assert torch.equal(c1.view(torch.uint8), c2.view(torch.uint8))


def test_reference_op_matches_oracle(cuda, oracle):
    """Pins the oracle: the reference op and the C oracle agree, including the
    reference's 2-byte block-size rule on a 4-byte dtype."""
    from oracle import build_ref

    ref = build_ref.load_module()
    cache = torch.arange(32 * 64, dtype=torch.float32, device=cuda).view(32, 64)
    swap_buf = torch.zeros(32 * 64, dtype=torch.float32).pin_memory()
    bb = ops.reference_block_bytes(cache)  # 128 bytes: half a row, as the reference computes
    assert bb == 128
    src, dst = [0, 5, 31, 17], [3, 1, 0, 60]
    exp = host_bytes(swap_buf).copy()
    oracle.swap(src, dst, False, host_bytes(cache.cpu()).copy(), exp, bb)
    ref.swap(src, dst, False, cache, swap_buf)
    torch.cuda.synchronize()
    assert np.array_equal(host_bytes(swap_buf), exp)
    mine = torch.zeros_like(swap_buf).pin_memory()
    ops.swap(src, dst, False, cache, mine)
    torch.cuda.synchronize()
    assert np.array_equal(host_bytes(mine), exp)


@pytest.mark.parametrize("mode", ["sm", "ce", "ce_extent"])
def test_duplicate_targets_last_wins(cuda, oracle, mode):
    cache = rand_cache((16, 4096), torch.uint8, cuda, 9)
    swap_buf = torch.zeros((8, 4096), dtype=torch.uint8).pin_memory()
    src, dst = [1, 2, 3, 4, 5], [0, 1, 0, 1, 0]
    exp = host_bytes(swap_buf).copy()
    oracle.swap(src, dst, False, host_bytes(cache.cpu()).copy(), exp, 8192)
    ops.swap(src, dst, False, cache, swap_buf, mode=mode)
    torch.cuda.synchronize()
    assert np.array_equal(host_bytes(swap_buf), exp)


def test_pageable_host_buffer_uses_copy_engine(cuda, oracle):
    cache = rand_cache((32, 2048), torch.float16, cuda, 10)
    swap_buf = torch.zeros((32, 2048), dtype=torch.float16)  # not pinned
    src, dst = perm(32, 20, 11), perm(32, 20, 12)
    ops.swap(src, dst, False, cache, swap_buf)
    torch.cuda.synchronize()
    assert _lib.last_mode_name() == "ce"
    exp = np.zeros(swap_buf.numel() * 2, np.uint8)
    oracle.swap(src, dst, False, host_bytes(cache.cpu()).copy(), exp, 4096)
    assert np.array_equal(host_bytes(swap_buf), exp)
    with pytest.raises(ValueError, match="page-locked"):
        ops.swap(src, dst, False, cache, swap_buf, mode="sm")


def test_invalid_ids_copy_nothing(cuda):
    cache = rand_cache((8, 1024), torch.uint8, cuda, 13)
    swap_buf = torch.zeros((4, 1024), dtype=torch.uint8).pin_memory()
    with pytest.raises(IndexError):
        ops.swap([0, 1, 9], [0, 1, 2], False, cache, swap_buf)
    with pytest.raises(IndexError):
        ops.swap([0, 1], [0, 4], False, cache, swap_buf)
    with pytest.raises(IndexError):
        ops.swap([-1], [0], False, cache, swap_buf)
    with pytest.raises(ValueError):
        ops.swap([0, 1], [0], False, cache, swap_buf)
    torch.cuda.synchronize()
    assert int(swap_buf.sum()) == 0
    ops.swap([], [], False, cache, swap_buf)


def test_swap_uses_current_stream(cuda):
    cache = rand_cache((64, 32768), torch.float16, cuda, 14)
    swap_buf = torch.zeros((64, 32768), dtype=torch.float16).pin_memory()
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        ops.swap(list(range(64)), list(range(64)), False, cache, swap_buf)
        ev = torch.cuda.Event()
        ev.record(s)
    ev.synchronize()
    assert torch.equal(swap_buf.view(torch.uint8), cache.cpu().view(torch.uint8))


def make_swapper_from_scenario(scn, segs, pool, device):
    pages = scn["pages"]
    seg_t = [torch.from_numpy(s).to(device) for s in segs]
    host = torch.from_numpy(pool).pin_memory()
    segments = [swapper.CacheSegment(f"seg{i}", (f"seg{i}",), off, p)
                for i, (off, p) in enumerate(zip(scn["cpu_offsets"], pages))]
    owners = [frozenset(o) for o in scn["owners"]]
    sw = swapper.KVSwapper(device.index or 0, segments, seg_t, owners, gs.group_ratios(scn),
                           kv_swap=host, tp_rank=scn["tp_rank"], tp_size=scn["tp_size"])
    return sw, seg_t, host


@pytest.mark.parametrize("mode", MODES)
def test_swap_blocks_golden_on_gpu(cuda, golden, mode):
    """Worker.swap_blocks fixtures (hybrid groups, partial extents, TP rank
    offsets, 8-byte-granular pages) reproduced by the CUDA path."""
    for scn in golden("swap_blocks.json")["scenarios"]:
        segs, pool = gs.fresh_state(scn)
        sw, seg_t, host = make_swapper_from_scenario(scn, segs, pool, cuda)
        for step in scn["steps"]:
            n = len(step["source"])
            ev = sw.swap_blocks(list(range(n)), step["source"], step["target"], step["groups"],
                                step["first"], step["valid"], [None] * n, step["is_swap_in"],
                                mode=mode)
            ev.synchronize()
            gs.check_step(step, [t.cpu().numpy() for t in seg_t], host.numpy())
        sw.close()


def test_swap_blocks_events_order_moves(cuda):
    """A swap-in queued after a swap-out of the same request waits for it."""
    pages = [1 << 20] * 4
    segs = [torch.randint(0, 255, (8 * p,), dtype=torch.uint8, device=cuda) for p in pages]
    segments, comp = swapper.make_segments([((f"l{i}",), 8 * p) for i, p in enumerate(pages)], 8)
    host = torch.zeros(4 * comp, dtype=torch.uint8).pin_memory()
    sw = swapper.KVSwapper(0, segments, segs, [frozenset({0})] * 4, [1], kv_swap=host)
    e1 = sw.swap_blocks([7], [1, 2, 3], [0, 1, 2], [0] * 3, [0] * 3, [1] * 3, [None], False)
    e2 = sw.swap_blocks([7], [0, 1, 2], [5, 6, 7], [0] * 3, [0] * 3, [1] * 3, [e1], True)
    e2.synchronize()
    for t in segs:
        pg = t.view(8, -1)
        assert torch.equal(pg[5:8], pg[1:4])
    assert sw.last_stats == (3 * comp, 12)
    assert len(sw.move_event_table[7]) == 2
    sw.close()


@pytest.mark.parametrize("pipeline", [0, 1])
def test_staged_chunks_parity(cuda, oracle, pipeline):
    """Copy-engine mode over many staging chunks (small staging area), with
    and without the double-buffered pipeline: bytes equal the oracle's."""
    pages = [65536] * 6
    nb, rows = 96, 80
    segs = [torch.randint(0, 255, (nb * p,), dtype=torch.uint8, device=cuda) for p in pages]
    segments, comp = swapper.make_segments([((f"l{i}",), nb * p) for i, p in enumerate(pages)], nb)
    pool = torch.randint(0, 255, (rows * comp,), dtype=torch.uint8).pin_memory()
    sw = swapper.KVSwapper(0, segments, segs, [frozenset({0})] * 6, [1], kv_swap=pool)
    _lib.configure(staging_bytes=4 << 20, ce_pipeline=pipeline)
    try:
        g = torch.Generator().manual_seed(30 + pipeline)
        dev_ids = torch.randperm(nb, generator=g)[:70].tolist()
        host_ids = torch.randperm(rows, generator=g)[:70].tolist()
        n = 70
        for is_in in (False, True):
            exp_pool = pool.numpy().copy()
            exp_segs = [t.cpu().numpy().copy() for t in segs]
            src, dst = (host_ids, dev_ids) if is_in else (dev_ids, host_ids)
            oracle.swap_blocks(exp_segs, pages, [s.cpu_offset for s in segments], [1] * 6, [1],
                               exp_pool, comp, 0, src, dst, [0] * n, [0] * n, [1] * n, is_in)
            sw.swap_blocks([0], src, dst, [0] * n, [0] * n, [1] * n, [None], is_in,
                           mode="ce").synchronize()
            assert np.array_equal(pool.numpy(), exp_pool)
            for t, e in zip(segs, exp_segs):
                assert np.array_equal(t.cpu().numpy(), e)
            host_ids = torch.randperm(rows, generator=g)[:70].tolist()
    finally:
        _lib.configure(staging_bytes=1 << 30, ce_pipeline=0)
        sw.close()


def test_device_status_clean(cuda):
    assert _lib.device_status(0) == 0


@pytest.mark.parametrize("ctas", [0, 1, 3, 111, 185, 4096, (5, 300)])
@pytest.mark.parametrize("shape,dtype", [((64, 3, 5, 7), torch.bfloat16),
                                         ((64, 16, 8, 128), torch.bfloat16),
                                         ((32, 16, 32, 128), torch.float16)])
def test_sm_host_path_any_grid_matches_oracle(cuda, oracle, ctas, shape, dtype):
    """The SM zero-copy kernels split their tiles over however many CTAs the
    host-path grid gives them (by default 3/4 of the SMs writing host memory
    and 5/4 reading it; `sm_ctas_host` overrides both, `sm_ctas_host_out` /
    `sm_ctas_host_in` one direction each): one CTA, fewer CTAs than tiles,
    more CTAs than tiles, and blocks of 210 bytes (byte path), 32 KiB (one
    tile) and 128 KiB (four tiles) all give the oracle's bytes."""
    blocks = shape[0]
    slots = blocks // 2 + 3
    cache = rand_cache(shape, dtype, cuda, 21)
    swap_buf = torch.empty((slots,) + shape[1:], dtype=dtype).pin_memory()
    swap_buf.view(torch.uint8).fill_(0x3C)
    bb = ops.reference_block_bytes(cache)
    src, dst = perm(blocks, slots - 3, 22), perm(slots, slots - 3, 23)
    back = perm(blocks, slots - 3, 24)
    if isinstance(ctas, tuple):
        _lib.set_option("sm_ctas_host_out", ctas[0])
        _lib.set_option("sm_ctas_host_in", ctas[1])
    else:
        _lib.set_option("sm_ctas_host", ctas)
    try:
        exp_swap = host_bytes(swap_buf).copy()
        oracle.swap(src, dst, False, host_bytes(cache.cpu()).copy(), exp_swap, bb)
        ops.swap(src, dst, False, cache, swap_buf, mode="sm")
        torch.cuda.synchronize()
        assert _lib.last_mode_name() == "sm"
        assert np.array_equal(host_bytes(swap_buf), exp_swap)
        cache2 = torch.zeros_like(cache)
        exp_cache = np.zeros(cache2.numel() * cache2.element_size(), np.uint8)
        oracle.swap(dst, back, True, exp_cache, host_bytes(swap_buf).copy(), bb)
        ops.swap(dst, back, True, cache2, swap_buf, mode="sm")
        torch.cuda.synchronize()
        assert np.array_equal(host_bytes(cache2.cpu()), exp_cache)
    finally:
        for name in ("sm_ctas_host", "sm_ctas_host_out", "sm_ctas_host_in"):
            _lib.set_option(name, 0)
    assert _lib.device_status(cuda.index) == 0
