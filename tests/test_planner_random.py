"""Randomised host-side checks of the native planner against the C oracle.

For random layouts (uniform and mixed page sizes, several cache groups,
partial extents, tensor-parallel row offsets, repeated targets) the copies
libkvx.so plans are applied with memmove to host buffers and the bytes are
compared with the oracle's restatement of worker.py:2270-2329.  Uniform
layouts with distinct targets take the grid form, whose copies come from the
same tile resolver the kernels use; the others take the item planner.
"""

import ctypes
import random

import numpy as np
import pytest

from aegaeon_b200 import ops, swapper


def plan_copies(kvx, layout, src, dst, grp, first, valid, is_in):
    arr = swapper._entry_arrays(src, dst, grp, first, valid)
    n = arr[0]
    count = ctypes.c_int64(0)
    rc = kvx.kvx_plan_swap_blocks(layout.handle, n, *arr[1:], int(is_in), None, None, None,
                                  ctypes.byref(count))
    assert rc == 0, kvx.kvx_last_error()
    m = count.value
    S, D, L = ((ctypes.c_uint64 * max(m, 1))() for _ in range(3))
    assert kvx.kvx_plan_swap_blocks(layout.handle, n, *arr[1:], int(is_in), S, D, L,
                                    ctypes.byref(count)) == 0
    return [(S[i], D[i], L[i]) for i in range(m)]


@pytest.mark.parametrize("seed", range(24))
def test_random_layouts_match_oracle(kvx, oracle, seed):
    rng = random.Random(seed)
    uniform = seed % 3 != 0
    ns = rng.randint(1, 6)
    ratios = rng.choice([[1], [4], [4, 1], [2, 4]])
    base_page = 16 * rng.choice([1, 4, 12])
    base_page *= max(ratios)
    pages = [base_page] * ns if uniform else [base_page * rng.randint(1, 3) for _ in range(ns)]
    ng = len(ratios)
    owners = [(1 << ng) - 1 if uniform or rng.random() < 0.5 else 1 << rng.randrange(ng)
              for _ in range(ns)]
    nblocks, nrows = rng.randint(4, 24), rng.randint(4, 24)
    tp_size = rng.choice([1, 2])
    tp_rank = rng.randrange(tp_size)
    comp = sum(pages)
    offsets = list(np.cumsum([0] + pages[:-1]))
    gen = np.random.default_rng(seed)
    segs = [gen.integers(0, 256, nblocks * p, dtype=np.uint8) for p in pages]
    pool = gen.integers(0, 256, nrows * comp * tp_size, dtype=np.uint8)
    ref_segs = [s.copy() for s in segs]
    ref_pool = pool.copy()
    lay = swapper._Layout(0, [s.ctypes.data for s in segs], pages, [nblocks] * ns,
                          [int(o) for o in offsets], owners, ratios, pool.ctypes.data,
                          pool.size, comp * tp_size, tp_rank * comp)
    for step in range(4):
        is_in = bool(step % 2)
        n = rng.randint(0, min(nblocks, nrows))
        dev = rng.sample(range(nblocks), n)
        rows = rng.sample(range(nrows), n)
        if n > 2 and rng.random() < 0.3:  # repeated target
            (dev if is_in else rows)[0] = (dev if is_in else rows)[1]
        grp = [rng.randrange(ng) for _ in range(n)]
        first, valid = [], []
        for g in grp:
            r = ratios[g]
            f = rng.randrange(r)
            first.append(f)
            valid.append(rng.randint(0, r - f))
        src, dst = (rows, dev) if is_in else (dev, rows)
        for s_, d_, l_ in plan_copies(kvx, lay, src, dst, grp, first, valid, is_in):
            ctypes.memmove(d_, s_, l_)
        oracle.swap_blocks(ref_segs, pages, [int(o) for o in offsets], owners, ratios, ref_pool,
                           comp * tp_size, tp_rank * comp, src, dst, grp, first, valid, is_in)
        assert np.array_equal(pool, ref_pool), (seed, step)
        for a, b in zip(segs, ref_segs):
            assert np.array_equal(a, b), (seed, step)
    lay.close()


@pytest.mark.parametrize("seed", range(8))
def test_per_tensor_plan_matches_oracle(oracle, seed):
    rng = random.Random(100 + seed)
    block = 16 * rng.randint(1, 40)
    nb, ns = rng.randint(2, 40), rng.randint(2, 40)
    gen = np.random.default_rng(seed)
    cache = gen.integers(0, 256, nb * block, dtype=np.uint8)
    swap_buf = gen.integers(0, 256, ns * block, dtype=np.uint8)
    rc_cache, rc_swap = cache.copy(), swap_buf.copy()
    for is_in in (False, True, False):
        n = rng.randint(0, min(nb, ns))
        a = rng.sample(range(nb), n)
        b = rng.sample(range(ns), n)
        if n > 1 and rng.random() < 0.4:
            (a if is_in else b)[0] = (a if is_in else b)[-1]
        src, dst = (b, a) if is_in else (a, b)
        for s_, d_, l_ in ops.plan_swap(src, dst, is_in, cache.ctypes.data, cache.size, block,
                                        swap_buf.ctypes.data, swap_buf.size):
            ctypes.memmove(d_, s_, l_)
        oracle.swap(src, dst, is_in, rc_cache, rc_swap, block)
        assert np.array_equal(cache, rc_cache) and np.array_equal(swap_buf, rc_swap)
