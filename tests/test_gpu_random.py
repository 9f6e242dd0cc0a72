"""Randomised GPU parity: seeded random layouts and requests through the
public APIs, in every transfer mode, byte-compared with the CPU oracle.

The layouts mix what the kernels and the mode policy branch on: uniform and
mixed page sizes (grid lists vs item lists), one or two cache groups with
partial extents, per-segment owners, tensor-parallel row offsets, repeated
targets (ordered waves), extents that are not 16-byte aligned (the kernel's
byte fallback), pages of several 32 KiB tiles, and request sizes on both
sides of the 124-record inline work-list limit.  Each step's mode rotates
through auto, sm, ce and ce_extent.
"""

import random

import numpy as np
import pytest
import torch

from aegaeon_b200 import _lib, ops, swapper

pytestmark = pytest.mark.gpu

MODES = ["auto", "sm", "ce", "ce_extent"]


def scenario(seed):
    rng = random.Random(seed)
    uniform = seed % 3 != 0
    ns = rng.randint(1, 6)
    ratios = rng.choice([[1], [4], [4, 1], [2, 4]])
    # page bytes: multiples of 4 x 16 (aligned), of 4 x 25 (unaligned extents)
    # or multi-tile pages
    unit = rng.choice([64, 100, 4096, 24576])
    base = unit * rng.randint(1, 4)
    pages = [base] * ns if uniform else [base * rng.randint(1, 3) for _ in range(ns)]
    ng = len(ratios)
    owners = [frozenset(range(ng)) if uniform or rng.random() < 0.5
              else frozenset({rng.randrange(ng)}) for _ in range(ns)]
    nblocks = rng.choice([16, 64, 256])
    nrows = rng.choice([16, 64, 256])
    if base >= 24576:  # keep the page-locked pool to a few hundred MB
        nblocks, nrows = min(nblocks, 64), min(nrows, 64)
    tp_size = rng.choice([1, 2])
    return rng, pages, ratios, owners, nblocks, nrows, tp_size, rng.randrange(tp_size)


@pytest.mark.parametrize("seed", range(16))
def test_random_swap_blocks_all_modes(cuda, oracle, seed):
    rng, pages, ratios, owners, nblocks, nrows, tp_size, tp_rank = scenario(seed)
    ns, ng = len(pages), len(ratios)
    gen = torch.Generator(device=cuda).manual_seed(seed)
    seg_t = [torch.randint(0, 256, (nblocks * p,), dtype=torch.uint8, device=cuda, generator=gen)
             for p in pages]
    segments, comp = swapper.make_segments(
        [((f"l{i}",), nblocks * p) for i, p in enumerate(pages)], nblocks)
    pool = torch.randint(0, 256, (nrows * comp * tp_size,), dtype=torch.uint8,
                         generator=torch.Generator().manual_seed(seed)).pin_memory()
    sw = swapper.KVSwapper(0, segments, seg_t, owners, ratios, kv_swap=pool, tp_rank=tp_rank,
                           tp_size=tp_size)
    torch.cuda.synchronize()
    exp_segs = [t.cpu().numpy().copy() for t in seg_t]
    exp_pool = pool.numpy().copy()
    offsets = [s.cpu_offset for s in segments]
    masks = [sum(1 << g for g in o) for o in owners]
    try:
        for step in range(4):
            is_in = bool(step % 2)
            mode = MODES[(seed + step) % len(MODES)]
            n = rng.randint(0, min(nblocks, nrows))
            dev = rng.sample(range(nblocks), n)
            rows = rng.sample(range(nrows), n)
            if n > 2 and rng.random() < 0.3:  # repeated target: the later copy wins
                (dev if is_in else rows)[0] = (dev if is_in else rows)[1]
            grp = [rng.randrange(ng) for _ in range(n)]
            first, valid = [], []
            for g in grp:
                r = ratios[g]
                f = rng.randrange(r)
                first.append(f)
                valid.append(rng.randint(0, r - f))
            src, dst = (rows, dev) if is_in else (dev, rows)
            oracle.swap_blocks(exp_segs, pages, offsets, masks, ratios, exp_pool,
                               comp * tp_size, tp_rank * comp, src, dst, grp, first, valid, is_in)
            sw.swap_blocks([0], src, dst, grp, first, valid, [None], is_in,
                           mode=mode).synchronize()
            assert np.array_equal(pool.numpy(), exp_pool), (seed, step, mode)
            for t, e in zip(seg_t, exp_segs):
                assert np.array_equal(t.cpu().numpy(), e), (seed, step, mode)
        assert _lib.device_status(0) == 0
    finally:
        sw.close()


@pytest.mark.parametrize("seed", range(8))
def test_random_ops_swap_all_modes(cuda, oracle, seed):
    rng = random.Random(200 + seed)
    elems = rng.choice([8, 40, 1024, 16384, 49152])  # 2-byte elements per block
    nb, nslots = rng.choice([16, 128, 512]), rng.choice([16, 128, 512])
    cache = torch.randint(-30000, 30000, (nb, elems), dtype=torch.int16, device=cuda,
                          generator=torch.Generator(device=cuda).manual_seed(seed))
    host = torch.randint(-30000, 30000, (nslots, elems), dtype=torch.int16,
                         generator=torch.Generator().manual_seed(seed)).pin_memory()
    torch.cuda.synchronize()
    bb = ops.reference_block_bytes(cache)
    exp_cache = cache.cpu().view(torch.uint8).numpy().reshape(-1).copy()
    exp_host = host.view(torch.uint8).numpy().reshape(-1).copy()
    for step in range(4):
        is_in = bool(step % 2)
        mode = MODES[(seed + step) % len(MODES)]
        n = rng.randint(0, min(nb, nslots))
        a = rng.sample(range(nb), n)
        b = rng.sample(range(nslots), n)
        if n > 1 and rng.random() < 0.4:
            (a if is_in else b)[0] = (a if is_in else b)[-1]
        src, dst = (b, a) if is_in else (a, b)
        oracle.swap(src, dst, is_in, exp_cache, exp_host, bb)
        ops.swap(src, dst, is_in, cache, host, mode=mode)
        torch.cuda.synchronize()
        assert np.array_equal(cache.cpu().view(torch.uint8).numpy().reshape(-1), exp_cache), \
            (seed, step, mode)
        assert np.array_equal(host.view(torch.uint8).numpy().reshape(-1), exp_host), \
            (seed, step, mode)
