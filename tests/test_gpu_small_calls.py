"""Small requests: the launch forms chosen for them copy the same bytes.

* Grid plans of at most 1020 records (entries + segments) reach the vector
  kernel in its parameters instead of through the descriptor ring, in lists
  of 124, 508 or 1020 records; plans on either side of each limit must match
  the oracle byte for byte.
* In "auto" mode, a request that coalesces into one or two copies goes to the
  copy engine directly ("ce_extent"); one that does not, to the kernel.
"""

import numpy as np
import pytest
import torch

from aegaeon_b200 import _lib, ops, swapper

pytestmark = pytest.mark.gpu

INLINE_RECORDS = 124
INLINE_MID = 508
INLINE_MAX = 1020


def make(cuda, nsegs, nb, rows, page, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    segs = [torch.randint(0, 255, (nb * page,), dtype=torch.uint8, device=cuda, generator=g)
            for _ in range(nsegs)]
    segments, comp = swapper.make_segments([((f"l{i}",), nb * page) for i in range(nsegs)], nb)
    pool = torch.randint(0, 255, (rows * comp,), dtype=torch.uint8).pin_memory()
    sw = swapper.KVSwapper(0, segments, segs, [frozenset({0})] * nsegs, [1], kv_swap=pool)
    torch.cuda.synchronize()
    return sw, segs, segments, pool, comp


@pytest.mark.parametrize("records", [INLINE_RECORDS - 1, INLINE_RECORDS, INLINE_RECORDS + 1, 300,
                                     INLINE_MID, INLINE_MID + 1, INLINE_MAX, INLINE_MAX + 1])
def test_sm_swap_blocks_around_inline_limit(cuda, oracle, records):
    nsegs, page, nb, rows = 4, 4096, 1536, 1536
    n = records - nsegs
    sw, segs, segments, pool, comp = make(cuda, nsegs, nb, rows, page, records)
    g = torch.Generator().manual_seed(records)
    dev_ids = torch.randperm(nb, generator=g)[:n].tolist()
    host_ids = torch.randperm(rows, generator=g)[:n].tolist()
    try:
        for is_in in (False, True):
            exp_pool = pool.numpy().copy()
            exp_segs = [t.cpu().numpy().copy() for t in segs]
            src, dst = (host_ids, dev_ids) if is_in else (dev_ids, host_ids)
            oracle.swap_blocks(exp_segs, [page] * nsegs, [s.cpu_offset for s in segments],
                               [1] * nsegs, [1], exp_pool, comp, 0, src, dst, [0] * n, [0] * n,
                               [1] * n, is_in)
            sw.swap_blocks([0], src, dst, [0] * n, [0] * n, [1] * n, [None], is_in,
                           mode="sm").synchronize()
            assert _lib.last_mode_name() == "sm"
            assert np.array_equal(pool.numpy(), exp_pool)
            for t, e in zip(segs, exp_segs):
                assert np.array_equal(t.cpu().numpy(), e)
            host_ids = torch.randperm(rows, generator=g)[:n].tolist()
    finally:
        sw.close()


@pytest.mark.parametrize("n", [INLINE_RECORDS - 1, INLINE_RECORDS, 400, INLINE_MID,
                               INLINE_MAX - 1, INLINE_MAX])
def test_ops_swap_sm_around_inline_limit(cuda, oracle, n):
    """ops.swap plans have one segment: n entries + 1 record."""
    blocks, slots = 1536, 1536
    g = torch.Generator(device=cuda).manual_seed(n)
    cache = torch.randint(-30000, 30000, (blocks, 1024), dtype=torch.int16, device=cuda,
                          generator=g)
    swap_buf = torch.zeros((slots, 1024), dtype=torch.int16).pin_memory()
    torch.cuda.synchronize()
    cg = torch.Generator().manual_seed(n + 1)
    src = torch.randperm(blocks, generator=cg)[:n].tolist()
    dst = torch.randperm(slots, generator=cg)[:n].tolist()
    bb = ops.reference_block_bytes(cache)
    for is_in in (False, True):
        exp_swap = swap_buf.view(torch.uint8).numpy().reshape(-1).copy()
        exp_cache = cache.cpu().view(torch.uint8).numpy().reshape(-1).copy()
        if is_in:
            oracle.swap(dst, src, True, exp_cache, exp_swap.copy(), bb)
            ops.swap(dst, src, True, cache, swap_buf, mode="sm")
        else:
            oracle.swap(src, dst, False, exp_cache.copy(), exp_swap, bb)
            ops.swap(src, dst, False, cache, swap_buf, mode="sm")
        torch.cuda.synchronize()
        assert _lib.last_mode_name() == "sm"
        assert np.array_equal(swap_buf.view(torch.uint8).numpy().reshape(-1), exp_swap)
        assert np.array_equal(cache.cpu().view(torch.uint8).numpy().reshape(-1), exp_cache)
        if not is_in:
            cache.zero_()
            torch.cuda.synchronize()


def test_auto_sends_one_or_two_copies_to_copy_engine(cuda, oracle):
    blocks = 64
    g = torch.Generator(device=cuda).manual_seed(9)
    cache = torch.randn((blocks, 16, 8, 128), device=cuda, generator=g).to(torch.bfloat16)
    swap_buf = torch.zeros((blocks, 16, 8, 128), dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    bb = ops.reference_block_bytes(cache)

    def host_view(t):
        return t.reshape(-1).view(torch.uint8).numpy()

    cache_host = host_view(cache.cpu()).copy()
    cases = [
        ([5], [9], "ce_extent"),                        # one copy
        ([1, 2, 3, 4], [10, 11, 12, 13], "ce_extent"),  # coalesces into one copy
        ([1, 7], [3, 40], "ce_extent"),                 # two copies
        ([1, 7, 20], [3, 40, 41], "sm"),                # three copies: the kernel
    ]
    for src, dst, want in cases:
        exp = host_view(swap_buf).copy()
        oracle.swap(src, dst, False, cache_host, exp, bb)
        ops.swap(src, dst, False, cache, swap_buf)
        torch.cuda.synchronize()
        assert _lib.last_mode_name() == want, (src, dst)
        assert np.array_equal(host_view(swap_buf), exp)
        # and back in, to other blocks
        back = [b + 32 for b in src]
        exp_cache = cache_host.copy()
        oracle.swap(dst, back, True, exp_cache, host_view(swap_buf).copy(), bb)
        ops.swap(dst, back, True, cache, swap_buf)
        torch.cuda.synchronize()
        assert _lib.last_mode_name() == want
        cache_host = host_view(cache.cpu()).copy()
        assert np.array_equal(cache_host, exp_cache)


@pytest.mark.parametrize("n", [INLINE_RECORDS - 4, INLINE_RECORDS - 3, 300, INLINE_MAX - 4,
                               INLINE_MAX - 3])
def test_copy_blocks_local_around_inline_limit(cuda, n):
    """On-GPU block copies (migration path, one device): 4 segments."""
    nsegs, page, nb = 4, 8192, 2048
    sw, segs, _, _, _ = make(cuda, nsegs, nb, 8, page, n)
    g = torch.Generator().manual_seed(n)
    ids = torch.randperm(nb, generator=g)[: 2 * n].tolist()
    src, dst = ids[:n], ids[n:]
    before = [t.view(nb, page).clone() for t in segs]
    torch.cuda.synchronize()
    try:
        sw.copy_blocks_local(src, dst, mode="sm").synchronize()
        for t, b in zip(segs, before):
            v = t.view(nb, page)
            assert torch.equal(v[dst], b[src])
            keep = torch.ones(nb, dtype=torch.bool, device=cuda)
            keep[dst] = False
            assert torch.equal(v[keep], b[keep])
    finally:
        sw.close()
