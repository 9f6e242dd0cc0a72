"""Byte-exact parity at the benchmark configurations' full shapes.

The reference's own swap op (ops/swap.cu, built unmodified into oracle/_ref)
and this build run on identical seeded inputs at the full BASELINE shapes;
host buffers and swapped-in caches are compared with torch.equal on uint8
views, on the device:

* configuration 1 (72 tensors [1024,16,8,128] bf16, 256 blocks each way) and
  configuration 2 (64 tensors [4096,16,32,128] fp16, 1024 blocks each way):
  the per-tensor op (ops.swap -> kvx_swap) against the reference op tensor by
  tensor, and the segmented path (KVSwapper.swap_blocks -> kvx_swap_blocks,
  composite host rows) against the reference op's per-tensor slots;
* configuration 5 (24 layers, 16,384 fragmented entries): the segmented
  swap-out against the reference op, segment by segment, then the swap-in of
  the same rows back into the zeroed blocks.
"""

import pytest
import torch

from aegaeon_b200 import _lib, ops, swapper, workloads

pytestmark = pytest.mark.gpu

GIB = 1 << 30


@pytest.fixture(scope="module")
def ref():
    from oracle import build_ref

    return build_ref.load_module()


def release():
    """Return cached device memory and cached page-locked host blocks."""
    import gc

    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    torch._C._host_emptyCache()


def host_gib_available() -> float:
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable"):
                return int(line.split()[1]) / (1 << 20)
    except OSError:
        pass
    return 0.0


def seeded_pages(sh, num_blocks, dev, seed=0):
    gen = torch.Generator(device=dev).manual_seed(seed)
    pages = []
    for _ in range(sh.num_segments):
        t = torch.empty(num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
        workloads.fill_segment(t, sh, gen)
        pages.append(t)
    return pages


def as_tensor(page_u8, sh, num_blocks):
    """A segment's pages as the reference op sees a K or V cache tensor."""
    return page_u8.view(sh.dtype).view(num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)


def u8(t):
    return t.view(torch.uint8)


def full_shape_parity(dev, ref, sh, num_blocks, out_ids, in_ids, mode):
    n = len(out_ids)
    slots = list(range(n))
    pages = seeded_pages(sh, num_blocks, dev)
    slot_shape = (n, sh.block_size, sh.kv_heads, sh.head_dim)
    ref_host = [torch.empty(slot_shape, dtype=sh.dtype, pin_memory=True)
                for _ in range(sh.num_segments)]
    kvx_host = torch.empty(slot_shape, dtype=sh.dtype, pin_memory=True)
    back_ref = torch.empty((num_blocks,) + slot_shape[1:], dtype=sh.dtype, device=dev)
    back_kvx = torch.empty_like(back_ref)
    # 1. per-tensor op against the reference op, tensor by tensor
    for s, p in enumerate(pages):
        cache = as_tensor(p, sh, num_blocks)
        kvx_host.zero_()
        ref.swap(out_ids, slots, False, cache, ref_host[s])
        ops.swap(out_ids, slots, False, cache, kvx_host, mode=mode)
        torch.cuda.synchronize()
        assert torch.equal(u8(ref_host[s]).to(dev), u8(kvx_host).to(dev)), ("out", s)
        back_ref.zero_()
        back_kvx.zero_()
        ref.swap(slots, in_ids, True, back_ref, ref_host[s])
        ops.swap(slots, in_ids, True, back_kvx, ref_host[s], mode=mode)
        torch.cuda.synchronize()
        assert torch.equal(u8(back_ref), u8(back_kvx)), ("in", s)
    del kvx_host
    # 2. segmented path (composite host rows) against the reference's slots
    segs, comp = swapper.make_segments(
        [((f"l{i}",), num_blocks * sh.page_bytes) for i in range(sh.num_segments)], num_blocks)
    pool = torch.zeros(n * comp, dtype=torch.uint8, pin_memory=True)
    sw = swapper.KVSwapper(dev.index, segs, pages, [frozenset({0})] * sh.num_segments, [1],
                           kv_swap=pool)
    z, one = [0] * n, [1] * n
    sw.swap_blocks([0], out_ids, slots, z, z, one, [None], False, mode=mode).synchronize()
    rows = pool.to(dev).view(n, sh.num_segments, sh.page_bytes)
    for s in range(sh.num_segments):
        assert torch.equal(rows[:, s], u8(ref_host[s]).to(dev).view(n, sh.page_bytes)), ("rows", s)
    del rows
    back_pages = [torch.zeros_like(p) for p in pages]
    torch.cuda.synchronize()  # the fills run on the current stream, the swap on its own
    sw_back = swapper.KVSwapper(dev.index, segs, back_pages, [frozenset({0})] * sh.num_segments,
                                [1], kv_swap=pool)
    sw_back.swap_blocks([0], slots, in_ids, z, z, one, [None], True, mode=mode).synchronize()
    for s in range(sh.num_segments):
        back_ref.zero_()
        ref.swap(slots, in_ids, True, back_ref, ref_host[s])
        torch.cuda.synchronize()
        assert torch.equal(u8(back_ref).view(-1), back_pages[s]), ("rows in", s)
    assert _lib.device_status(dev.index) == 0
    sw.close()
    sw_back.close()


@pytest.mark.parametrize("mode", ["auto", "sm", "ce"])
def test_cfg1_full_shape_matches_reference_op(cuda, ref, mode):
    sh = workloads.CFG1
    out_ids = workloads.randperm(sh.num_blocks, 0)[:256]
    in_ids = workloads.randperm(sh.num_blocks, 1)[:256]
    full_shape_parity(cuda, ref, sh, sh.num_blocks, out_ids, in_ids, mode)


def test_cfg2_full_shape_matches_reference_op(cuda, ref):
    if host_gib_available() < 40:
        pytest.skip("needs about 20 GiB of page-locked host memory")
    sh = workloads.CFG2
    out_ids, in_ids = workloads.swap_step_ids(sh.num_blocks, 1024, 0)
    full_shape_parity(cuda, ref, sh, sh.num_blocks, out_ids, in_ids, "auto")
    release()


def test_cfg5_full_shape_fragmented_matches_reference_op(cuda, ref):
    """All 24 layers and 16,384 entries: 48 GiB of host rows."""
    if host_gib_available() < 110:
        pytest.skip("needs about 49 GiB of page-locked host memory")
    sh = workloads.CFG5
    n = 16384
    ids, slots = workloads.fragmented_mapping(n, sh.num_blocks, seed=0)
    pages = seeded_pages(sh, sh.num_blocks, cuda, seed=5)
    segs, comp = swapper.make_segments(
        [((f"l{i}",), sh.num_blocks * sh.page_bytes) for i in range(sh.num_segments)],
        sh.num_blocks)
    pool = torch.empty(n * comp, dtype=torch.uint8, pin_memory=True)
    sw = swapper.KVSwapper(cuda.index, segs, pages, [frozenset({0})] * sh.num_segments, [1],
                           kv_swap=pool)
    z, one = [0] * n, [1] * n
    sw.swap_blocks([0], ids, slots, z, z, one, [None], False).synchronize()
    assert sw.last_stats == (n * comp, n * sh.num_segments)
    pool_dev = torch.empty(n * comp, dtype=torch.uint8, device=cuda)
    for o in range(0, n * comp, GIB):
        pool_dev[o:o + GIB].copy_(pool[o:o + GIB])
    rows = pool_dev.view(n, sh.num_segments, sh.page_bytes)
    ref_host = torch.empty((n, sh.block_size, sh.kv_heads, sh.head_dim), dtype=sh.dtype,
                           pin_memory=True)
    for s, p in enumerate(pages):
        ref.swap(ids, slots, False, as_tensor(p, sh, sh.num_blocks), ref_host)
        torch.cuda.synchronize()
        assert torch.equal(rows[:, s], u8(ref_host).to(cuda).view(n, sh.page_bytes)), s
    # the same rows back into the zeroed blocks
    idx = torch.tensor(ids, device=cuda)
    for p in pages:
        p.view(-1, sh.page_bytes)[idx] = 0
    sw.swap_blocks([0], slots, ids, z, z, one, [None], True).synchronize()
    for s, p in enumerate(pages):
        assert torch.equal(p.view(-1, sh.page_bytes)[idx], rows[:, s]), s
    assert _lib.device_status(cuda.index) == 0
    sw.close()
    del pool_dev, rows, pages, pool, ref_host, sw
    release()

