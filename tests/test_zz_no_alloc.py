"""kvx_swap_noalloc, the allocation-free swap, checked against kvx_swap.

Some callers cannot allocate GPU memory while they swap: a serving runtime
that hands all of HBM to its own arena (Aegaeon carves the KV cache out of one
arena), or a process swapping out near its memory limit during a model switch.
For them libkvx.so exports kvx_swap_noalloc, whose scratch (the id lists of a
call) is a fixed device array inside the library instead of memory the library
allocates.  This test calls it through the C ABI and compares what it writes
with what the regular entry point kvx_swap writes, bit for bit (the tolerance
of every swap test: these are byte copies), on two calls in a row.  It also
checks that those calls leave the device's free memory unchanged and that a
request above the array's capacity is refused.

The file name makes pytest collect it last, so a run that stops at the first
failure has run every other test before it.
"""

import ctypes

import pytest
import torch

from aegaeon_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_IDS = 65536  # KVX_NOALLOC_MAX_IDS in include/kvx.h


def ids(values):
    return (ctypes.c_int64 * max(len(values), 1))(*values)


def call(fn, src, dst, is_in, cache, host, *extra):
    block = cache.numel() * 2 // cache.size(0)
    stream = torch.cuda.current_stream().cuda_stream
    return fn(ids(src), ids(dst), len(src), 1 if is_in else 0, cache.data_ptr(),
              cache.numel() * cache.element_size(), block, host.data_ptr(),
              host.numel() * host.element_size(), *extra, stream)


def regular(src, dst, is_in, cache, host):
    rc = call(_lib.lib().kvx_swap, src, dst, is_in, cache, host, _lib.MODE_SM)
    assert rc == 0, _lib.lib().kvx_last_error()


def noalloc(src, dst, is_in, cache, host):
    return call(_lib.lib().kvx_swap_noalloc, src, dst, is_in, cache, host)


def test_noalloc_matches_regular_entry_point():
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(21)
    cache = torch.randn((128, 16, 8, 128), generator=g, device=dev).to(torch.bfloat16)
    host_a = torch.zeros((96, 16, 8, 128), dtype=torch.bfloat16).pin_memory()
    host_b = torch.zeros_like(host_a).pin_memory()
    cache_a = torch.zeros_like(cache)
    cache_b = torch.zeros_like(cache)
    cpu = torch.Generator().manual_seed(22)
    out_src = torch.randperm(128, generator=cpu)[:80].tolist()
    out_dst = torch.randperm(96, generator=cpu)[:80].tolist()
    in_src = torch.randperm(96, generator=cpu)[:70].tolist()
    in_dst = torch.randperm(128, generator=cpu)[:70].tolist()
    in_dst[5] = in_dst[40]  # a repeated target: the later copy must win

    # The regular entry point first (it sets up its own work areas), then the
    # allocation-free one: first call (does the one-time address lookup) ...
    regular(out_src, out_dst, False, cache, host_a)
    torch.cuda.synchronize()
    assert noalloc(out_src, out_dst, False, cache, host_b) == 0, _lib.lib().kvx_last_error()
    torch.cuda.synchronize()
    assert torch.equal(host_a.view(torch.uint8), host_b.view(torch.uint8))

    # ... and the second call in a row, which must not allocate anything.
    regular(in_src, in_dst, True, cache_a, host_a)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(dev)
    torch_before = torch.cuda.memory_allocated(dev)
    assert noalloc(in_src, in_dst, True, cache_b, host_b) == 0, _lib.lib().kvx_last_error()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(dev)
    assert torch.equal(cache_a.view(torch.uint8), cache_b.view(torch.uint8))
    assert free_after == free_before
    assert torch.cuda.memory_allocated(dev) == torch_before


def test_noalloc_refuses_more_ids_than_its_scratch_holds():
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cache = torch.ones((4, 1024), dtype=torch.float16, device=dev)
    host = torch.zeros((4, 1024), dtype=torch.float16).pin_memory()
    n = MAX_IDS + 1
    rc = noalloc([0] * n, [0] * n, False, cache, host)
    assert rc == _lib.KVX_ERR_INVALID_ARGUMENT
    assert b"KVX_NOALLOC_MAX_IDS" in _lib.lib().kvx_last_error()
    torch.cuda.synchronize()
    assert int(host.view(torch.int16).abs().sum()) == 0
