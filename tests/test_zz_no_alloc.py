"""kvx_swap_noalloc, the allocation-free swap, checked against kvx_swap.

Some callers cannot allocate GPU memory while they swap: a serving runtime
that hands all of HBM to its own arena (Aegaeon carves the KV cache out of one
arena), or a process swapping out near its memory limit during a model switch.
For them libkvx.so exports kvx_swap_noalloc, whose scratch (the id lists of a
call) is a fixed device array inside the library instead of memory the library
allocates.  This test calls it through the C ABI and compares what it writes
with what the regular entry point kvx_swap writes, bit for bit (the tolerance
of every swap test: these are byte copies), on two calls in a row.  It also
checks that those calls leave the device's free memory unchanged, that a
request above the array's capacity and a call on a capturing stream are
refused, and that managed memory is accepted on both sides as kvx_swap accepts
it.

The file name makes pytest collect it last, so a run that stops at the first
failure has run every other test before it.
"""

import ctypes

import numpy as np
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


def test_noalloc_refuses_a_capturing_stream():
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cache = torch.ones((4, 1024), dtype=torch.float16, device=dev)
    host = torch.zeros((4, 1024), dtype=torch.float16).pin_memory()
    # the one-time set-up call, outside any capture
    assert noalloc([0], [1], False, cache, host) == 0, _lib.lib().kvx_last_error()
    torch.cuda.synchronize()
    host.zero_()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    with torch.cuda.stream(side):
        graph.capture_begin()
        try:
            rc = noalloc([0, 1], [2, 3], False, cache, host)
            msg = _lib.lib().kvx_last_error()
        finally:
            graph.capture_end()
    assert rc == _lib.KVX_ERR_INVALID_ARGUMENT
    assert b"capturing" in msg
    torch.cuda.synchronize()
    assert int(host.view(torch.int16).abs().sum()) == 0


def _cudart():
    for name in ("libcudart.so.12", "libcudart.so"):
        try:
            return ctypes.CDLL(name)
        except OSError:
            continue
    pytest.skip("no CUDA runtime library to allocate managed memory with")


def test_noalloc_accepts_managed_memory_like_kvx_swap():
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    rt = _cudart()
    rt.cudaMallocManaged.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t,
                                     ctypes.c_uint]
    rt.cudaFree.argtypes = [ctypes.c_void_p]
    blocks, slots, block = 32, 24, 16 * 8 * 128 * 2
    cache_m, host_m = ctypes.c_void_p(), ctypes.c_void_p()
    assert rt.cudaMallocManaged(ctypes.byref(cache_m), blocks * block, 1) == 0
    assert rt.cudaMallocManaged(ctypes.byref(host_m), slots * block, 1) == 0
    try:
        content = np.random.default_rng(23).integers(0, 256, blocks * block, dtype=np.uint8)
        torch.cuda.synchronize()
        ctypes.memmove(cache_m.value, content.ctypes.data, blocks * block)
        ctypes.memset(host_m.value, 0, slots * block)
        cpu = torch.Generator().manual_seed(24)
        src = torch.randperm(blocks, generator=cpu)[:slots].tolist()
        dst = torch.randperm(slots, generator=cpu).tolist()
        stream = torch.cuda.current_stream().cuda_stream
        rc = _lib.lib().kvx_swap_noalloc(ids(src), ids(dst), len(src), 0, cache_m.value,
                                         blocks * block, block, host_m.value, slots * block,
                                         stream)
        assert rc == 0, _lib.lib().kvx_last_error()
        # the regular entry point on ordinary device / page-locked buffers
        cache = torch.from_numpy(content).to(dev).view(blocks, block)
        host = torch.zeros((slots, block), dtype=torch.uint8).pin_memory()
        rc = _lib.lib().kvx_swap(ids(src), ids(dst), len(src), 0, cache.data_ptr(),
                                 blocks * block, block, host.data_ptr(), slots * block,
                                 _lib.MODE_SM, stream)
        assert rc == 0, _lib.lib().kvx_last_error()
        torch.cuda.synchronize()
        got = np.ctypeslib.as_array((ctypes.c_uint8 * (slots * block)).from_address(host_m.value))
        assert np.array_equal(got, host.numpy().reshape(-1))
    finally:
        torch.cuda.synchronize()
        rt.cudaFree(cache_m)
        rt.cudaFree(host_m)
