"""Model-switch transfers (switch.switch_in / kvx_upload_weights): weight
storages uploaded in pieces beside a KV swap-in, one completion event.

Reference: Worker.switch (aegaeon/worker.py:455-551) loads weights through
the quick loader (load_tensors_content, aegaeon/loader/quick_loader.py:326-340;
pipeline_storage_transfer, quick_model_loader/.../model_loader.py:348-369)
while the KV working set is swapped back in by Worker.swap_blocks.  The
uploaded bytes must equal the host storages and the swapped-in pages must
equal the CPU oracle's swap_blocks result, byte for byte.
"""

import ctypes

import numpy as np
import pytest
import torch

from aegaeon_b200 import _lib, swapper, switch

pytestmark = pytest.mark.gpu

# odd sizes: pieces that do not divide the storage, a storage below one piece
SHARD_BYTES = [(64 << 20) + 4096 + 3, 200 << 20, (1 << 20) + 17]


def host_storages(pinned: bool, seed: int):
    rng = np.random.default_rng(seed)
    out = []
    for n in SHARD_BYTES:
        t = torch.from_numpy(rng.integers(0, 256, n, dtype=np.uint8))
        out.append(t.pin_memory() if pinned else t)
    return out


def kv_setup(dev, seed):
    layers, blocks, page, rows = 8, 96, 16384, 64
    g = torch.Generator(device=dev).manual_seed(seed)
    pages = [torch.randint(0, 256, (blocks * page,), generator=g, dtype=torch.uint8, device=dev)
             for _ in range(layers)]
    segs, comp = swapper.make_segments([((f"l{i}",), blocks * page) for i in range(layers)],
                                       blocks)
    pool = torch.from_numpy(np.random.default_rng(seed).integers(
        0, 256, rows * comp, dtype=np.uint8)).pin_memory()
    sw = swapper.KVSwapper(dev.index, segs, pages, [frozenset({0})] * layers, [1], kv_swap=pool)
    return sw, pages, segs, comp, pool, page, rows


@pytest.mark.parametrize("pinned,chunk", [(True, 64 << 20), (False, 64 << 20), (False, 1 << 20)])
def test_switch_in_matches_oracle(cuda, oracle, pinned, chunk):
    torch.cuda.set_device(cuda)
    sw, pages, segs, comp, pool, page, rows = kv_setup(cuda, 31)
    hosts = host_storages(pinned, 32)
    devs = [torch.zeros(h.numel(), dtype=torch.uint8, device=cuda) for h in hosts]
    g = torch.Generator().manual_seed(33)
    n = 48
    src_rows = torch.randperm(rows, generator=g)[:n].tolist()
    dst_blocks = torch.randperm(96, generator=g)[:n].tolist()
    # the oracle's result on host copies of the same bytes
    seg_np = [p.cpu().numpy().copy() for p in pages]
    pool_np = pool.numpy().copy()
    oracle.swap_blocks(seg_np, [page] * len(pages), [s.cpu_offset for s in segs],
                       [1] * len(pages), [1], pool_np, comp, 0, src_rows, dst_blocks,
                       [0] * n, [0] * n, [1] * n, True)
    torch.cuda.synchronize()
    done = switch.switch_in(sw, list(zip(devs, hosts)), [7], src_rows, dst_blocks, [0] * n,
                            [0] * n, [1] * n, [None], chunk_bytes=chunk)
    done.synchronize()
    for d, h in zip(devs, hosts):
        assert torch.equal(d.cpu(), h)
    for p, e in zip(pages, seg_np):
        assert np.array_equal(p.cpu().numpy(), e)
    assert _lib.device_status(0) == 0
    sw.close()


def test_upload_weights_back_to_back_reuses_bounce_buffers(cuda):
    """Two pageable uploads in a row through small pieces (many reuses of each
    bounce buffer), then a pinned one on another stream: all bytes exact."""
    torch.cuda.set_device(cuda)
    a, b = host_storages(False, 41), host_storages(False, 42)
    da = [torch.zeros(h.numel(), dtype=torch.uint8, device=cuda) for h in a]
    db = [torch.zeros(h.numel(), dtype=torch.uint8, device=cuda) for h in b]
    s = torch.cuda.Stream(cuda)
    switch.upload_weights(list(zip(da, a)), chunk_bytes=3 << 20, host_threads=4, stream=s)
    switch.upload_weights(list(zip(db, b)), chunk_bytes=5 << 20 | 1, host_threads=2, stream=s)
    c = host_storages(True, 43)
    dc = [torch.zeros(h.numel(), dtype=torch.uint8, device=cuda) for h in c]
    s2 = torch.cuda.Stream(cuda)
    switch.upload_weights(list(zip(dc, c)), stream=s2)
    torch.cuda.synchronize()
    for d, h in zip(da + db + dc, a + b + c):
        assert torch.equal(d.cpu(), h)


def test_upload_weights_rejects_bad_arguments(cuda):
    torch.cuda.set_device(cuda)
    h = torch.zeros(4096, dtype=torch.uint8)
    with pytest.raises(ValueError):
        switch.upload_weights([(torch.zeros(4095, dtype=torch.uint8, device=cuda), h)])
    with pytest.raises(ValueError):
        switch.upload_weights([(h.clone(), h)])
    lib = _lib.lib()
    one = lambda t, v: (t * 1)(v)  # noqa: E731
    # a host pointer as the destination: refused before anything is queued
    rc = lib.kvx_upload_weights(one(ctypes.c_void_p, h.data_ptr()),
                                one(ctypes.c_void_p, h.data_ptr()),
                                one(ctypes.c_uint64, 4096), 1, 1 << 20, 1, None)
    assert rc == _lib.KVX_ERR_INVALID_ARGUMENT
    d = torch.zeros(4096, dtype=torch.uint8, device=cuda)
    rc = lib.kvx_upload_weights(one(ctypes.c_void_p, d.data_ptr()),
                                one(ctypes.c_void_p, h.data_ptr()),
                                one(ctypes.c_uint64, 4096), 1, 0, 1, None)
    assert rc == _lib.KVX_ERR_INVALID_ARGUMENT


def test_upload_weights_mixed_sources_in_one_call(cuda):
    """Page-locked and pageable storages (and an empty one) in one call: each
    goes its own way (direct pieces or the bounce buffers), all bytes exact."""
    torch.cuda.set_device(cuda)
    rng = np.random.default_rng(51)
    sizes = [(5 << 20) + 1, 0, (70 << 20) + 33, 4096, (3 << 20) + 7]
    hosts = []
    for k, n in enumerate(sizes):
        t = torch.from_numpy(rng.integers(0, 256, n, dtype=np.uint8))
        hosts.append(t.pin_memory() if k % 2 == 0 else t)
    devs = [torch.zeros(n, dtype=torch.uint8, device=cuda) for n in sizes]
    switch.upload_weights(list(zip(devs, hosts)), chunk_bytes=2 << 20, host_threads=3)
    torch.cuda.synchronize()
    for d, h in zip(devs, hosts):
        assert torch.equal(d.cpu(), h)
