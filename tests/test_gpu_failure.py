"""Device-side failure handling without a GPU fault.

The only device-side waits of the library are the TMA copy kernel's mbarrier
waits, each bounded by a deadline.  kvx_selftest_bounded_wait runs that same
wait on a barrier nothing arrives on: it must give up after its limit, record
KVX_ERR_DEVICE_TIMEOUT in the device status word, and leave the context
usable for the next copies.
"""

import time

import pytest
import torch

from aegaeon_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports(cuda):
    lib = _lib.lib()
    assert _lib.device_status(0, reset=True) in (0, _lib.KVX_ERR_DEVICE_TIMEOUT)
    s = torch.cuda.current_stream()
    t0 = time.perf_counter()
    _lib.check(lib.kvx_selftest_bounded_wait(50_000_000, s.cuda_stream))  # 50 ms
    assert _lib.device_status(0) == _lib.KVX_ERR_DEVICE_TIMEOUT
    assert time.perf_counter() - t0 < 5.0
    assert _lib.device_status(0, reset=True) == _lib.KVX_ERR_DEVICE_TIMEOUT
    assert _lib.device_status(0) == 0
    # the context is still usable
    cache = torch.randn((16, 16, 8, 128), device=cuda).to(torch.bfloat16)
    host = torch.zeros((16, 16, 8, 128), dtype=torch.bfloat16).pin_memory()
    ops.swap(list(range(16)), list(range(16)), False, cache, host)
    torch.cuda.synchronize()
    assert torch.equal(host.view(torch.uint8), cache.cpu().view(torch.uint8))
    assert _lib.device_status(0) == 0


def test_selftest_rejects_bad_limits(cuda):
    lib = _lib.lib()
    assert lib.kvx_selftest_bounded_wait(0, None) == _lib.KVX_ERR_INVALID_ARGUMENT
    assert lib.kvx_selftest_bounded_wait(11 * 10**9, None) == _lib.KVX_ERR_INVALID_ARGUMENT


def test_native_events_local(cuda):
    """Pool events record/query/synchronize; a handle exported on this device
    rebuilds to None (the caller then uses its local event)."""
    from aegaeon_b200 import events as kev

    s = torch.cuda.Stream(cuda)
    ev = kev.Event(interprocess=True)
    x = torch.randn(4096, 4096, device=cuda)
    with torch.cuda.stream(s):
        y = x @ x
    ev.record(s)
    ev.synchronize()
    assert ev.query()
    h = kev.reduce_event(ev)
    assert h[0] == torch.cuda.current_device() and len(h[1]) == 64
    assert kev.rebuild_event(h) is None
    s2 = torch.cuda.Stream(cuda)
    kev.stream_wait(s2, [ev])
    with torch.cuda.stream(s2):
        z = y.sum()
    torch.cuda.synchronize()
    assert torch.isfinite(z)
    handle = ev.handle
    ev.release()
    again = kev.Event(interprocess=True)
    assert again.handle == handle  # reused from the pool
    again.release()


def test_chunked_upload_parity(cuda):
    """kvx_upload_chunked (the weight upload of a model switch) moves the
    exact bytes, with chunk sizes that do not divide the length."""
    from aegaeon_b200 import _lib

    n = (3 << 20) + 12345
    pageable = torch.randint(0, 255, (n,), dtype=torch.uint8)
    dev = torch.zeros(n, dtype=torch.uint8, device=cuda)
    s = torch.cuda.current_stream()
    # page-locked: queued copies; pageable: through the library's bounce buffers
    for host in (pageable.pin_memory(), pageable):
        for chunk in (1 << 20, 4096 + 7, n, 0):
            dev.zero_()
            _lib.check(_lib.lib().kvx_upload_chunked(dev.data_ptr(), host.data_ptr(), n, chunk,
                                                     s.cuda_stream))
            torch.cuda.synchronize()
            assert torch.equal(dev.cpu(), host)
