"""Events that order KV moves across workers (native pool and IPC cache).

Mirrors the reference's event plumbing with the same data format:
``reduce_event`` returns ``(device, handle_bytes)`` like
``reduce_cuda_event`` (aegaeon/utils.py:263-274) and ``rebuild_event`` follows
``rebuild_cuda_event`` (utils.py:277-288): a worker cannot open a handle its
own process exported, so a handle from the current device yields None and the
caller uses its local event.  Unlike the reference, opened handles are cached
(libkvx keeps them by handle bytes), so a waiter does not reopen and destroy
the same producer event on every call.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib


class Event:
    """A pooled CUDA event of the current device (kvx_event)."""

    def __init__(self, interprocess: bool = True, _handle: Optional[int] = None):
        if _handle is None:
            out = ctypes.c_void_p()
            _lib.check(_lib.lib().kvx_event_create(1 if interprocess else 0, ctypes.byref(out)))
            _handle = out.value
        self.handle = _handle
        self.device = torch.cuda.current_device()

    def record(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        stream = stream or torch.cuda.current_stream()
        _lib.check(_lib.lib().kvx_event_record(self.handle, stream.cuda_stream))

    def query(self) -> bool:
        done = ctypes.c_int(0)
        _lib.check(_lib.lib().kvx_event_query(self.handle, ctypes.byref(done)))
        return bool(done.value)

    def synchronize(self) -> None:
        _lib.check(_lib.lib().kvx_event_synchronize(self.handle))

    def ipc_handle(self) -> bytes:
        h = (ctypes.c_uint8 * 64)()
        _lib.check(_lib.lib().kvx_event_ipc_handle(self.handle, h))
        return bytes(h)

    def release(self) -> None:
        if self.handle:
            _lib.check(_lib.lib().kvx_event_release(self.handle))
            self.handle = None


def reduce_event(ev: Event) -> tuple:
    """(device, handle bytes) for another process (utils.py:263-274)."""
    return torch.cuda.current_device(), ev.ipc_handle()


def rebuild_event(handle: tuple, is_worker: bool = True) -> Optional[Event]:
    """The event behind a reduced handle, or None when it was exported by a
    worker on the current device (utils.py:277-288)."""
    device, raw = handle
    if is_worker and device == torch.cuda.current_device():
        return None
    h = (ctypes.c_uint8 * 64).from_buffer_copy(raw)
    out = ctypes.c_void_p()
    _lib.check(_lib.lib().kvx_event_open_ipc(h, ctypes.byref(out)))
    return Event(_handle=out.value)


def stream_wait(stream: torch.cuda.Stream, events: Sequence[Event]) -> None:
    """`stream` waits for every event of the list (one native call)."""
    arr = (ctypes.c_void_p * max(len(events), 1))(*[e.handle for e in events])
    _lib.check(_lib.lib().kvx_stream_wait_events(stream.cuda_stream, arr, len(events)))


def forget(handle: tuple) -> None:
    """Close a cached imported handle (e.g. after its producer departed)."""
    h = (ctypes.c_uint8 * 64).from_buffer_copy(handle[1])
    _lib.check(_lib.lib().kvx_event_forget_ipc(h))
