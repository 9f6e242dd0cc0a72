"""Drop-in replacement for the reference's native ``aegaeon.ops`` module.

``swap`` keeps the reference's Python-visible signature and semantics
(pybind registration ``ops/ops.cpp:4-6``, implementation ``ops/swap.cu:25-60``):

* ``source_block_ids[i]`` is copied to ``target_block_ids[i]``; swap-in moves
  host slots into device blocks, swap-out device blocks into host slots;
* a block is ``kv_cache.numel() * 2 // kv_cache.size(0)`` bytes (the reference
  assumes 2-byte elements, ``swap.cu:34``) and block ``id`` starts at byte
  ``id * block_bytes`` of both buffers;
* the copy is queued on the current CUDA stream of ``kv_cache``'s device and
  the call returns before it completes; the caller records an event.

Differences, all on inputs the reference leaves undefined: ids are checked
against both buffers before anything is queued (the reference copies out of
bounds), mismatched list lengths raise ``ValueError`` (the reference reads past
the shorter list), and repeated target ids keep the last copy, as the
reference's in-order copies do.

The copy itself runs in libkvx.so: an sm_100a kernel writing or reading the
page-locked host buffer through its device mapping, or copy-engine copies of
coalesced runs through a device staging area, chosen per call (``mode``).
"""

from __future__ import annotations

from typing import Sequence

import torch

from . import _lib


def span_bytes(t: torch.Tensor) -> int:
    """Bytes addressable from ``t.data_ptr()`` to the end of its storage."""
    return t.untyped_storage().nbytes() - t.storage_offset() * t.element_size()


def reference_block_bytes(kv_cache: torch.Tensor) -> int:
    """Block size the reference derives from the cache (ops/swap.cu:34)."""
    if kv_cache.dim() == 0 or kv_cache.size(0) == 0:
        raise ValueError("kv_cache must have a non-empty leading block dimension")
    return kv_cache.numel() * 2 // kv_cache.size(0)


def swap(
    source_block_ids: Sequence[int],
    target_block_ids: Sequence[int],
    is_swap_in: bool,
    kv_cache: torch.Tensor,
    kv_swap: torch.Tensor,
    *,
    mode: str | int = "auto",
) -> None:
    """Swap whole blocks between ``kv_cache`` (device) and ``kv_swap`` (host).

    Drop-in for ``aegaeon.ops.swap`` (ops/swap.cu:25-60).  ``mode`` selects
    the transfer engine: "auto" (default), "sm", "ce" or "ce_extent".
    """
    if not kv_cache.is_cuda:
        raise ValueError("kv_cache must be a CUDA tensor")
    if kv_swap.is_cuda:
        raise ValueError("kv_swap must be a host (CPU) tensor")
    device = kv_cache.device.index
    if torch.cuda.current_device() == device:
        _swap_here(source_block_ids, target_block_ids, is_swap_in, kv_cache, kv_swap, mode,
                   device)
    else:
        with torch.cuda.device(device):
            _swap_here(source_block_ids, target_block_ids, is_swap_in, kv_cache, kv_swap,
                       mode, device)


def _swap_here(source_block_ids, target_block_ids, is_swap_in, kv_cache, kv_swap, mode,
               device) -> None:
    """Body of swap; runs with ``device`` (kv_cache's) current.  The call shim
    converts the ids and checks their lengths (ValueError) in C."""
    status = _lib.shim().swap(
        _lib.ids_arg(source_block_ids),
        _lib.ids_arg(target_block_ids),
        is_swap_in,
        kv_cache.data_ptr(),
        span_bytes(kv_cache),
        reference_block_bytes(kv_cache),
        kv_swap.data_ptr(),
        span_bytes(kv_swap),
        _lib.mode_of(mode),
        _lib.current_stream_handle(device),
    )
    if status:
        _lib.check(status)


def plan_swap(
    source_block_ids: Sequence[int],
    target_block_ids: Sequence[int],
    is_swap_in: bool,
    kv_cache_ptr: int,
    kv_cache_bytes: int,
    block_bytes: int,
    kv_swap_ptr: int,
    kv_swap_bytes: int,
) -> list[tuple[int, int, int]]:
    """The (source address, destination address, bytes) copies ``swap`` would
    issue, from the native planner, without touching a GPU."""
    import ctypes

    n = len(source_block_ids)
    if len(target_block_ids) != n:
        raise ValueError("id lists differ in length")
    lib = _lib.lib()
    src = _lib.i64_array(source_block_ids)
    dst = _lib.i64_array(target_block_ids)
    count = ctypes.c_int64(0)
    _lib.check(
        lib.kvx_plan_swap(src, dst, n, 1 if is_swap_in else 0, kv_cache_ptr, kv_cache_bytes,
                          block_bytes, kv_swap_ptr, kv_swap_bytes, None, None, None,
                          ctypes.byref(count))
    )
    m = count.value
    a = (ctypes.c_uint64 * max(m, 1))()
    b = (ctypes.c_uint64 * max(m, 1))()
    c = (ctypes.c_uint64 * max(m, 1))()
    _lib.check(
        lib.kvx_plan_swap(src, dst, n, 1 if is_swap_in else 0, kv_cache_ptr, kv_cache_bytes,
                          block_bytes, kv_swap_ptr, kv_swap_bytes, a, b, c, ctypes.byref(count))
    )
    return [(a[i], b[i], c[i]) for i in range(m)]
