"""Transfers of a model switch: weight storages up to the GPU and the KV
working set swapped in beside them, ending in one completion event.

In the reference, ``Worker.switch`` (aegaeon/worker.py:455-551) loads the new
model's weights through the quick loader (one host-to-device copy per cached
safetensors storage, aegaeon/loader/quick_loader.py:326-340, or through a
page-locked bounce buffer in pieces when the storage is pageable,
quick_model_loader/quick_model_loader/model_loader.py:348-369) and the decode
scheduler then swaps the requests' KV blocks back in (Worker.swap_blocks).
Both cross the same host link.  Here both are queued at once on two streams:

* the KV swap-in on the swapper's swap-in stream (``KVSwapper.swap_blocks``);
* the weights on a weight stream through ``kvx_upload_weights``, in pieces of
  ``chunk_bytes`` (64 MiB by default, the cut size of quick_loader.py:412).

``switch_in`` returns one event recorded after both.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence, Tuple

import torch

from . import _lib

DEFAULT_CHUNK_BYTES = 64 << 20


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def upload_weights(weights: Sequence[Tuple[torch.Tensor, torch.Tensor]], *,
                   chunk_bytes: int = DEFAULT_CHUNK_BYTES, host_threads: Optional[int] = None,
                   stream: Optional[torch.cuda.Stream] = None) -> None:
    """Copy each host tensor into its device tensor (same byte size, both
    contiguous) in pieces of ``chunk_bytes`` on ``stream`` (default: the
    current stream).  Page-locked sources are queued and the call returns at
    once; pageable sources go through the library's two page-locked bounce
    buffers, ``host_threads`` threads filling one while the copy engine
    drains the other (default: every host thread of this process)."""
    if not weights:
        return
    dev = None
    for dst, src in weights:
        if not dst.is_cuda or src.is_cuda:
            raise ValueError("weights are (device tensor, host tensor) pairs")
        if not dst.is_contiguous() or not src.is_contiguous():
            raise ValueError("weight tensors must be contiguous")
        if _nbytes(dst) != _nbytes(src):
            raise ValueError(f"size mismatch: device {_nbytes(dst)} B, host {_nbytes(src)} B")
        if dev is None:
            dev = dst.device
        elif dst.device != dev:
            raise ValueError("all destination tensors must be on one device")
    if stream is None:
        stream = torch.cuda.current_stream(dev)
    if host_threads is None:
        host_threads = len(os.sched_getaffinity(0))
    n = len(weights)
    dsts = (ctypes.c_void_p * n)(*[d.data_ptr() for d, _ in weights])
    srcs = (ctypes.c_void_p * n)(*[s.data_ptr() for _, s in weights])
    sizes = (ctypes.c_uint64 * n)(*[_nbytes(d) for d, _ in weights])
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().kvx_upload_weights(dsts, srcs, sizes, n, chunk_bytes,
                                                 host_threads, stream.cuda_stream))


def switch_in(swapper, weights: Sequence[Tuple[torch.Tensor, torch.Tensor]],
              request_ids: Sequence[int], source_block_ids: Sequence[int],
              target_block_ids: Sequence[int], group_ids: Sequence[int],
              first_kernel_blocks: Sequence[int], valid_kernel_blocks: Sequence[int],
              source_events: Sequence, *, chunk_bytes: int = DEFAULT_CHUNK_BYTES,
              kv_stream: Optional[torch.cuda.Stream] = None,
              weight_stream: Optional[torch.cuda.Stream] = None, mode: str | int = "auto",
              host_threads: Optional[int] = None) -> torch.cuda.Event:
    """Swap a KV working set in (``swapper.swap_blocks`` with host rows as
    sources, the reference's ``swap_blocks`` lists) and upload the new
    model's weight storages at the same time; returns one event recorded
    after both.  The swap is queued first so the copy engines start on it
    while the host is still busy with pageable weight pieces."""
    if kv_stream is None:
        kv_stream = swapper.swap_in_stream
    if weight_stream is None:
        # one weight stream per swapper, made on first use
        weight_stream = getattr(swapper, "_weight_stream", None)
        if weight_stream is None:
            weight_stream = torch.cuda.Stream(torch.device("cuda", swapper.device_index))
            swapper._weight_stream = weight_stream
    swapper.swap_blocks(request_ids, source_block_ids, target_block_ids, group_ids,
                        first_kernel_blocks, valid_kernel_blocks, source_events, True,
                        mode=mode, stream=kv_stream)
    upload_weights(weights, chunk_bytes=chunk_bytes, host_threads=host_threads,
                   stream=weight_stream)
    weights_done = torch.cuda.Event()
    weights_done.record(weight_stream)
    kv_stream.wait_event(weights_done)
    done = torch.cuda.Event()
    done.record(kv_stream)
    return done
