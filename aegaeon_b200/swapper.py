"""Worker-side KV movement: the segmented swap and GPU->GPU migration.

``KVSwapper`` holds what the reference's ``Worker`` sets up for swapping
(``aegaeon/worker.py:253-281`` streams and host pool, ``:1396-1433`` segment
owners and the ``kv_swap_view`` row layout) and exposes the same operations:

* ``swap_blocks``           - worker.py:2204-2349 (hot loop :2270-2329 runs in
                              libkvx.so as one planned launch instead of one
                              ``copy_`` per extent);
* ``wait_for_all_move_in/out`` - worker.py:2406-2418;
* ``migrate_blocks`` and the IPC handle registration - the reference's stubs
  at worker.py:2420-2451, implemented here over NVLink peer mappings.

Host row layout (worker.py:2304-2309): row ``r`` of the host pool holds, for
tensor-parallel rank ``tp_rank``, the composite page at byte
``tp_rank * composite_page``; segment ``s`` sits at ``segment.cpu_offset``
inside it, and a partial extent at ``byte_offset`` inside the segment page.
"""

from __future__ import annotations

import ctypes
import logging
from collections import defaultdict
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib

logger = logging.getLogger(__name__)


@dataclass(frozen=True)
class CacheSegment:
    """One backing tensor's bytes inside a composite cache block
    (vllm_cache.py:28-40)."""

    layer_name: str
    shared_by: tuple
    cpu_offset: int
    page_size_bytes: int


def make_segments(
    tensor_specs: Sequence[tuple[tuple[str, ...], int]], num_blocks: int
) -> tuple[list[CacheSegment], int]:
    """Segments and composite page size from ``(shared_by, size_bytes)`` per
    backing tensor, in order (make_composite_config, vllm_cache.py:75-101):
    the page of a tensor is ``size // num_blocks`` and its host offset is the
    running sum of the earlier pages."""
    if num_blocks <= 0:
        raise MemoryError(
            "Not enough cache memory for one group-aware cache block: "
            f"num_blocks={num_blocks}"
        )
    segments: list[CacheSegment] = []
    offset = 0
    for shared_by, size in tensor_specs:
        page, rem = divmod(size, num_blocks)
        if rem:
            raise ValueError(
                "KV-cache tensor size must contain an integral page per block: "
                f"size={size}, blocks={num_blocks}"
            )
        shared_by = tuple(shared_by)
        if not shared_by:
            raise ValueError("KV-cache tensor is not bound to any layer")
        segments.append(CacheSegment(shared_by[0], shared_by, offset, page))
        offset += page
    return segments, offset


def segment_owner_groups(
    segments: Sequence[CacheSegment], group_layer_names: Sequence[Sequence[str]]
) -> list[frozenset]:
    """Cache groups allowed to copy each segment: the groups with a layer in
    the segment's ``shared_by`` (worker.py:1396-1415)."""
    names = [set(g) for g in group_layer_names]
    owners = []
    for seg in segments:
        own = frozenset(g for g, layer_names in enumerate(names) if set(seg.shared_by) & layer_names)
        if not own:
            raise ValueError(f"Cache segment {seg.layer_name} is not owned by any KV-cache group")
        owners.append(own)
    return owners


def host_row_view(kv_swap: torch.Tensor, composite_page: int, tp_size: int = 1) -> torch.Tensor:
    """``kv_swap`` as ``[num_cpu_blocks, tp_size * composite_page]`` bytes
    (worker.py:1419-1433)."""
    row = composite_page * tp_size
    if row % kv_swap.element_size():
        raise ValueError(
            f"Composite cache page {row} is not aligned to CPU cache dtype size "
            f"{kv_swap.element_size()}"
        )
    flat = kv_swap.reshape(-1).view(torch.uint8)
    rows = flat.numel() // row
    return flat.narrow(0, 0, rows * row).view(rows, row)


class _Layout:
    """Owns one native kvx_layout handle."""

    def __init__(self, device: int, pages: Sequence[int], page_bytes: Sequence[int],
                 num_blocks: Sequence[int], cpu_offsets: Sequence[int],
                 owner_masks: Sequence[int], group_ratios: Sequence[int],
                 host_ptr: int = 0, host_bytes: int = 0, row_bytes: int = 0,
                 row_offset: int = 0):
        ns = len(pages)
        lib = _lib.lib()
        P = (ctypes.c_void_p * max(ns, 1))(*pages)
        U = lambda v: (ctypes.c_uint64 * max(len(v), 1))(*v)  # noqa: E731
        G = (ctypes.c_int64 * max(len(group_ratios), 1))(*group_ratios)
        out = ctypes.c_void_p()
        _lib.check(
            lib.kvx_layout_create(
                device, ns, P, U(page_bytes), U(num_blocks), U(cpu_offsets), U(owner_masks),
                len(group_ratios), G, host_ptr or None, host_bytes, row_bytes, row_offset,
                ctypes.byref(out),
            )
        )
        self.handle = out.value
        self.page_bytes = list(page_bytes)

    def close(self) -> None:
        if self.handle:
            _lib.lib().kvx_layout_destroy(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


def _check_lengths(source_block_ids, target_block_ids, group_ids, first_kernel_blocks,
                   valid_kernel_blocks) -> int:
    n = len(source_block_ids)
    if (len(target_block_ids) == n and len(group_ids) == n and len(first_kernel_blocks) == n
            and len(valid_kernel_blocks) == n):
        return n
    _entry_arrays(source_block_ids, target_block_ids, group_ids, first_kernel_blocks,
                  valid_kernel_blocks)  # raises with the reference's message
    raise AssertionError("unreachable")


def _entry_arrays(source_block_ids, target_block_ids, group_ids, first_kernel_blocks,
                  valid_kernel_blocks):
    lengths = {
        len(source_block_ids),
        len(target_block_ids),
        len(group_ids),
        len(first_kernel_blocks),
        len(valid_kernel_blocks),
    }
    if len(lengths) != 1:  # worker.py:2230-2243
        raise ValueError(
            "Swap block ids and metadata must have equal lengths: "
            f"source={len(source_block_ids)}, target={len(target_block_ids)}, "
            f"groups={len(group_ids)}, first={len(first_kernel_blocks)}, "
            f"valid={len(valid_kernel_blocks)}"
        )
    a = _lib.i64_array
    return (len(source_block_ids), a(source_block_ids), a(target_block_ids), a(group_ids),
            a(first_kernel_blocks), a(valid_kernel_blocks))


class KVSwapper:
    """Swap / migration executor for one GPU's composite KV cache.

    Args:
        device: CUDA device index of the cache.
        segments: composite layout (``make_segments``).
        segment_pages: per segment, a CUDA tensor whose storage holds its
            ``num_blocks`` pages (any dtype; only bytes are moved).
        segment_owners: per segment, the cache-group ids that own it.
        group_blocks_per_kv_block: per cache group, kernel blocks per physical
            block (1 for plain paged attention).
        kv_swap: host pool (page-locked for the SM path), or None for a
            migration-only endpoint.
        tp_rank, tp_size: tensor-parallel placement inside a host row.
    """

    def __init__(self, device: int, segments: Sequence[CacheSegment],
                 segment_pages: Sequence[torch.Tensor],
                 segment_owners: Sequence[frozenset],
                 group_blocks_per_kv_block: Sequence[int],
                 kv_swap: Optional[torch.Tensor] = None,
                 tp_rank: int = 0, tp_size: int = 1):
        if len(segment_pages) != len(segments) or len(segment_owners) != len(segments):
            raise ValueError("segments, segment_pages and segment_owners differ in length")
        if kv_swap is not None and kv_swap.is_cuda:
            raise ValueError("kv_swap must be a host (CPU) tensor")
        for t, s in zip(segment_pages, segments):
            if not t.is_cuda:
                raise ValueError(f"segment {s.layer_name}: pages must be a CUDA tensor")
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.device_index = self.device.index if self.device.index is not None else 0
        self.segments = list(segments)
        self.segment_pages = list(segment_pages)
        self.segment_owners = [frozenset(o) for o in segment_owners]
        self.group_ratios = [int(r) for r in group_blocks_per_kv_block]
        self.composite_page = sum(s.page_size_bytes for s in segments)
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.kv_swap = kv_swap
        self.kv_swap_view = (
            host_row_view(kv_swap, self.composite_page, tp_size) if kv_swap is not None else None
        )
        for t, s in zip(segment_pages, segments):
            if not t.is_contiguous():
                raise ValueError(f"segment {s.layer_name}: page tensor must be contiguous")
        # worker.py:2274: num_gpu_blocks = raw.numel() // page (raw is int8)
        num_blocks = [t.numel() * t.element_size() // s.page_size_bytes
                      for t, s in zip(segment_pages, segments)]
        self.num_gpu_blocks = num_blocks
        masks = [sum(1 << g for g in o) for o in self.segment_owners]
        host_ptr = host_bytes = row_bytes = 0
        if self.kv_swap_view is not None:
            host_ptr = self.kv_swap_view.data_ptr()
            host_bytes = self.kv_swap_view.numel()
            row_bytes = self.kv_swap_view.size(1)
        self._layout = _Layout(
            self.device_index, [t.data_ptr() for t in segment_pages],
            [s.page_size_bytes for s in segments], num_blocks,
            [s.cpu_offset for s in segments], masks, self.group_ratios,
            host_ptr, host_bytes, row_bytes, tp_rank * self.composite_page,
        )
        self._masks = masks
        self._swap_in_stream = None
        self._swap_out_stream = None
        self.move_event_table: dict = defaultdict(list)
        self._peers: dict = {}  # engine id -> (_Layout, [mapped pointers])
        self.last_stats = (0, 0)

    # ---- streams (worker.py:278-280) ------------------------------------
    @property
    def swap_in_stream(self) -> torch.cuda.Stream:
        if self._swap_in_stream is None:
            self._swap_in_stream = torch.cuda.Stream(self.device)
        return self._swap_in_stream

    @property
    def swap_out_stream(self) -> torch.cuda.Stream:
        if self._swap_out_stream is None:
            self._swap_out_stream = torch.cuda.Stream(self.device)
        return self._swap_out_stream

    # ---- swap (worker.py:2204-2349) -------------------------------------
    def swap_blocks(self, request_ids: Sequence[int], source_block_ids: Sequence[int],
                    target_block_ids: Sequence[int], group_ids: Sequence[int],
                    first_kernel_blocks: Sequence[int], valid_kernel_blocks: Sequence[int],
                    source_events: Sequence[Optional[torch.cuda.Event]], is_swap_in: bool,
                    *, mode: str | int = "auto", stream: Optional[torch.cuda.Stream] = None,
                    interprocess: bool = False, return_handle: bool = False):
        """Swap the live extents of blocks between GPU pages and host rows.

        Queued on the swap-in / swap-out stream after the given source events
        (see ``_wait_source_events``) and returns an event recorded after the
        copies; with ``return_handle`` it returns ``(device, handle bytes)`` of
        an interprocess event instead, the reference's return value
        (worker.py:2349).  ``copied_bytes`` / ``copy_extents`` of the call are
        left in ``last_stats``.
        """
        if self.kv_swap_view is None:
            raise ValueError("this KVSwapper has no host pool")
        _check_lengths(source_block_ids, target_block_ids, group_ids, first_kernel_blocks,
                       valid_kernel_blocks)
        if stream is None:
            stream = self.swap_in_stream if is_swap_in else self.swap_out_stream
        a = _lib.ids_arg
        args = (request_ids, a(source_block_ids), a(target_block_ids), a(group_ids),
                a(first_kernel_blocks), a(valid_kernel_blocks), source_events, is_swap_in, mode,
                stream, interprocess, return_handle)
        if torch.cuda.current_device() == self.device_index:
            return self._swap_blocks_here(*args)
        with torch.cuda.device(self.device_index):
            return self._swap_blocks_here(*args)

    def _swap_blocks_here(self, request_ids, src, dst, grp, first, valid, source_events,
                          is_swap_in, mode, stream, interprocess, return_handle):
        """Body of swap_blocks; runs with this cache's device current.  The call
        shim converts the ids and checks the five lengths (ValueError) in C."""
        if return_handle:
            from . import events as kev

            new_event = kev.Event(interprocess=True)
        else:
            new_event = torch.cuda.Event(interprocess=interprocess)
        self._wait_source_events(stream, new_event, request_ids, source_events)
        status, copied, extents = _lib.shim().swap_blocks(
            self._layout.handle, src, dst, grp, first, valid, is_swap_in, _lib.mode_of(mode),
            stream.cuda_stream)
        if status:
            _lib.check(status)
        new_event.record(stream)
        self.last_stats = (copied, extents)
        if logger.isEnabledFor(logging.DEBUG):
            full = len(src) * self.composite_page
            logger.debug(
                "swap requests %s (%s to %s): copied %d/%d bytes (saved %.2f%%), "
                "%d DMA extents", list(request_ids), "CPU" if is_swap_in else "GPU",
                "GPU" if is_swap_in else "CPU", copied, full,
                0.0 if full == 0 else 100.0 * (1 - copied / full), extents,
            )
        if return_handle:
            return kev.reduce_event(new_event)
        return new_event

    def plan_swap_blocks(self, source_block_ids, target_block_ids, group_ids,
                         first_kernel_blocks, valid_kernel_blocks, is_swap_in):
        """The (src, dst, bytes) copies ``swap_blocks`` would issue, in the
        reference's order, with host addresses of the pool; no GPU needed."""
        n, src, dst, grp, first, valid = _entry_arrays(
            source_block_ids, target_block_ids, group_ids, first_kernel_blocks,
            valid_kernel_blocks)
        lib = _lib.lib()
        count = ctypes.c_int64(0)
        _lib.check(lib.kvx_plan_swap_blocks(self._layout.handle, n, src, dst, grp, first, valid,
                                            1 if is_swap_in else 0, None, None, None,
                                            ctypes.byref(count)))
        m = count.value
        a = (ctypes.c_uint64 * max(m, 1))()
        b = (ctypes.c_uint64 * max(m, 1))()
        c = (ctypes.c_uint64 * max(m, 1))()
        _lib.check(lib.kvx_plan_swap_blocks(self._layout.handle, n, src, dst, grp, first, valid,
                                            1 if is_swap_in else 0, a, b, c, ctypes.byref(count)))
        return [(a[i], b[i], c[i]) for i in range(m)]

    def _wait_source_events(self, stream, new_event, request_ids, source_events):
        """Order this move after earlier moves of the same requests
        (worker.py:2351-2394).  An entry may be None (nothing to wait for), a
        torch or kvx event, or a ``(device, handle bytes)`` pair as produced
        by ``swap_blocks(..., return_handle=True)`` in any worker (the
        reference's ``reduce_cuda_event`` format).  A handle exported on this
        device stands for the request's latest local event, as in the
        reference; other handles are opened once and cached natively, and all
        kvx events are waited on in one call."""
        from . import events as kev

        if source_events is None:
            source_events = [None] * len(request_ids)
        batch = []
        for request_id, ev in zip(request_ids, source_events):
            if ev is not None:
                if isinstance(ev, tuple):
                    opened = kev.rebuild_event(ev, is_worker=True)
                    if opened is None:
                        if not self.move_event_table.get(request_id):
                            raise ValueError(
                                f"request {request_id} should have a local event here")
                        ev = self.move_event_table[request_id][-1]
                    else:
                        ev = opened
                if isinstance(ev, kev.Event):
                    batch.append(ev)
                else:
                    stream.wait_event(ev)
            self.move_event_table[request_id].append(new_event)
        if batch:
            kev.stream_wait(stream, batch)

    def clear_request_resource(self, request_id: int) -> None:
        self.move_event_table.pop(request_id, None)

    def clear_request_resource_batched(self, request_ids: Sequence[int]) -> None:
        for r in request_ids:
            self.clear_request_resource(r)

    def wait_for_all_move_in(self) -> None:
        self.swap_in_stream.synchronize()

    def wait_for_all_move_out(self) -> None:
        self.swap_out_stream.synchronize()

    # ---- migration (worker.py:2420-2451) --------------------------------
    def export_kvcache_mem_handles(self) -> list:
        """IPC handles of this cache's segment pages: one ``(handle bytes,
        offset, page bytes, num blocks)`` per segment, plus owners and group
        ratios, to ship to the peer worker."""
        lib = _lib.lib()
        out = []
        for t, s, nb in zip(self.segment_pages, self.segments, self.num_gpu_blocks):
            h = (ctypes.c_uint8 * 64)()
            off = ctypes.c_uint64(0)
            _lib.check(lib.kvx_ipc_export(t.data_ptr(), h, ctypes.byref(off)))
            out.append((bytes(h), off.value, s.page_size_bytes, nb))
        return [out, list(self._masks), list(self.group_ratios)]

    def register_kvcache_mem_handles(self, peer_engine_id, peer_parallel_config,
                                     kvcache_ipc_mem_handles) -> None:
        """Map a peer worker's cache pages into this process (peer access over
        NVLink) for later ``migrate_blocks`` calls.  ``peer_parallel_config``
        is accepted for signature parity and unused (TP=1)."""
        del peer_parallel_config
        seg_handles, masks, ratios = kvcache_ipc_mem_handles
        if len(seg_handles) != len(self.segments):
            raise ValueError("peer cache has a different number of segments")
        lib = _lib.lib()
        ptrs = []
        try:
            for hbytes, off, _, _ in seg_handles:
                h = (ctypes.c_uint8 * 64).from_buffer_copy(hbytes)
                p = ctypes.c_void_p()
                _lib.check(lib.kvx_ipc_import(self.device_index, h, off, ctypes.byref(p)))
                ptrs.append(p.value)
        except Exception:
            for p in ptrs:
                lib.kvx_ipc_close(self.device_index, p)
            raise
        layout = _Layout(self.device_index, ptrs, [h[2] for h in seg_handles],
                         [h[3] for h in seg_handles], [0] * len(ptrs), masks, ratios)
        self.unregister_kvcache_mem_handles(peer_engine_id)
        self._peers[peer_engine_id] = (layout, ptrs)

    def unregister_kvcache_mem_handles(self, peer_engine_id) -> None:
        entry = self._peers.pop(peer_engine_id, None)
        if entry is None:
            return
        layout, ptrs = entry
        layout.close()
        lib = _lib.lib()
        for p in ptrs:
            _lib.check(lib.kvx_ipc_close(self.device_index, p))

    def local_endpoint(self) -> _Layout:
        """This cache as a migration endpoint (no host pool)."""
        if not hasattr(self, "_local_ep"):
            self._local_ep = _Layout(
                self.device_index, [t.data_ptr() for t in self.segment_pages],
                [s.page_size_bytes for s in self.segments], self.num_gpu_blocks,
                [0] * len(self.segments), self._masks, self.group_ratios)
        return self._local_ep

    def migrate_blocks(self, request_ids: Sequence[int], source_engine_id,
                       source_block_ids: Sequence[int], target_block_ids: Sequence[int],
                       source_events: Sequence[Optional[torch.cuda.Event]] = None,
                       group_ids: Optional[Sequence[int]] = None,
                       first_kernel_blocks: Optional[Sequence[int]] = None,
                       valid_kernel_blocks: Optional[Sequence[int]] = None,
                       *, direction: str = "pull", mode: str | int = "auto",
                       stream: Optional[torch.cuda.Stream] = None,
                       liveness=None) -> torch.cuda.Event:
        """Copy blocks between this GPU and a registered peer over NVLink.

        ``direction="pull"`` (the reference's decode-side signature): the peer
        ``source_engine_id`` holds ``source_block_ids`` and this cache receives
        them at ``target_block_ids``.  ``direction="push"``: this cache is the
        source and the registered peer ``source_engine_id`` the target.
        Without group / extent lists every entry is a full page of group 0.
        ``liveness`` (e.g. ``Heartbeat.guard(peer)``) is called before anything
        is queued and raises when the peer process has gone, so no copy ever
        touches the memory of a departed peer.
        """
        if liveness is not None:
            liveness()
        if source_engine_id not in self._peers:
            raise ValueError(f"no KV-cache handles registered for engine {source_engine_id}")
        n = len(source_block_ids)
        if group_ids is None:
            group_ids = [0] * n
        if first_kernel_blocks is None:
            first_kernel_blocks = [0] * n
        if valid_kernel_blocks is None:
            valid_kernel_blocks = [self.group_ratios[g] for g in group_ids]
        _check_lengths(source_block_ids, target_block_ids, group_ids, first_kernel_blocks,
                       valid_kernel_blocks)
        a = _lib.ids_arg
        src, dst, grp, first, valid = (a(source_block_ids), a(target_block_ids), a(group_ids),
                                       a(first_kernel_blocks), a(valid_kernel_blocks))
        peer_layout = self._peers[source_engine_id][0]
        if direction == "pull":
            s_layout, t_layout = peer_layout, self.local_endpoint()
        elif direction == "push":
            s_layout, t_layout = self.local_endpoint(), peer_layout
        else:
            raise ValueError("direction must be 'pull' or 'push'")
        if stream is None:
            stream = self.swap_in_stream
        new_event = torch.cuda.Event()
        self._wait_source_events(stream, new_event, request_ids, source_events)
        args = (s_layout.handle, t_layout.handle, src, dst, grp, first, valid,
                _lib.mode_of(mode), stream.cuda_stream)
        if torch.cuda.current_device() == self.device_index:
            status, copied, extents = _lib.shim().migrate_blocks(*args)
        else:
            with torch.cuda.device(self.device_index):
                status, copied, extents = _lib.shim().migrate_blocks(*args)
        if status:
            _lib.check(status)
        new_event.record(stream)
        self.last_stats = (copied, extents)
        return new_event

    def copy_blocks_local(self, source_block_ids, target_block_ids, *, mode="auto",
                          stream=None) -> torch.cuda.Event:
        """Full-page copies between blocks of this same cache (on-GPU
        migration; HBM bound).  Overlapping source / target ids are ordered
        as a sequential loop would order them."""
        n = len(source_block_ids)
        if len(target_block_ids) != n:
            raise ValueError(f"source_block_ids has {n} ids but target_block_ids has "
                             f"{len(target_block_ids)}")
        ep = self.local_endpoint()
        stream = stream or torch.cuda.current_stream(self.device)
        ev = torch.cuda.Event()
        args = (ep.handle, ep.handle, _lib.ids_arg(source_block_ids),
                _lib.ids_arg(target_block_ids), [0] * n, [0] * n, [self.group_ratios[0]] * n,
                _lib.mode_of(mode), stream.cuda_stream)
        with torch.cuda.device(self.device_index):
            status, _, _ = _lib.shim().migrate_blocks(*args)
            if status:
                _lib.check(status)
            ev.record(stream)
        return ev

    def close(self) -> None:
        for eid in list(self._peers):
            self.unregister_kvcache_mem_handles(eid)
        if hasattr(self, "_local_ep"):
            self._local_ep.close()
        self._layout.close()
