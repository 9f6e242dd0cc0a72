"""Destination reservation of the block manager: GPU free lists and the CPU
slab allocator, with the same choices of block ids as the reference.

Mirrors the allocator half of ``aegaeon/block_manager.py``:

* ``register_gpu_space`` (block_manager.py:718-792): a GPU engine's free list
  is ids 1 .. num_max_blocks-1 (id 0 is vLLM's null block);
* ``reserve`` (``_get_free_blocks``, :942-1031): GPU ids from the front of the
  engine's free list; CPU ids from the free deque of the block shape, which
  is topped up by carving whole slabs (the last free slab first) into block
  ranges, each id counted in its slab's usage;
* ``free`` (``free_blocks``, :1264-1277), ``reclaim_moved``
  (``_reclaim_gpu/cpu_move_blocks_once``, :661-689) and ``reclaim_cpu_slabs``
  (``_reclaim_cpu_slabs``, :918-940): ids back to the free lists, usage
  counts down, empty slabs back to the free slab list.

Where the reference awaits the completion of earlier moves before it gives
up (``_reclaim_gpu_move_blocks`` / ``_reclaim_cpu_move_blocks``, which wait
on the moves' CUDA events), ``reserve`` calls the ``reclaim`` hook the caller
passes (for example: wait on the moves' events, then ``reclaim_moved`` each).
The ids a reservation returns decide where a swap's host rows lie, and so
whether the swap's host runs are long (copy engines) or scattered (SM path).
"""

from __future__ import annotations

import math
from collections import defaultdict, deque
from typing import Callable, Dict, List, Optional, Sequence, Tuple

from .block_table import CacheGroupConfig

VLLM_NULL_BLOCK_ID = 0


def _prod(shape: Sequence[int]) -> int:
    out = 1
    for x in shape:
        out *= x
    return out


class BlockAllocator:
    """Free-block bookkeeping of one block manager (all GPU engines and the
    CPU slab pool)."""

    def __init__(self, cpu_num_slabs: int, cpu_slab_size_bytes: int, dtype_size: int = 2):
        self.dtype_size = dtype_size
        self.cpu_num_slabs = cpu_num_slabs
        self.cpu_slab_size_bytes = cpu_slab_size_bytes
        self.cpu_free_blocks: Dict[Tuple[int, ...], deque] = defaultdict(deque)
        self.cpu_free_slabs: List[int] = list(range(cpu_num_slabs))
        self.cpu_slab_usage: List[int] = [0] * cpu_num_slabs
        self.cpu_block_shape: List[Optional[Tuple[int, ...]]] = [None] * cpu_num_slabs
        self.gpu_block_shape: Dict[int, Tuple[int, ...]] = {}
        self.gpu_num_max_blocks: Dict[int, int] = {}
        self.gpu_cache_groups: Dict[int, Tuple[CacheGroupConfig, ...]] = {}
        self.gpu_free_blocks: Dict[int, List[int]] = {}

    # ---- sizes ----------------------------------------------------------------
    def block_size_bytes(self, block_shape: Sequence[int]) -> int:
        return _prod(block_shape) * self.dtype_size

    def slab_range(self, slab: int, block_size_bytes: int) -> Tuple[int, int]:
        """Ids of the blocks that lie wholly inside `slab`."""
        lo = math.ceil(slab * self.cpu_slab_size_bytes / block_size_bytes)
        hi = math.floor((slab + 1) * self.cpu_slab_size_bytes / block_size_bytes)
        return lo, hi

    def _slab_of(self, block: int, block_size_bytes: int) -> int:
        return block * block_size_bytes // self.cpu_slab_size_bytes

    # ---- GPU spaces -------------------------------------------------------------
    def register_gpu_space(self, engine_id: int, num_max_blocks: int,
                           block_shape: Tuple[int, ...],
                           cache_groups: Sequence[Tuple[str, int, int, Optional[int]]],
                           resident_request_ids: Sequence[int] = ()) -> None:
        """A GPU engine's cache space: every id but the null block free.
        ``resident_request_ids`` are requests whose tables still point into
        an earlier space of this engine (replacing it is then refused)."""
        if self.gpu_free_blocks.get(engine_id) is not None and resident_request_ids:
            raise ValueError(
                f"Error registering new GPU cache space for engine_id {engine_id}; "
                f"Request #{resident_request_ids[0]} still resides in the cache.")
        if num_max_blocks <= 1:
            raise ValueError("GPU cache must contain at least one usable block in addition "
                             "to vLLM's reserved NULL_BLOCK_ID")
        self.gpu_block_shape[engine_id] = tuple(block_shape)
        groups = tuple(
            CacheGroupConfig(kind, int(bs), int(kbs), None if w is None else int(w))
            for kind, bs, kbs, w in cache_groups)
        if not groups:
            raise ValueError("GPU cache must expose at least one cache group")
        self.gpu_cache_groups[engine_id] = groups
        self.gpu_num_max_blocks[engine_id] = num_max_blocks - 1
        self.gpu_free_blocks[engine_id] = list(range(VLLM_NULL_BLOCK_ID + 1, num_max_blocks))

    # ---- reservation --------------------------------------------------------------
    def _slabs_hold(self, block_size_bytes: int, needed: int) -> bool:
        if needed <= 0:
            return True
        for slab in self.cpu_free_slabs:
            lo, hi = self.slab_range(slab, block_size_bytes)
            needed -= hi - lo
            if needed <= 0:
                return True
        return False

    def reserve(self, num_blocks: int, location: int, block_shape: Tuple[int, ...],
                reclaim: Optional[Callable[[int, Tuple[int, ...]], None]] = None) -> List[int]:
        """`num_blocks` free ids at `location` (>= 0: a GPU engine, -1: the
        CPU pool), as ``_get_free_blocks`` chooses them.  When they are not
        there, ``reclaim(location, block_shape)`` may return ids of finished
        moves (through ``reclaim_moved``) before the last check; then
        ResourceWarning, with nothing taken."""
        shape = tuple(block_shape)
        bsb = self.block_size_bytes(shape)
        if location >= 0:
            assert location in self.gpu_free_blocks, f"unknown gpu location {location}"
            free = self.gpu_free_blocks[location]
            if len(free) < num_blocks:
                if reclaim is not None:
                    reclaim(location, shape)
                free = self.gpu_free_blocks[location]
                if len(free) < num_blocks:
                    raise ResourceWarning(f"not enough free blocks on GPU, requested "
                                          f"{num_blocks}, available {len(free)}")
            taken = free[:num_blocks]
            free[:] = free[num_blocks:]
            return taken
        free = self.cpu_free_blocks[shape]
        if not self._slabs_hold(bsb, num_blocks - len(free)):
            if reclaim is not None:
                reclaim(location, shape)
            free = self.cpu_free_blocks[shape]
            if not self._slabs_hold(bsb, num_blocks - len(free)):
                raise ResourceWarning(
                    f"not enough free blocks on CPU, requested {num_blocks}, available "
                    f"{len(free)} and {len(self.cpu_free_slabs)} slabs")
        while len(free) < num_blocks:
            slab = self.cpu_free_slabs.pop()
            lo, hi = self.slab_range(slab, bsb)
            self.cpu_block_shape[slab] = shape
            free.extend(range(lo, hi))
        taken = []
        for _ in range(num_blocks):
            block = free.popleft()
            self.cpu_slab_usage[self._slab_of(block, bsb)] += 1
            taken.append(block)
        return taken

    # ---- release ---------------------------------------------------------------------
    def free(self, location: int, block_shape: Tuple[int, ...], blocks: Sequence[int]) -> None:
        """A freed request's blocks (``BlockTable.blocks``) back to its
        location's free list."""
        shape = tuple(block_shape)
        if location >= 0:
            self.gpu_free_blocks[location].extend(blocks)
            return
        bsb = self.block_size_bytes(shape)
        self.cpu_free_blocks[shape].extend(blocks)
        for block in blocks:
            self.cpu_slab_usage[self._slab_of(block, bsb)] -= 1

    def reclaim_moved(self, source_location: int, block_shape: Tuple[int, ...],
                      source_blocks: Sequence[int]) -> int:
        """The source blocks of a finished move back to the free list of the
        location they were moved from; returns their number."""
        self.free(source_location, block_shape, source_blocks)
        return len(source_blocks)

    def reclaim_cpu_slabs(self) -> bool:
        """Slabs with no block in use return to the free slab list (their ids
        leave the shape's free deque); True if any did."""
        reclaimed = 0
        for slab, usage in enumerate(self.cpu_slab_usage):
            shape = self.cpu_block_shape[slab]
            if usage != 0 or shape is None:
                continue
            reclaimed += 1
            lo, hi = self.slab_range(slab, self.block_size_bytes(shape))
            free = self.cpu_free_blocks[shape]
            # keep the survivors in the deque's rotation order
            for _ in range(len(free)):
                block = free[0]
                if lo <= block < hi:
                    free.popleft()
                else:
                    free.rotate(-1)
            self.cpu_free_slabs.append(slab)
            self.cpu_block_shape[slab] = None
        return reclaimed > 0

    # ---- introspection ---------------------------------------------------------------
    def state(self) -> dict:
        return {
            "gpu_free_blocks": {str(k): list(v) for k, v in sorted(self.gpu_free_blocks.items())},
            "cpu_free_blocks": {str(list(k)): list(v)
                                for k, v in sorted(self.cpu_free_blocks.items()) if v},
            "cpu_free_slabs": list(self.cpu_free_slabs),
            "cpu_slab_usage": list(self.cpu_slab_usage),
            "cpu_block_shape": [None if s is None else list(s) for s in self.cpu_block_shape],
            "gpu_num_max_blocks": {str(k): v for k, v in sorted(self.gpu_num_max_blocks.items())},
        }
