"""Transfer planning: which pages of a request move and which bytes of them.

Mirrors the planning half of the reference's block manager
(``aegaeon/block_manager.py``) with the same names and results:

* ``CacheGroupConfig`` (block_manager.py:133-266): allocation policy of one
  cache group and the live kernel-block extent of a page;
* ``CacheGroupRuntimeConfig`` (block_manager.py:269-343): the execution-side
  ratio and byte extents;
* ``BlockTable`` (block_manager.py:358-515): ``transfer_entries``,
  ``moved_group_blocks``, ``swap_metadata``, ``release_skipped_blocks``;
* ``plan_swap_lists`` (block_manager.py:1434-1478): the parallel
  src/dst/group/first/valid lists that ``swap_blocks`` consumes, with
  zero-length entries kept in the destination tables but dropped from the
  copy lists;
* ``plan_move_requests`` (block_manager.py:1355-1478): the whole list-building
  step of ``BlockManager.move_requests`` (request de-duplication, location,
  shape and cache-group checks, one destination reservation, table updates).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

from .cache_transfer import (
    byte_extent_for_kernel_blocks,
    kernel_block_extent_for_attention_page,
    logical_blocks_for_tokens,
    num_skipped_sliding_window_blocks,
    sliding_window_resident_block_bound,
)

LOGICAL_NULL_BLOCK_ID = -1
VLLM_NULL_BLOCK_ID = 0

_KINDS = ("attention", "mamba_none")


def _check_group(kind: str, physical: int, kernel: int, sliding_window: Optional[int],
                 what: str) -> None:
    if physical <= 0 or kernel <= 0:
        raise ValueError(
            f"Cache block sizes must both be positive: physical={physical}, kernel={kernel}"
            if what == "Cache"
            else f"KV-manager and kernel block sizes must both be positive: "
            f"kv={physical}, kernel={kernel}"
        )
    if kind == "attention":
        if physical % kernel:
            raise ValueError(
                f"Attention kernel block size {kernel} must divide "
                f"{'physical' if what == 'Cache' else 'KV-manager'} block size {physical}"
            )
    elif kind == "mamba_none":
        if physical != kernel:
            raise ValueError(
                "Mamba/GDN state pages cannot be split into kernel blocks"
                if what == "Cache"
                else "Mamba/GDN state pages cannot be split into virtual kernel blocks")
        if sliding_window is not None:
            raise ValueError("Mamba/GDN cache groups cannot have a sliding window")
    else:
        raise NotImplementedError(f"Unsupported cache group kind: {kind}")
    if sliding_window is not None and sliding_window <= 0:
        raise ValueError(f"sliding_window must be positive, got {sliding_window}")


@dataclass
class CacheGroupConfig:
    """Scheduler-side policy of one KV-cache group (block_manager.py:133-266).
    ``block_size`` is the physical (manager) block, ``kernel_block_size`` the
    attention kernel's page."""

    kind: str
    block_size: int
    kernel_block_size: int
    sliding_window: Optional[int] = None

    def __post_init__(self) -> None:
        _check_group(self.kind, self.block_size, self.kernel_block_size,
                     self.sliding_window, "Cache")

    def blocks_for_tokens(self, num_tokens: int) -> int:
        if num_tokens < 0:
            raise ValueError(f"num_tokens must be non-negative, got {num_tokens}")
        if self.kind == "mamba_none":
            return 1
        if self.sliding_window is None:
            return self.table_blocks_for_tokens(num_tokens)
        return sliding_window_resident_block_bound(num_tokens, self.block_size,
                                                   self.sliding_window)

    def table_blocks_for_tokens(self, num_tokens: int) -> int:
        if num_tokens < 0:
            raise ValueError(f"num_tokens must be non-negative, got {num_tokens}")
        if self.kind == "mamba_none":
            return 1
        return logical_blocks_for_tokens(num_tokens, self.block_size)

    def num_skipped_blocks(self, processed_computed_tokens: int) -> int:
        if processed_computed_tokens < 0:
            raise ValueError(
                "processed_computed_tokens must be non-negative, got "
                f"{processed_computed_tokens}"
            )
        if self.kind != "attention" or self.sliding_window is None:
            return 0
        return num_skipped_sliding_window_blocks(
            processed_computed_tokens, self.block_size, self.sliding_window)

    def block_is_skipped(self, processed_computed_tokens: int, logical_block_index: int) -> bool:
        if logical_block_index < 0:
            raise ValueError(
                f"logical_block_index must be non-negative, got {logical_block_index}")
        return logical_block_index < self.num_skipped_blocks(processed_computed_tokens)

    @property
    def kernel_blocks_per_physical_block(self) -> int:
        return self.block_size // self.kernel_block_size

    def kernel_block_extent(self, cached_tokens: int, block_index: int) -> Tuple[int, int]:
        """(first kernel page, live kernel-page count) of one physical page."""
        if self.kind == "mamba_none":
            return (0, 1)
        return kernel_block_extent_for_attention_page(
            cached_tokens, block_index, self.block_size, self.kernel_block_size,
            self.sliding_window)

    def valid_kernel_blocks(self, cached_tokens: int, block_index: int) -> int:
        if cached_tokens < 0:
            raise ValueError(f"cached_tokens must be non-negative, got {cached_tokens}")
        if block_index < 0:
            raise ValueError(f"block_index must be non-negative, got {block_index}")
        if self.kind == "mamba_none":
            return 1
        return self.kernel_block_extent(cached_tokens, block_index)[1]


@dataclass(frozen=True)
class CacheGroupRuntimeConfig:
    """Execution-side block-size contract of one group (block_manager.py:269-343)."""

    kind: str
    kv_block_size: int
    kernel_block_size: int
    sliding_window: Optional[int] = None

    def __post_init__(self) -> None:
        _check_group(self.kind, self.kv_block_size, self.kernel_block_size,
                     self.sliding_window, "KV")

    @property
    def blocks_per_kv_block(self) -> int:
        return self.kv_block_size // self.kernel_block_size

    def byte_extent_for_kernel_blocks(self, page_size_bytes: int, first_kernel_block: int,
                                      num_kernel_blocks: int) -> Tuple[int, int]:
        return byte_extent_for_kernel_blocks(page_size_bytes, self.blocks_per_kv_block,
                                             first_kernel_block, num_kernel_blocks)

    def bytes_for_kernel_blocks(self, page_size_bytes: int, valid_kernel_blocks: int) -> int:
        return self.byte_extent_for_kernel_blocks(page_size_bytes, 0, valid_kernel_blocks)[1]

    def to_kernel_block_ids(self, kv_block_ids: Sequence[int]) -> List[int]:
        """Physical ids -> attention-kernel ids (released columns map to the
        null block), block_manager.py:339-356."""
        if self.kind != "attention":
            return list(kv_block_ids)
        r = self.blocks_per_kv_block
        out: List[int] = []
        for b in kv_block_ids:
            out.extend([VLLM_NULL_BLOCK_ID] * r if b < 0 else range(b * r, b * r + r))
        return out


@dataclass
class BlockTable:
    """A request's pages per cache group (block_manager.py:358-515)."""

    location: int
    block_shape: Tuple[int, ...]
    cache_groups: Tuple[CacheGroupConfig, ...]
    group_blocks: List[List[int]]

    @property
    def blocks(self) -> List[int]:
        return [b for g in self.group_blocks for b in g if b != LOGICAL_NULL_BLOCK_ID]

    def release_skipped_blocks(self, processed_computed_tokens: int) -> List[int]:
        released: List[int] = []
        for group, blocks in zip(self.cache_groups, self.group_blocks):
            stop = min(group.num_skipped_blocks(processed_computed_tokens), len(blocks))
            for i in range(stop):
                if blocks[i] != LOGICAL_NULL_BLOCK_ID:
                    released.append(blocks[i])
                    blocks[i] = LOGICAL_NULL_BLOCK_ID
        return released

    def transfer_entries(self, processed_computed_tokens: int
                         ) -> List[Tuple[int, int, int, int, int]]:
        """Retained pages as (group, column, block id, first, count); count 0
        means "allocate at the destination, copy nothing"."""
        entries = []
        for gid, (group, blocks) in enumerate(zip(self.cache_groups, self.group_blocks)):
            for col, block_id in enumerate(blocks):
                if block_id == LOGICAL_NULL_BLOCK_ID or group.block_is_skipped(
                        processed_computed_tokens, col):
                    continue
                first, count = group.kernel_block_extent(processed_computed_tokens, col)
                entries.append((gid, col, block_id, first, count))
        return entries

    def moved_group_blocks(self, processed_computed_tokens: int,
                           target_block_ids: Sequence[int]) -> List[List[int]]:
        entries = self.transfer_entries(processed_computed_tokens)
        if len(entries) != len(target_block_ids):
            raise ValueError(
                f"Expected {len(entries)} target blocks, got {len(target_block_ids)}")
        moved = [[LOGICAL_NULL_BLOCK_ID] * len(b) for b in self.group_blocks]
        for (gid, col, _, _, _), target in zip(entries, target_block_ids):
            moved[gid][col] = target
        return moved

    def swap_metadata(self, cached_tokens: int) -> Tuple[List[int], List[int], List[int]]:
        live = [e for e in self.transfer_entries(cached_tokens) if e[4] > 0]
        return [e[0] for e in live], [e[3] for e in live], [e[4] for e in live]


@dataclass
class SwapLists:
    """Arguments of one ``swap_blocks`` call plus the destination tables."""

    source_block_ids: List[int]
    target_block_ids: List[int]
    group_ids: List[int]
    first_kernel_blocks: List[int]
    valid_kernel_blocks: List[int]
    release_source_block_ids: List[int]
    destination_tables: List[List[List[int]]]


def plan_swap_lists(plans: Sequence[Tuple[BlockTable, int]],
                    target_block_ids: Sequence[int]) -> SwapLists:
    """Copy lists for moving a batch of requests (block_manager.py:1419-1478).

    ``plans`` holds (block table, processed computed tokens) per request;
    ``target_block_ids`` the destination ids reserved for all retained pages
    of all requests, in order.  Zero-count pages get a destination id but no
    copy.  The tables are not modified.
    """
    out = SwapLists([], [], [], [], [], [], [])
    entries_per = [bt.transfer_entries(p) for bt, p in plans]
    need = sum(len(e) for e in entries_per)
    if need != len(target_block_ids):
        raise ValueError(f"Expected {need} target blocks, got {len(target_block_ids)}")
    cursor = 0
    for (bt, processed), entries in zip(plans, entries_per):
        targets = list(target_block_ids[cursor:cursor + len(entries)])
        cursor += len(entries)
        out.release_source_block_ids.extend(bt.blocks)
        for (gid, _, block_id, first, count), target in zip(entries, targets):
            if count <= 0:
                continue
            out.source_block_ids.append(block_id)
            out.target_block_ids.append(target)
            out.group_ids.append(gid)
            out.first_kernel_blocks.append(first)
            out.valid_kernel_blocks.append(count)
        out.destination_tables.append(bt.moved_group_blocks(processed, targets))
    return out


@dataclass
class MovePlan:
    """Everything ``move_requests`` decides for one batch: the requests that
    move, where the transfer runs, the parallel copy lists and the source
    ids to release once the move has completed."""

    swapped_request_ids: List[int]
    source_location: int
    target_location: int
    block_shape: Tuple[int, ...]
    engine_id: int
    is_swap_in: bool
    is_migration: bool
    source_block_ids: List[int]
    target_block_ids: List[int]
    group_ids: List[int]
    first_kernel_blocks: List[int]
    valid_kernel_blocks: List[int]
    release_source_block_ids: List[int]


def plan_move_requests(block_tables, requests, target_location: int, gpu_cache_groups,
                       reserve, *, allow_migration: bool = False) -> Optional[MovePlan]:
    """The list-building half of ``BlockManager.move_requests``
    (block_manager.py:1355-1478), with the same checks and results.

    ``block_tables`` maps request id -> BlockTable; ``requests`` are objects
    with ``request_id`` and ``get_first_new_token_index()``;
    ``gpu_cache_groups`` maps a GPU location to its cache-group tuple;
    ``reserve(n, location, block_shape)`` returns n free destination ids
    (the block manager's ``_get_free_blocks``).  Repeated requests count
    once and requests already at ``target_location`` are left alone.  The
    whole destination is reserved in one call before any table changes; then
    every moved table gets its destination ids and the target location.
    Retained pages with nothing to copy keep a destination id but stay out of
    the copy lists.  Returns None when nothing moves.

    GPU -> GPU moves raise NotImplementedError as in the reference unless
    ``allow_migration`` is set; then they produce a migration plan for
    ``KVSwapper.migrate_blocks`` run on the target GPU (pull).
    """
    moving = []  # (table, processed tokens, transfer entries)
    swapped: List[int] = []
    release: List[int] = []
    cur_loc: Optional[int] = None
    shape: Optional[Tuple[int, ...]] = None
    seen = set()
    for req in requests:
        rid = req.request_id
        if rid in seen:
            continue
        seen.add(rid)
        table = block_tables.get(rid, None)
        assert table, f"request {rid} not allocated"
        here = table.location
        if here == target_location:
            continue
        if here >= 0 and target_location >= 0 and not allow_migration:
            raise NotImplementedError("Migration is not implemented")
        if cur_loc is not None:
            assert here == cur_loc, f"request {rid} is on {here}; expected {cur_loc}"
        if shape is not None:
            assert table.block_shape == shape, f"request {rid}'s shape is not {shape}"
        cur_loc, shape = here, table.block_shape
        swapped.append(rid)
        if target_location >= 0 and table.cache_groups != gpu_cache_groups[target_location]:
            raise ValueError(f"request {rid} cache groups do not match target engine "
                             f"#{target_location}")
        processed = req.get_first_new_token_index()
        moving.append((table, processed, table.transfer_entries(processed)))
        release.extend(table.blocks)
    if not swapped:
        return None
    targets = list(reserve(sum(len(e) for _, _, e in moving), target_location, shape))
    plan = MovePlan(swapped, cur_loc, target_location, shape,
                    target_location if target_location >= 0 else cur_loc,
                    target_location >= 0 and cur_loc < 0, cur_loc >= 0 and target_location >= 0,
                    [], [], [], [], [], release)
    new_tables = []
    at = 0
    for table, processed, entries in moving:
        mine = targets[at:at + len(entries)]
        at += len(entries)
        for (gid, _, block_id, first, count), dst in zip(entries, mine):
            if count > 0:
                plan.source_block_ids.append(block_id)
                plan.target_block_ids.append(dst)
                plan.group_ids.append(gid)
                plan.first_kernel_blocks.append(first)
                plan.valid_kernel_blocks.append(count)
        new_tables.append(table.moved_group_blocks(processed, mine))
    for (table, _, _), groups in zip(moving, new_tables):
        table.group_blocks = groups
        table.location = target_location
    return plan
