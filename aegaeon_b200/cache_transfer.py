"""Extent arithmetic for partial KV-page transfers.

Same functions, arguments, results and exceptions as the reference's
``aegaeon/cache_transfer.py`` (cited per function).  The copy path itself does
this arithmetic natively (``kvx_byte_extent`` / the planner in
``csrc/kvx_plan.cpp``); these Python versions serve the block-table planner
(``block_table.py``) and callers that plan on the host.
"""

from __future__ import annotations


def _require_positive_block_size(block_size: int) -> None:
    if block_size <= 0:
        raise ValueError(f"block_size must be positive, got {block_size}")


def logical_blocks_for_tokens(num_tokens: int, block_size: int) -> int:
    """Table columns that address positions [0, num_tokens)
    (cache_transfer.py:4-10)."""
    if num_tokens < 0:
        raise ValueError(f"num_tokens must be non-negative, got {num_tokens}")
    _require_positive_block_size(block_size)
    return -(-num_tokens // block_size)


def sliding_window_resident_block_bound(
    num_tokens: int, block_size: int, sliding_window: int
) -> int:
    """Pages a sliding-window request may keep resident: the current page plus
    the pages spanned by the W-1 committed tokens before it, capped by the
    table length (cache_transfer.py:13-28)."""
    if sliding_window <= 0:
        raise ValueError(f"sliding_window must be positive, got {sliding_window}")
    columns = logical_blocks_for_tokens(num_tokens, block_size)
    if columns == 0:
        return 0
    history_pages = -(-(sliding_window - 1) // block_size)
    return min(columns, history_pages + 1)


def num_skipped_sliding_window_blocks(
    processed_computed_tokens: int, block_size: int, sliding_window: int
) -> int:
    """Whole leading pages that the next query's window no longer sees
    (cache_transfer.py:31-45)."""
    if processed_computed_tokens < 0:
        raise ValueError(
            "processed_computed_tokens must be non-negative, got "
            f"{processed_computed_tokens}"
        )
    _require_positive_block_size(block_size)
    if sliding_window <= 0:
        raise ValueError(f"sliding_window must be positive, got {sliding_window}")
    invisible = processed_computed_tokens - (sliding_window - 1)
    return max(0, invisible) // block_size


def kernel_block_extent_for_attention_page(
    cached_tokens: int,
    physical_block_index: int,
    physical_block_size: int,
    kernel_block_size: int,
    sliding_window: int | None = None,
) -> tuple[int, int]:
    """(first kernel block, kernel-block count) of the live tokens inside one
    physical page; (0, 0) when the page holds no live token
    (cache_transfer.py:48-94).

    Live tokens are [max(0, cached - W + 1), cached) under a window W, else
    [0, cached); the next query brings its own K/V, so W-1 history tokens
    suffice.
    """
    if cached_tokens < 0:
        raise ValueError(f"cached_tokens must be non-negative, got {cached_tokens}")
    if physical_block_index < 0:
        raise ValueError(
            "physical_block_index must be non-negative, got " f"{physical_block_index}"
        )
    if physical_block_size <= 0 or kernel_block_size <= 0:
        raise ValueError("physical and kernel block sizes must be positive")
    if physical_block_size % kernel_block_size:
        raise ValueError(
            f"Kernel block size {kernel_block_size} must divide physical "
            f"block size {physical_block_size}"
        )
    if sliding_window is not None and sliding_window <= 0:
        raise ValueError(f"sliding_window must be positive, got {sliding_window}")

    page_start = physical_block_index * physical_block_size
    live_from = 0 if sliding_window is None else max(0, cached_tokens - sliding_window + 1)
    lo = max(page_start, live_from) - page_start
    hi = min(page_start + physical_block_size, cached_tokens) - page_start
    if hi <= lo:
        return (0, 0)
    first = lo // kernel_block_size
    last = -(-hi // kernel_block_size)
    return first, last - first


def valid_kernel_blocks_for_attention_page(
    cached_tokens: int,
    physical_block_index: int,
    physical_block_size: int,
    kernel_block_size: int,
) -> int:
    """Live kernel-page count of a full-attention page (cache_transfer.py:97-110)."""
    return kernel_block_extent_for_attention_page(
        cached_tokens, physical_block_index, physical_block_size, kernel_block_size
    )[1]


def prefix_bytes_for_kernel_blocks(
    page_size_bytes: int,
    kernel_blocks_per_page: int,
    valid_kernel_blocks: int,
) -> int:
    """Bytes of the first `valid_kernel_blocks` kernel pages of a backing page
    (cache_transfer.py:113-135)."""
    if page_size_bytes <= 0:
        raise ValueError(f"page_size_bytes must be positive, got {page_size_bytes}")
    if kernel_blocks_per_page <= 0:
        raise ValueError(
            "kernel_blocks_per_page must be positive, got " f"{kernel_blocks_per_page}"
        )
    if valid_kernel_blocks < 0 or valid_kernel_blocks > kernel_blocks_per_page:
        raise ValueError(
            f"valid kernel blocks {valid_kernel_blocks} outside [0, "
            f"{kernel_blocks_per_page}]"
        )
    per_kernel_block, rem = divmod(page_size_bytes, kernel_blocks_per_page)
    if rem:
        raise ValueError(
            f"Backing page size {page_size_bytes} is not divisible by "
            f"{kernel_blocks_per_page} kernel blocks"
        )
    return per_kernel_block * valid_kernel_blocks


def byte_extent_for_kernel_blocks(
    page_size_bytes: int,
    kernel_blocks_per_page: int,
    first_kernel_block: int,
    num_kernel_blocks: int,
) -> tuple[int, int]:
    """(byte offset, byte length) of kernel blocks [first, first+num) inside a
    backing page (cache_transfer.py:138-165)."""
    if first_kernel_block < 0:
        raise ValueError(
            f"first_kernel_block must be non-negative, got {first_kernel_block}"
        )
    stop = first_kernel_block + num_kernel_blocks
    if stop > kernel_blocks_per_page:
        raise ValueError(
            f"Kernel-block extent [{first_kernel_block}, {stop}) "
            f"exceeds page size {kernel_blocks_per_page}"
        )
    return (
        prefix_bytes_for_kernel_blocks(
            page_size_bytes, kernel_blocks_per_page, first_kernel_block
        ),
        prefix_bytes_for_kernel_blocks(
            page_size_bytes, kernel_blocks_per_page, num_kernel_blocks
        ),
    )
