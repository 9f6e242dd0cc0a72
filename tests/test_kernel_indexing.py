"""The copy kernels' work split, emulated on the host.

kvx_copy_vec / kvx_copy_bulk give each CTA a contiguous span of tiles
(cta_span), find the span's first item by binary search (find_item) and walk
forward; tile t of item i covers bytes [(t - tile_begin) * T, min(len, ...)).
This checks, for item tables built like the runtime builds them, that every
byte of every item is covered exactly once and never beyond the item, for a
range of grid sizes.  (Index arithmetic only; the kernels run in the GPU
tests.)
"""

import random

import pytest


def build_items(lengths, tile):
    items, tiles = [], 0
    max_item = 1 << 30
    for ln in lengths:
        done = 0
        while done < ln:
            n = min(ln - done, max_item)
            items.append((n, tiles))
            tiles += -(-n // tile)
            done += n
    return items, tiles


def cta_span(n_tiles, g, b):
    per, rem = divmod(n_tiles, g)
    t0 = b * per + min(b, rem)
    return t0, t0 + per + (1 if b < rem else 0)


def find_item(items, t):
    lo, hi = 0, len(items) - 1
    while lo < hi:
        mid = (lo + hi + 1) >> 1
        if items[mid][1] <= t:
            lo = mid
        else:
            hi = mid - 1
    return lo


@pytest.mark.parametrize("tile", [1 << 14, 1 << 15])
@pytest.mark.parametrize("seed", range(6))
def test_spans_cover_items_exactly_once(tile, seed):
    rng = random.Random(seed)
    lengths = [rng.choice([16, 48, tile - 16, tile, tile + 16, 3 * tile, 131072, 7])
               for _ in range(rng.randint(1, 60))]
    items, n_tiles = build_items(lengths, tile)
    for grid in (1, 2, 3, 7, 148, 1184, n_tiles, n_tiles + 5):
        grid = max(1, min(grid, n_tiles))
        covered = [0] * len(items)
        seen_tiles = 0
        for b in range(grid):
            t0, t1 = cta_span(n_tiles, grid, b)
            if t0 >= t1:
                continue
            i = find_item(items, t0)
            for t in range(t0, t1):
                while i + 1 < len(items) and items[i + 1][1] <= t:
                    i += 1
                ln, tb = items[i]
                off = (t - tb) * tile
                n = min(ln - off, tile)
                assert 0 < n and off + n <= ln
                covered[i] += n
                seen_tiles += 1
        assert seen_tiles == n_tiles
        assert covered == [ln for ln, _ in items]
