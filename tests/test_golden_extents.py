"""Extent arithmetic against fixtures produced by the reference's own
cache_transfer.py / block_manager.py (tests/golden/make_golden.py)."""

import ctypes

import pytest

from aegaeon_b200 import block_table as bt
from aegaeon_b200 import cache_transfer as ct

FUNCS = [
    "logical_blocks_for_tokens",
    "sliding_window_resident_block_bound",
    "num_skipped_sliding_window_blocks",
    "kernel_block_extent_for_attention_page",
    "prefix_bytes_for_kernel_blocks",
    "byte_extent_for_kernel_blocks",
]


def run(fn, args):
    try:
        r = fn(*args)
        return {"ok": list(r) if isinstance(r, tuple) else r}
    except Exception as e:  # noqa: BLE001
        return {"error": type(e).__name__, "message": str(e)}


@pytest.mark.parametrize("name", FUNCS)
def test_python_mirror_matches_reference(golden, name):
    cases = golden("extents.json")[name]
    assert len(cases) > 20
    fn = getattr(ct, name)
    for args, expect in cases:
        assert run(fn, args) == expect, (name, args)


def test_native_extent_matches_reference(golden, kvx):
    """kvx_byte_extent (used by the copy planner) agrees with the reference on
    every case where the reference's arguments are representable (page >= 0)."""
    off, ln = ctypes.c_uint64(), ctypes.c_uint64()
    n = 0
    for (page, ratio, first, count), expect in golden("extents.json")["byte_extent_for_kernel_blocks"]:
        if page < 0:
            continue
        rc = kvx.kvx_byte_extent(page, ratio, first, count, ctypes.byref(off), ctypes.byref(ln))
        if "ok" in expect:
            assert rc == 0, (page, ratio, first, count, kvx.kvx_last_error())
            assert [off.value, ln.value] == expect["ok"]
        else:
            assert rc == 4, (page, ratio, first, count)
            assert kvx.kvx_last_error().decode() == expect["message"]
        n += 1
    assert n > 50


def test_oracle_extent_matches_reference(golden, oracle):
    for (page, ratio, first, count), expect in golden("extents.json")["byte_extent_for_kernel_blocks"]:
        if page < 0:
            continue
        if "ok" in expect:
            assert list(oracle.byte_extent(page, ratio, first, count)) == expect["ok"]
        else:
            with pytest.raises(ValueError):
                oracle.byte_extent(page, ratio, first, count)


def test_runtime_config_extents(golden):
    data = golden("block_tables.json")
    for (kind, kvb, kb, w, page, first, num), expect in data["runtime_extents"]:
        cfg = bt.CacheGroupRuntimeConfig(kind, kvb, kb, w)
        assert run(cfg.byte_extent_for_kernel_blocks, (page, first, num)) == expect
    for (kind, kvb, kb, w), ids in data["to_kernel_ids"]:
        assert bt.CacheGroupRuntimeConfig(kind, kvb, kb, w).to_kernel_block_ids([3, -1, 0, 7]) == ids


def test_block_tables(golden):
    for rec in golden("block_tables.json")["tables"]:
        groups = tuple(bt.CacheGroupConfig(*g) for g in rec["groups"])
        table = bt.BlockTable(0, (1,), groups, [list(b) for b in rec["group_blocks"]])
        p = rec["processed"]
        assert [list(e) for e in table.transfer_entries(p)] == rec["transfer_entries"]
        assert table.moved_group_blocks(p, rec["targets"]) == rec["moved"]
        assert [list(x) for x in table.swap_metadata(p)] == rec["swap_metadata"]
        assert table.blocks == rec["blocks"]
        assert table.release_skipped_blocks(p) == rec["released"]
        assert table.group_blocks == rec["after_release"]


def test_plan_swap_lists_drops_zero_count_entries(golden):
    recs = golden("block_tables.json")["tables"]
    plans, targets, expect_src = [], [], []
    for rec in recs[:12]:
        groups = tuple(bt.CacheGroupConfig(*g) for g in rec["groups"])
        table = bt.BlockTable(0, (1,), groups, [list(b) for b in rec["group_blocks"]])
        plans.append((table, rec["processed"]))
        targets += rec["targets"]
        expect_src += [e[2] for e in rec["transfer_entries"] if e[4] > 0]
    lists = bt.plan_swap_lists(plans, targets)
    assert lists.source_block_ids == expect_src
    assert len(lists.target_block_ids) == len(expect_src)
    assert all(v > 0 for v in lists.valid_kernel_blocks)
    assert [t for t in lists.destination_tables] == [
        rec["moved"] for rec in recs[:12]]
    with pytest.raises(ValueError):
        bt.plan_swap_lists(plans, targets[:-1])
