"""The block manager's destination reservation (GPU free lists and CPU slab
allocator, aegaeon/block_manager.py:580-620, 653-689, 718-792, 918-1031,
1264-1277) against the reference's own methods
(tests/golden/block_allocator.json, written by tests/golden/make_golden.py).

Every step of the recorded script must give the same result (the block ids
chosen, or the same exception type and message) and leave the same allocator
state: GPU free lists, the CPU free deque of each block shape in its order,
free slabs, slab usage counts and slab shapes.
"""

import pytest

from aegaeon_b200.block_allocator import BlockAllocator

EXC = {"ValueError": ValueError, "ResourceWarning": ResourceWarning,
       "AssertionError": AssertionError}


def test_block_allocator_matches_reference(golden):
    data = golden("block_allocator.json")
    alloc = BlockAllocator(data["slabs"], data["slab_bytes"])
    results = []
    held = {}
    for step in data["steps"]:
        op = step["op"]
        picked = [results[op["from"]][i] for i in op["take"]] if "from" in op else None

        def run():
            kind = op["op"]
            if kind == "register":
                resident = [rid for rid, (loc, _, _) in held.items() if loc == op["engine"]]
                return alloc.register_gpu_space(op["engine"], op["num_max_blocks"],
                                                tuple(op["shape"]),
                                                [tuple(g) for g in op["groups"]], resident)
            if kind == "reserve":
                return alloc.reserve(op["n"], op["location"], tuple(op["shape"]))
            if kind == "free":
                return alloc.free(op["location"], tuple(op["shape"]), picked)
            if kind == "moved":
                return alloc.reclaim_moved(op["location"], tuple(op["shape"]), picked)
            if kind == "slabs":
                return alloc.reclaim_cpu_slabs()
            if kind == "hold":
                held[op["rid"]] = (op["location"], tuple(op["shape"]), picked)
                return None
            if kind == "release":
                loc, shape, blocks = held.pop(op["rid"])
                return alloc.free(loc, shape, blocks)
            raise AssertionError(kind)

        want = step["result"]
        if "error" in want:
            with pytest.raises(EXC[want["error"]]) as info:
                run()
            assert str(info.value) == want["message"], op
            results.append(None)
        else:
            out = run()
            assert out == want["ok"], op
            results.append(out)
        assert alloc.state() == step["state"], op


def test_reservations_feed_move_planning():
    """The allocator as plan_move_requests' reserve: a swap-out of two
    requests takes host slots from one slab in order (a contiguous run)."""
    from aegaeon_b200 import block_table as bt

    alloc = BlockAllocator(4, 1 << 20)
    alloc.register_gpu_space(0, 64, (2, 16, 8, 128), [("attention", 16, 16, None)])
    g = (bt.CacheGroupConfig("attention", 16, 16),)
    gpu_ids = alloc.reserve(6, 0, (2, 16, 8, 128))
    tables = {1: bt.BlockTable(0, (2, 16, 8, 128), g, [gpu_ids[:4]]),
              2: bt.BlockTable(0, (2, 16, 8, 128), g, [gpu_ids[4:]])}

    class Req:
        def __init__(self, rid):
            self.request_id = rid

        def get_first_new_token_index(self):
            return 64 if self.request_id == 1 else 32

    plan = bt.plan_move_requests(tables, [Req(1), Req(2)], -1, {0: g}, alloc.reserve)
    assert plan.source_block_ids == gpu_ids
    slots = plan.target_block_ids
    assert slots == list(range(slots[0], slots[0] + 6))  # one run: the copy engines' case
    assert tables[1].location == -1 and tables[1].group_blocks == [slots[:4]]
