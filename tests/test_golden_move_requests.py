"""BlockManager.move_requests list building (block_manager.py:1355-1478)
against the reference's own method run on a stub manager
(tests/golden/move_requests.json, written by tests/golden/make_golden.py).

Per move: the same outcome (True / False / exception type and message), the
same destination reservation (count, location, shape), the same swap_blocks
arguments (engine, request ids, source / target / group / first / valid
lists, direction), the same tables afterwards and the same released source
ids (the move event's source blocks).
"""

import pytest

from aegaeon_b200 import block_table as bt


class Req:
    def __init__(self, request_id, processed):
        self.request_id = request_id
        self._processed = processed

    def get_first_new_token_index(self):
        return self._processed


def scenarios(golden):
    data = golden("move_requests.json")
    specs = data["group_specs"]
    for sc in data["scenarios"]:
        yield specs, sc


def groups_of(specs, name):
    return tuple(bt.CacheGroupConfig(*g) for g in specs[name])


def test_move_requests_matches_reference(golden):
    checked = 0
    for specs, sc in scenarios(golden):
        tables = {t["request_id"]: bt.BlockTable(t["location"], tuple(t["block_shape"]),
                                                 groups_of(specs, t["groups"]),
                                                 [list(b) for b in t["group_blocks"]])
                  for t in sc["tables"]}
        gpu_groups = {int(k): groups_of(specs, v) for k, v in sc["gpu_groups"].items()}
        for m in sc["moves"]:
            pending = [list(r) for r in m["reserve"]]

            def reserve(n, location, shape):
                want = pending.pop(0)
                assert [n, location, list(shape)] == want[:3]
                return want[3]

            reqs = [Req(rid, p) for rid, p in m["requests"]]
            if "error" in m["result"]:
                exc = {"AssertionError": AssertionError, "ValueError": ValueError,
                       "NotImplementedError": NotImplementedError}[m["result"]["error"]]
                with pytest.raises(exc) as info:
                    bt.plan_move_requests(tables, reqs, m["target"], gpu_groups, reserve)
                assert str(info.value) == m["result"]["message"]
            else:
                plan = bt.plan_move_requests(tables, reqs, m["target"], gpu_groups, reserve)
                assert (plan is not None) == m["result"]["ok"]
                if plan is not None:
                    (engine, method, args), = m["rpc"]
                    assert method == "swap_blocks"
                    assert engine == plan.engine_id
                    assert args[0] == plan.swapped_request_ids
                    assert args[1] == plan.source_block_ids
                    assert args[2] == plan.target_block_ids
                    assert args[3] == plan.group_ids
                    assert args[4] == plan.first_kernel_blocks
                    assert args[5] == plan.valid_kernel_blocks
                    assert args[7] == plan.is_swap_in
                    ev = max(m["move_events"], key=lambda e: e[0])  # the newest event
                    assert ev[1:4] == [plan.source_location, plan.target_location,
                                       plan.release_source_block_ids]
                    assert ev[4] == plan.swapped_request_ids
                else:
                    assert m["rpc"] == []
            assert pending == []
            got = {str(rid): {"location": t.location,
                              "group_blocks": [list(b) for b in t.group_blocks]}
                   for rid, t in sorted(tables.items())}
            assert got == m["tables"]
            checked += 1
    assert checked >= 30


def test_migration_plan_when_enabled():
    """GPU -> GPU: the reference stops with NotImplementedError; with
    allow_migration the same lists become a pull migration on the target."""
    g = (bt.CacheGroupConfig("attention", 16, 16),)
    tables = {7: bt.BlockTable(0, (2, 16), g, [[11, 12, 13]])}
    with pytest.raises(NotImplementedError):
        bt.plan_move_requests(tables, [Req(7, 40)], 1, {0: g, 1: g}, lambda n, l, s: [0] * n)
    plan = bt.plan_move_requests(tables, [Req(7, 40)], 1, {0: g, 1: g},
                                 lambda n, l, s: list(range(100, 100 + n)),
                                 allow_migration=True)
    assert plan.is_migration and not plan.is_swap_in and plan.engine_id == 1
    assert plan.source_block_ids == [11, 12, 13]
    assert plan.target_block_ids == [100, 101, 102]
    assert tables[7].location == 1 and tables[7].group_blocks == [[100, 101, 102]]
