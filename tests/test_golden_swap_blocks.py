"""Worker.swap_blocks semantics (worker.py:2204-2349) on CPU.

The fixtures hold the reference's own loop executed on CPU tensors.  Replayed
here through (1) the C oracle and (2) the native planner of libkvx.so, whose
(source, destination, bytes) copies are applied with memmove on host buffers.
"""

import ctypes

import numpy as np
import pytest

import golden_swap as gs
from aegaeon_b200 import swapper


def test_oracle_replays_reference(golden, oracle):
    for scn in golden("swap_blocks.json")["scenarios"]:
        segs, pool = gs.fresh_state(scn)
        for step in scn["steps"]:
            oracle.swap_blocks(segs, scn["pages"], scn["cpu_offsets"], gs.owner_masks(scn),
                               gs.group_ratios(scn), pool, gs.row_bytes(scn), gs.row_offset(scn),
                               step["source"], step["target"], step["groups"], step["first"],
                               step["valid"], step["is_swap_in"])
            gs.check_step(step, segs, pool)


def native_layout(scn, segs, pool):
    return swapper._Layout(
        0, [s.ctypes.data for s in segs], scn["pages"], [scn["num_blocks"]] * len(segs),
        scn["cpu_offsets"], gs.owner_masks(scn), gs.group_ratios(scn),
        pool.ctypes.data, pool.size, gs.row_bytes(scn), gs.row_offset(scn))


def plan(kvx, layout, step):
    a = swapper._entry_arrays(step["source"], step["target"], step["groups"], step["first"],
                              step["valid"])
    n = a[0]
    count = ctypes.c_int64(0)
    rc = kvx.kvx_plan_swap_blocks(layout.handle, n, *a[1:], int(step["is_swap_in"]),
                                  None, None, None, ctypes.byref(count))
    if rc:
        return rc, None
    m = count.value
    S, D, L = ((ctypes.c_uint64 * max(m, 1))() for _ in range(3))
    rc = kvx.kvx_plan_swap_blocks(layout.handle, n, *a[1:], int(step["is_swap_in"]), S, D, L,
                                  ctypes.byref(count))
    return rc, [(S[i], D[i], L[i]) for i in range(m)]


def test_native_planner_replays_reference(golden, kvx):
    for scn in golden("swap_blocks.json")["scenarios"]:
        segs, pool = gs.fresh_state(scn)
        layout = native_layout(scn, segs, pool)
        for step in scn["steps"]:
            rc, copies = plan(kvx, layout, step)
            assert rc == 0, kvx.kvx_last_error()
            for s, d, n in copies:
                ctypes.memmove(d, s, n)
            gs.check_step(step, segs, pool)
        layout.close()


def test_native_planner_errors_match_reference(golden, kvx):
    expected_status = {"ValueError": {2, 3, 4}, "IndexError": {5}}
    for scn in golden("swap_blocks.json")["scenarios"]:
        segs, pool = gs.fresh_state(scn)
        layout = native_layout(scn, segs, pool)
        for label, args, outcome in scn["errors"]:
            src, dst, grp, first, valid, inn = args
            assert "error" in outcome, label
            if label == "bad_lengths":
                with pytest.raises(ValueError):
                    swapper._entry_arrays(src, dst, grp, first, valid)
                continue
            rc, _ = plan(kvx, layout, dict(source=src, target=dst, groups=grp, first=first,
                                           valid=valid, is_swap_in=inn))
            assert rc in expected_status[outcome["error"]], (label, rc, outcome)
        layout.close()


def test_planner_issue_order_is_segment_major(kvx):
    """Copies come out segment by segment, entries in call order inside each
    (worker.py:2272-2329), so repeated targets resolve like the reference."""
    pages = [32, 64]
    segs = [np.zeros(4 * p, np.uint8) for p in pages]
    pool = np.zeros(3 * 96, np.uint8)
    lay = swapper._Layout(0, [s.ctypes.data for s in segs], pages, [4, 4], [0, 32], [1, 1], [1],
                          pool.ctypes.data, pool.size, 96, 0)
    rc, copies = plan(kvx, lay, dict(source=[2, 0], target=[1, 1], groups=[0, 0], first=[0, 0],
                                     valid=[1, 1], is_swap_in=False))
    assert rc == 0
    base0, base1, pb = segs[0].ctypes.data, segs[1].ctypes.data, pool.ctypes.data
    assert copies == [(base0 + 64, pb + 96, 32), (base0, pb + 96, 32),
                      (base1 + 128, pb + 128, 64), (base1, pb + 128, 64)]
    lay.close()


def test_layout_validation(kvx):
    pool = np.zeros(256, np.uint8)
    seg = np.zeros(64, np.uint8)
    with pytest.raises(ValueError, match="not owned"):
        swapper._Layout(0, [seg.ctypes.data], [16], [4], [0], [0], [1], pool.ctypes.data, 256, 64, 0)
    with pytest.raises(ValueError, match="beyond"):
        swapper._Layout(0, [seg.ctypes.data], [16], [4], [56], [1], [1], pool.ctypes.data, 256, 64, 0)
    with pytest.raises(ValueError, match="positive"):
        swapper._Layout(0, [seg.ctypes.data], [16], [4], [0], [1], [0], pool.ctypes.data, 256, 64, 0)
    with pytest.raises(ValueError, match="group >= 1"):
        swapper._Layout(0, [seg.ctypes.data], [16], [4], [0], [2], [1], pool.ctypes.data, 256, 64, 0)
