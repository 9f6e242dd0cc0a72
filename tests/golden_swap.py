"""Helpers to replay the swap_blocks golden scenarios (see make_golden.py)."""

import hashlib

import numpy as np


def owner_masks(scn):
    return [sum(1 << g for g in o) for o in scn["owners"]]


def group_ratios(scn):
    return [kv // kb for _, kv, kb in scn["groups"]]


def fresh_state(scn):
    segs = [np.frombuffer(bytes.fromhex(h), dtype=np.uint8).copy() for h in scn["init_segments"]]
    pool = np.frombuffer(bytes.fromhex(scn["init_pool"]), dtype=np.uint8).copy()
    return segs, pool


def row_bytes(scn):
    return sum(scn["pages"]) * scn["tp_size"]


def row_offset(scn):
    return scn["tp_rank"] * sum(scn["pages"])


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def check_step(step, segs, pool):
    assert sha(pool) == step["pool_sha256"]
    assert [sha(s) for s in segs] == step["segments_sha256"]
    if "pool" in step:
        assert pool.tobytes().hex() == step["pool"]
        assert [s.tobytes().hex() for s in segs] == step["segments"]
