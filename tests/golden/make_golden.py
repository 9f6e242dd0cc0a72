"""Generate golden fixtures by running the reference's own Python code.

Run where an Aegaeon checkout is present (its directory is the
AEGAEON_REFERENCE environment variable, else a directory named
``reference`` beside the repository root); the fixtures
it writes are committed and the tests never read the checkout.  Nothing is written into the checkout (the
reference logger writes ``output.log`` into the working directory, so this
script runs from a temporary one).

Fixtures:
  extents.json       cache_transfer.py helpers over a grid of arguments
                     (results, or exception type + message)
  block_tables.json  BlockTable.transfer_entries / moved_group_blocks /
                     swap_metadata and CacheGroupRuntimeConfig extents from
                     block_manager.py (``ray`` stubbed; it is not used there)
  block_allocator.json  BlockManager's free-block allocator (GPU free lists,
                     CPU slabs) through a scripted sequence of reservations,
                     frees, move reclaims and slab reclaims
  move_requests.json BlockManager.move_requests (block_manager.py:1355-1525)
                     run on a stub manager: request lists, reservations,
                     swap_blocks arguments, tables and move events per move
  swap_blocks.json   Worker.swap_blocks (worker.py:2204-2349), extracted from
                     the source with ``ast`` and executed on CPU tensors with
                     CUDA streams/events stubbed, on seeded byte contents:
                     the resulting host pool and GPU pages (hex) per step.

Usage:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import ast
import contextlib
import hashlib
import json
import os
import sys
import tempfile
import types

import numpy as np

OUT = os.path.dirname(os.path.abspath(__file__))
# The Aegaeon checkout: AEGAEON_REFERENCE, else a directory named "reference"
# beside this repository's root (tests/golden -> tests -> repo -> its parent).
REF = os.environ.get("AEGAEON_REFERENCE",
                     os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(OUT))),
                                  "reference"))


def stub_ray() -> None:
    ray = types.ModuleType("ray")
    ray.ObjectRef = object
    ray.remote = lambda *a, **k: (lambda f: f)
    ray.get = lambda x: x
    actor = types.ModuleType("ray.actor")
    actor.exit_actor = lambda: None
    ray.actor = actor
    sys.modules.setdefault("ray", ray)
    sys.modules.setdefault("ray.actor", actor)


def outcome(fn, *args):
    try:
        r = fn(*args)
        if isinstance(r, tuple):
            r = list(r)
        return {"ok": r}
    except Exception as e:  # noqa: BLE001 - the exception is the recorded result
        return {"error": type(e).__name__, "message": str(e)}


def gen_extents(ct) -> dict:
    cases = {k: [] for k in (
        "logical_blocks_for_tokens", "sliding_window_resident_block_bound",
        "num_skipped_sliding_window_blocks", "kernel_block_extent_for_attention_page",
        "prefix_bytes_for_kernel_blocks", "byte_extent_for_kernel_blocks")}
    for n in (-1, 0, 1, 15, 16, 17, 255, 256, 257, 1057):
        for bs in (-1, 0, 1, 16, 528):
            cases["logical_blocks_for_tokens"].append(
                [[n, bs], outcome(ct.logical_blocks_for_tokens, n, bs)])
            for w in (-3, 0, 1, 2, 16, 17, 100, 4096):
                cases["sliding_window_resident_block_bound"].append(
                    [[n, bs, w], outcome(ct.sliding_window_resident_block_bound, n, bs, w)])
                cases["num_skipped_sliding_window_blocks"].append(
                    [[n, bs, w], outcome(ct.num_skipped_sliding_window_blocks, n, bs, w)])
    for cached in (-1, 0, 15, 17, 100, 528, 529, 1057):
        for idx in (-1, 0, 1, 3):
            for pbs, kbs in ((16, 16), (528, 16), (64, 16), (48, 32), (0, 16)):
                for w in (None, -1, 1, 17, 600):
                    cases["kernel_block_extent_for_attention_page"].append(
                        [[cached, idx, pbs, kbs, w],
                         outcome(ct.kernel_block_extent_for_attention_page, cached, idx, pbs,
                                 kbs, w)])
    for page in (-16, 0, 17, 65536, 17301504 // 8):
        for ratio in (-1, 0, 1, 4, 33):
            for valid in (-1, 0, 1, 4, 34):
                cases["prefix_bytes_for_kernel_blocks"].append(
                    [[page, ratio, valid], outcome(ct.prefix_bytes_for_kernel_blocks, page,
                                                   ratio, valid)])
                for first in (-1, 0, 3):
                    cases["byte_extent_for_kernel_blocks"].append(
                        [[page, ratio, first, valid],
                         outcome(ct.byte_extent_for_kernel_blocks, page, ratio, first, valid)])
    return cases


def gen_block_tables(bm) -> dict:
    rng = np.random.default_rng(7)
    out = {"runtime_extents": [], "tables": []}
    for kind, kvb, kb, w in (("attention", 16, 16, None), ("attention", 528, 16, None),
                             ("attention", 64, 16, 40), ("mamba_none", 1, 1, None)):
        cfg = bm.CacheGroupRuntimeConfig(kind, kvb, kb, w)
        for page in (16, 4096, 17301504 // 8, 65536):
            for first in range(0, cfg.blocks_per_kv_block + 1, max(1, cfg.blocks_per_kv_block // 3)):
                for num in (0, 1, cfg.blocks_per_kv_block - first, cfg.blocks_per_kv_block + 1):
                    out["runtime_extents"].append(
                        [[kind, kvb, kb, w, page, first, num],
                         outcome(cfg.byte_extent_for_kernel_blocks, page, first, num)])
        out.setdefault("to_kernel_ids", []).append(
            [[kind, kvb, kb, w], cfg.to_kernel_block_ids([3, -1, 0, 7])])
    group_sets = [
        [("attention", 16, 16, None)],
        [("attention", 528, 16, None), ("mamba_none", 528, 528, None)],
        [("attention", 64, 16, 40), ("attention", 16, 16, None)],
        [("attention", 32, 16, 1)],
    ]
    for gs in group_sets:
        groups = tuple(bm.CacheGroupConfig(*g) for g in gs)
        for processed in (0, 1, 15, 16, 17, 63, 64, 65, 200, 529, 1100):
            blocks = []
            for g in groups:
                n = g.table_blocks_for_tokens(max(processed, 1))
                ids = [int(x) for x in rng.choice(10000, size=n, replace=False)]
                if g.sliding_window is not None and n > 2:
                    ids[0] = bm.LOGICAL_NULL_BLOCK_ID
                blocks.append(ids)
            bt = bm.BlockTable(0, (1,), groups, [list(b) for b in blocks])
            entries = bt.transfer_entries(processed)
            targets = [int(x) for x in rng.choice(10000, size=len(entries), replace=False)]
            rec = {
                "groups": gs, "processed": processed, "group_blocks": blocks,
                "transfer_entries": [list(e) for e in entries],
                "targets": targets,
                "moved": bt.moved_group_blocks(processed, targets),
                "swap_metadata": [list(x) for x in bt.swap_metadata(processed)],
                "blocks": bt.blocks,
            }
            bt2 = bm.BlockTable(0, (1,), groups, [list(b) for b in blocks])
            rec["released"] = bt2.release_skipped_blocks(processed)
            rec["after_release"] = bt2.group_blocks
            out["tables"].append(rec)
    return out


def load_swap_blocks(bm):
    """Worker.swap_blocks from worker.py, runnable on CPU tensors."""
    import torch

    src = open(os.path.join(REF, "aegaeon", "worker.py")).read()
    tree = ast.parse(src)
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "Worker")
    fn = next(n for n in cls.body if isinstance(n, ast.FunctionDef) and n.name == "swap_blocks")
    fn.decorator_list = []
    code = compile(ast.Module(body=[fn], type_ignores=[]), "worker.py", "exec")

    class FakeEvent:
        def __init__(self, *a, **k):
            pass

        def record(self, *a, **k):
            pass

    fake_cuda = types.SimpleNamespace(Event=FakeEvent, stream=lambda s: contextlib.nullcontext())

    class TorchProxy(types.ModuleType):
        def __getattr__(self, name):
            if name == "cuda":
                return fake_cuda
            return getattr(torch, name)

    class Logger:
        def info(self, *a, **k):
            pass

        debug = error = warning = info

    ray = sys.modules["ray"]
    ns = {"torch": TorchProxy("torch"), "ray": ray, "cudaStream_t": lambda x: x,
          "reduce_cuda_event": lambda *a: None, "logger": Logger()}
    exec(code, ns)
    return ns["swap_blocks"]


def gen_swap_blocks(bm) -> dict:
    import torch

    swap_blocks = load_swap_blocks(bm)
    scenarios = []
    specs = [
        # name, segment page bytes, owners, groups (kind, kv, kernel), gpu blocks,
        # host rows, tp (rank, size)
        ("hybrid", [64, 128, 64, 256], [[0], [0, 1], [1], [0]],
         [("attention", 64, 16), ("mamba_none", 16, 16)], 12, 10, (1, 2)),
        ("uniform", [96, 96, 96], [[0], [0], [0]], [("attention", 16, 16)], 9, 8, (0, 1)),
        ("ragged", [24, 48, 24], [[0], [0, 1], [1]], [("attention", 24, 8), ("mamba_none", 8, 8)],
         7, 6, (0, 1)),
    ]
    for name, pages, owners, groups, nblocks, nrows, (tp_rank, tp_size) in specs:
        rng = np.random.default_rng(11 + len(scenarios))
        descs = [bm.CacheGroupRuntimeConfig(k, kv, kb) for k, kv, kb in groups]
        composite = sum(pages)
        offsets = list(np.cumsum([0] + pages[:-1]))
        seg_init = [rng.integers(0, 256, size=nblocks * p, dtype=np.uint8) for p in pages]
        pool_init = rng.integers(0, 256, size=nrows * composite * tp_size, dtype=np.uint8)
        raw = {f"seg{i}": torch.from_numpy(seg_init[i].copy()).view(torch.int8)
               for i in range(len(pages))}
        pool = torch.from_numpy(pool_init.copy())
        view = pool.view(nrows, composite * tp_size)
        segs = [types.SimpleNamespace(layer_name=f"seg{i}", cpu_offset=int(offsets[i]),
                                      page_size_bytes=p) for i, p in enumerate(pages)]
        self = types.SimpleNamespace(
            cache_group_descriptors=descs,
            swap_in_stream=types.SimpleNamespace(cuda_stream=0),
            swap_out_stream=types.SimpleNamespace(cuda_stream=0),
            _wait_source_events=lambda *a, **k: None,
            composite_cache=types.SimpleNamespace(page_size_bytes=composite, segments=segs,
                                                  raw_tensors=raw),
            cache_segment_group_ids=[frozenset(o) for o in owners],
            parallel_config=types.SimpleNamespace(tensor_parallel_rank=tp_rank),
            kv_swap_view=view, cudart=None)
        steps = []
        for step in range(3):
            is_in = step == 1
            n = int(rng.integers(3, 7))
            dev_ids = [int(x) for x in rng.choice(nblocks, size=n, replace=False)]
            rows = [int(x) for x in rng.choice(nrows, size=n, replace=False)]
            gids, firsts, valids = [], [], []
            for _ in range(n):
                g = int(rng.integers(0, len(descs)))
                r = descs[g].blocks_per_kv_block
                f = int(rng.integers(0, r))
                v = int(rng.integers(0, r - f + 1))
                if step == 2:
                    f, v = 0, r
                gids.append(g)
                firsts.append(f)
                valids.append(v)
            srcs, dsts = (rows, dev_ids) if is_in else (dev_ids, rows)
            swap_blocks(self, list(range(n)), srcs, dsts, gids, firsts, valids, [None] * n, is_in)
            steps.append({
                "is_swap_in": is_in, "source": srcs, "target": dsts, "groups": gids,
                "first": firsts, "valid": valids,
                "pool_sha256": hashlib.sha256(pool.numpy().tobytes()).hexdigest(),
                "segments_sha256": [
                    hashlib.sha256(raw[f"seg{i}"].view(torch.uint8).numpy().tobytes()).hexdigest()
                    for i in range(len(pages))],
            })
        steps[-1]["pool"] = pool.numpy().tobytes().hex()
        steps[-1]["segments"] = [raw[f"seg{i}"].view(torch.uint8).numpy().tobytes().hex()
                                 for i in range(len(pages))]
        errors = []
        for label, args in (
            ("bad_group", ([0], [0], [len(descs)], [0], [1], False)),
            ("bad_extent", ([0], [0], [0], [descs[0].blocks_per_kv_block], [1], False)),
            ("bad_row", ([0], [nrows], [0], [0], [1], False)),
            ("bad_lengths", ([0, 1], [0], [0], [0], [1], False)),
        ):
            s_, d_, g_, f_, v_, inn = args
            errors.append([label, list(args),
                           outcome(swap_blocks, self, [0] * len(s_), s_, d_, g_, f_, v_,
                                   [None] * len(s_), inn)])
        scenarios.append({
            "name": name, "pages": pages, "owners": owners, "groups": groups,
            "num_blocks": nblocks, "num_rows": nrows, "tp_rank": tp_rank, "tp_size": tp_size,
            "cpu_offsets": [int(x) for x in offsets],
            "init_segments": [a.tobytes().hex() for a in seg_init],
            "init_pool": pool_init.tobytes().hex(), "steps": steps, "errors": errors,
        })
    return {"scenarios": scenarios}


class _Req:
    """The two members move_requests reads from a request."""

    def __init__(self, request_id, processed):
        self.request_id = request_id
        self._processed = processed

    def get_first_new_token_index(self):
        return self._processed


def gen_move_requests(bm) -> dict:
    """BlockManager.move_requests (block_manager.py:1355-1525) run on a stub
    manager: the reference's own BlockTable objects, a free-block reservation
    that hands out recorded ids, and a worker RPC that records its
    arguments.  Each scenario is a sequence of moves on one manager; per move
    the fixture keeps the request list, the target, the reservation calls,
    the swap_blocks arguments, the tables afterwards, the move event and the
    outcome (return value or exception)."""
    import asyncio
    import itertools
    from collections import defaultdict

    rng = np.random.default_rng(17)
    group_specs = {
        "uniform": [("attention", 16, 16, None)],
        "hybrid": [("attention", 528, 16, None), ("mamba_none", 528, 528, None)],
        "window": [("attention", 64, 16, 40), ("attention", 16, 16, None)],
        "w1": [("attention", 32, 16, 1)],
    }

    def groups_of(name):
        return tuple(bm.CacheGroupConfig(*g) for g in group_specs[name])

    def new_manager(gpu_groups):
        calls = {"reserve": [], "rpc": []}
        next_id = itertools.count(20000)

        async def get_free(n, location, shape):
            ids = [next(next_id) for _ in range(n)]
            calls["reserve"].append([n, location, list(shape), ids])
            return ids

        def rpc_for(engine):
            def call(method, *args):
                calls["rpc"].append([engine, method, [list(a) if isinstance(a, list) else a
                                                      for a in args]])
                return f"event-refs-{len(calls['rpc'])}"
            return call

        mgr = types.SimpleNamespace(
            block_tables={}, gpu_cache_groups={k: groups_of(v) for k, v in gpu_groups.items()},
            _get_free_blocks=get_free, latest_events={},
            remote_callables=defaultdict(lambda: None), event_counter=itertools.count(),
            move_gpu_num_blocks=defaultdict(int), move_events_gpu=defaultdict(list),
            move_cpu_num_blocks=defaultdict(int), move_events_cpu=defaultdict(list))
        for loc in list(gpu_groups) + [-1]:
            mgr.remote_callables[loc] = rpc_for(loc)
        return mgr, calls

    def add_table(mgr, rid, loc, shape, gname, processed):
        groups = groups_of(gname)
        blocks = []
        for g in groups:
            n = g.table_blocks_for_tokens(max(processed + int(rng.integers(0, 20)), 1))
            ids = [int(x) for x in rng.choice(10000, size=n, replace=False)]
            if g.sliding_window is not None and n > 2:
                ids[0] = bm.LOGICAL_NULL_BLOCK_ID
            blocks.append(ids)
        mgr.block_tables[rid] = bm.BlockTable(loc, tuple(shape), groups, blocks)
        return {"request_id": rid, "location": loc, "block_shape": list(shape), "groups": gname,
                "group_blocks": [list(b) for b in blocks]}

    def snapshot(mgr):
        return {str(rid): {"location": t.location, "group_blocks": [list(b) for b in t.group_blocks]}
                for rid, t in sorted(mgr.block_tables.items())}

    def move(mgr, calls, reqs, target):
        calls["reserve"].clear()
        calls["rpc"].clear()
        requests = [_Req(rid, p) for rid, p in reqs]
        try:
            result = {"ok": asyncio.run(bm.BlockManager.move_requests(mgr, requests, target))}
        except Exception as e:  # noqa: BLE001 - the exception is the recorded result
            result = {"error": type(e).__name__, "message": str(e)}
        events = [[ev.serial, ev.source_location, ev.target_location, list(ev.source_blocks),
                   [r.request_id for r in ev.requests]]
                  for d in (mgr.move_events_gpu, mgr.move_events_cpu) for evs in d.values()
                  for ev in evs]
        return {"requests": [list(r) for r in reqs], "target": target, "result": result,
                "reserve": [list(c) for c in calls["reserve"]],
                "rpc": [list(c) for c in calls["rpc"]], "tables": snapshot(mgr),
                "move_events": events,
                "move_gpu_num_blocks": {str(k): v for k, v in mgr.move_gpu_num_blocks.items()},
                "move_cpu_num_blocks": {str(list(k)): v for k, v in mgr.move_cpu_num_blocks.items()},
                "latest_events": sorted(mgr.latest_events)}

    scenarios = []
    for gname in group_specs:
        mgr, calls = new_manager({0: gname, 1: gname})
        tables = []
        procs = {}
        for rid in range(6):
            p = int(rng.choice([0, 1, 15, 16, 17, 63, 200, 529, 1100]))
            procs[rid] = p
            tables.append(add_table(mgr, rid, 0 if rid < 5 else -1, (2, 16), gname, p))
        moves = [
            # out: duplicates counted once; request 5 is already on the CPU
            move(mgr, calls, [(0, procs[0]), (1, procs[1]), (0, procs[0]), (2, procs[2]),
                              (5, procs[5])], -1),
            # in again, with a request already on the GPU mixed in
            move(mgr, calls, [(1, procs[1]), (3, procs[3]), (0, procs[0])], 0),
            # nothing to do
            move(mgr, calls, [(0, procs[0]), (3, procs[3])], 0),
            # GPU -> GPU is not implemented in the reference
            move(mgr, calls, [(4, procs[4])], 1),
            # mixed source locations
            move(mgr, calls, [(4, procs[4]), (2, procs[2])], 1),
            # unknown request
            move(mgr, calls, [(99, 0)], -1),
            # out and back in with more tokens processed
            move(mgr, calls, [(4, procs[4] + 40), (3, procs[3] + 40)], -1),
            move(mgr, calls, [(3, procs[3] + 41), (4, procs[4] + 41), (5, procs[5])], 0),
        ]
        scenarios.append({"groups": gname, "gpu_groups": {"0": gname, "1": gname},
                          "tables": tables, "moves": moves})
    # shape mismatch, and a target engine with other cache groups
    mgr, calls = new_manager({0: "uniform", 1: "window"})
    tables = [add_table(mgr, 0, 0, (2, 16), "uniform", 40),
              add_table(mgr, 1, 0, (2, 8), "uniform", 40),
              add_table(mgr, 2, -1, (2, 16), "uniform", 40),
              add_table(mgr, 3, 1, (2, 16), "uniform", 40)]
    moves = [move(mgr, calls, [(0, 40), (1, 40)], -1),
             move(mgr, calls, [(0, 40), (3, 40)], -1),
             move(mgr, calls, [(2, 40)], 1),
             move(mgr, calls, [(2, 40)], 0)]
    scenarios.append({"groups": "mixed", "gpu_groups": {"0": "uniform", "1": "window"},
                      "tables": tables, "moves": moves})
    return {"group_specs": group_specs, "scenarios": scenarios}


# The operation script of block_allocator.json: interpreted by gen_block_allocator
# on the reference's BlockManager and by tests/test_golden_block_allocator.py on
# the mirror.  "from"/"take" pick ids out of an earlier reservation's result.
SHAPE_A = [2, 16, 8, 128]   # 65,536-byte blocks
SHAPE_B = [2, 16, 4, 128]   # 32,768-byte blocks
ALLOC_OPS = [
    {"op": "register", "engine": 0, "num_max_blocks": 40, "shape": SHAPE_A,
     "groups": [["attention", 16, 16, None]]},
    {"op": "register", "engine": 1, "num_max_blocks": 1, "shape": SHAPE_A,
     "groups": [["attention", 16, 16, None]]},
    {"op": "register", "engine": 2, "num_max_blocks": 8, "shape": SHAPE_A, "groups": []},
    {"op": "reserve", "n": 10, "location": 0, "shape": SHAPE_A},
    {"op": "reserve", "n": 7, "location": -1, "shape": SHAPE_A},
    {"op": "reserve", "n": 3, "location": -1, "shape": SHAPE_B},
    {"op": "reserve", "n": 6, "location": -1, "shape": SHAPE_A},
    {"op": "free", "location": -1, "shape": SHAPE_A, "from": 4, "take": [0, 2, 5]},
    {"op": "free", "location": 0, "shape": SHAPE_A, "from": 3, "take": [9, 1, 4]},
    {"op": "reserve", "n": 5, "location": -1, "shape": SHAPE_A},
    {"op": "reserve", "n": 4, "location": 0, "shape": SHAPE_A},
    {"op": "moved", "location": -1, "shape": SHAPE_A, "from": 6, "take": [0, 1, 2, 3, 4, 5]},
    {"op": "moved", "location": 0, "shape": SHAPE_A, "from": 10, "take": [3, 0]},
    {"op": "slabs"},
    {"op": "free", "location": -1, "shape": SHAPE_B, "from": 5, "take": [0, 1, 2]},
    {"op": "slabs"},
    {"op": "reserve", "n": 30, "location": 0, "shape": SHAPE_A},
    {"op": "reserve", "n": 80, "location": -1, "shape": SHAPE_A},
    {"op": "reserve", "n": 12, "location": -1, "shape": SHAPE_B},
    {"op": "hold", "rid": 50, "location": 0, "shape": SHAPE_A, "from": 3, "take": [0]},
    {"op": "register", "engine": 0, "num_max_blocks": 40, "shape": SHAPE_A,
     "groups": [["attention", 16, 16, None]]},
    {"op": "release", "rid": 50},
    {"op": "register", "engine": 0, "num_max_blocks": 24, "shape": SHAPE_A,
     "groups": [["attention", 16, 16, None]]},
    {"op": "reserve", "n": 23, "location": 0, "shape": SHAPE_A},
    {"op": "reserve", "n": 1, "location": 0, "shape": SHAPE_A},
]
ALLOC_SLABS = 6
ALLOC_SLAB_BYTES = 300_000  # not a multiple of either block size: partial blocks at slab edges


def gen_block_allocator(bm) -> dict:
    """BlockManager's allocator (block_manager.py:580-620, 653-689, 718-792,
    918-1031, 1264-1277) run through ALLOC_OPS: each step's result (ids, or
    exception type and message) and the allocator state after it."""
    import asyncio
    from collections import deque

    bm.CudaRTLibrary = lambda: None  # the allocator never touches the CUDA runtime
    mgr = bm.BlockManager(ALLOC_SLABS, ALLOC_SLAB_BYTES)
    results = []

    def state():
        return {
            "gpu_free_blocks": {str(k): list(v) for k, v in sorted(mgr.gpu_free_blocks.items())},
            "cpu_free_blocks": {str(list(k)): list(v)
                                for k, v in sorted(mgr.cpu_free_blocks.items()) if v},
            "cpu_free_slabs": list(mgr.cpu_free_slabs),
            "cpu_slab_usage": list(mgr.cpu_slab_usage),
            "cpu_block_shape": [None if x is None else list(x) for x in mgr.cpu_block_shape],
            "gpu_num_max_blocks": {str(k): v for k, v in sorted(mgr.gpu_num_max_blocks.items())},
        }

    def table(loc, shape, blocks):
        return bm.BlockTable(loc, tuple(shape), (bm.CacheGroupConfig("attention", 16, 16),),
                             [list(blocks)])

    next_rid = [1000]
    steps = []
    for op in ALLOC_OPS:
        picked = None
        if "from" in op:
            src = results[op["from"]]
            picked = [src[i] for i in op["take"]]
        try:
            kind = op["op"]
            if kind == "register":
                mgr.register_gpu_space(op["engine"], op["num_max_blocks"], tuple(op["shape"]),
                                       [tuple(g) for g in op["groups"]], None)
                out = None
            elif kind == "reserve":
                out = asyncio.run(mgr._get_free_blocks(op["n"], op["location"],
                                                        tuple(op["shape"])))
            elif kind == "free":
                rid = next_rid[0]
                next_rid[0] += 1
                mgr.block_tables[rid] = table(op["location"], op["shape"], picked)
                mgr.free_blocks(rid)
                out = None
            elif kind == "moved":
                ev = bm.MoveEvent(0, [], tuple(op["shape"]), op["location"], 99, list(picked), [])
                if op["location"] >= 0:
                    out = mgr._reclaim_gpu_move_blocks_once(ev)
                else:
                    out = mgr._reclaim_cpu_move_blocks_once(ev)
            elif kind == "slabs":
                out = mgr._reclaim_cpu_slabs()
            elif kind == "hold":
                mgr.block_tables[op["rid"]] = table(op["location"], op["shape"], picked)
                out = None
            elif kind == "release":
                mgr.free_blocks(op["rid"])
                out = None
            result = {"ok": out}
        except Exception as e:  # noqa: BLE001 - the exception is the recorded result
            out = None
            result = {"error": type(e).__name__, "message": str(e)}
        results.append(out)
        steps.append({"op": op, "result": result, "state": state()})
    assert isinstance(mgr.cpu_free_blocks[tuple(SHAPE_A)], deque)
    return {"slabs": ALLOC_SLABS, "slab_bytes": ALLOC_SLAB_BYTES, "steps": steps}


def main() -> None:
    if not os.path.isdir(os.path.join(REF, "aegaeon")):
        sys.exit(f"reference checkout not found at {REF}")
    sys.path.insert(0, REF)
    stub_ray()
    cwd = os.getcwd()
    with tempfile.TemporaryDirectory() as tmp:
        os.chdir(tmp)
        try:
            import aegaeon.block_manager as bm
            import aegaeon.cache_transfer as ct

            fixtures = {
                "extents.json": gen_extents(ct),
                "block_tables.json": gen_block_tables(bm),
                "swap_blocks.json": gen_swap_blocks(bm),
                "move_requests.json": gen_move_requests(bm),
                "block_allocator.json": gen_block_allocator(bm),
            }
        finally:
            os.chdir(cwd)
    for name, data in fixtures.items():
        with open(os.path.join(OUT, name), "w") as f:
            json.dump({"generator": "tests/golden/make_golden.py",
                       "reference_files": {
                           "extents.json": "aegaeon/cache_transfer.py",
                           "block_tables.json": "aegaeon/block_manager.py",
                           "swap_blocks.json": "aegaeon/worker.py (Worker.swap_blocks)",
                           "move_requests.json": "aegaeon/block_manager.py "
                                                 "(BlockManager.move_requests)",
                           "block_allocator.json": "aegaeon/block_manager.py (BlockManager "
                                                   "allocator: register_gpu_space, "
                                                   "_get_free_blocks, free_blocks, reclaims)"}[name],
                       "data": data}, f, separators=(",", ":"))
        print(name, os.path.getsize(os.path.join(OUT, name)), "bytes")


if __name__ == "__main__":
    main()
