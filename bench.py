"""Benchmark of the KV-cache swap path (BASELINE.json's metric).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kvx|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)

Workload (N=1 and every rank at N>1): configuration 2 of BASELINE.json, the
Llama-2-7B-shaped per-GPU swap.  32 layers with separate K and V caches
[4096, 16, 32, 128] fp16 filled with U(-2,2) (64 segments, 32 GiB per GPU);
one step swaps 1024 random blocks out to host rows 0..1023 and 1024 other
random blocks in from host rows 1024..2047 (8 GiB each way), out and in on
the two swap streams, as the reference worker does.  Each rank swaps its own
cache (weak scaling, no collective on the data path).

Printed JSON line (rank 0): ``value`` is the device-timed box aggregate GB/s
(CUDA events on the launching streams, max over ranks); ``e2e`` is the same
metric timed by the wall clock through the public API from block tables
(plan_move_requests -> KVSwapper.swap_blocks -> wait), with the payload crossing
the host link inside the timed region.  ``roofline`` is the device-side
gather kernel against the measured HBM copy peak, with the binding host-link
roofline nested in it (``roofline.host_link``: the measured concurrent
copy-engine peak of all GPUs of the run and the host DRAM copy bandwidth).
At N=1 the line ends with ``baseline_configs``: configurations 1, 4 and 5,
both arms, each checked byte for byte.  At N >= 2 the ``migration`` (pull)
and ``migration_push`` objects add configuration 3 (NVLink P->D migration,
pairs (i, i+N/2)) with an exact cross-GPU comparison and a measured
peer-copy peak, and ``migration_summary`` ends the line.

``--impl reference`` times the reference's own swap op (ops/swap.cu, built
from the reference sources into oracle/_ref) on the same configuration and
the same ``config`` object: one call per K or V tensor, one cudaMemcpyAsync
per block, out and in on two streams.  Under torchrun every rank runs it on
its own GPU (one reference Worker per GPU) and the box aggregate uses the
slowest rank's time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "KV swap GB/s per GPU & box (1/2/4/8) vs host-link/NVLink roofline; switch ms"
GIB = 1 << 30
_OUT = sys.stdout


def emit(line: dict) -> None:
    """Print the result line on the real stdout."""
    _OUT.write(json.dumps(line) + "\n")
    _OUT.flush()


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["kvx", "reference"], default="kvx")
    p.add_argument("--ref-variant", choices=["op", "live-loop"], default="op",
                   help="reference arm, config 2: 'op' = the reference's compiled swap op "
                        "(one cudaMemcpyAsync per block and tensor); 'live-loop' = a "
                        "restatement of Worker.swap_blocks' hot loop (worker.py:2270-2329: "
                        "one torch copy_ per segment and block into composite host rows), "
                        "which cannot run as-is without Ray and vLLM")
    p.add_argument("--config", type=int, choices=[1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11], default=2,
                   help="BASELINE.json configuration (2 = the headline line; 3 is the "
                        "migration object of the N>=2 line; 7 = latency of small swap calls; "
                        "8 = migration transfer forms at N>=2; 9 = fragmented host slots, both "
                        "directions; 10 = copy-engine knobs on the headline step; 11 = weight "
                        "upload from pageable memory, both arms)")
    p.add_argument("--mode", default="auto", help="transfer mode: auto|sm|ce|ce_extent")
    p.add_argument("--blocks", type=int, default=1024, help="blocks per direction per step")
    p.add_argument("--cache-blocks", type=int, default=4096,
                   help="blocks per K/V tensor (4096 in the configuration; smaller only for "
                        "profiling captures)")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-migration", action="store_true")
    p.add_argument("--set", action="append", default=[], metavar="NAME=VALUE",
                   help="set a library tuning option (kvx_set_option) before running, e.g. "
                        "--set sm_ctas_host=296; may repeat")
    p.add_argument("--no-extras", action="store_true",
                   help="N=1: skip the configuration 1/4/5 objects of the default line")
    p.add_argument("--migration-direction", choices=["pull", "push"], default="pull",
                   help="pull: the decode rank copies from the prefill rank's mapped cache "
                        "(the reference's decode-side migrate_blocks); push: the prefill "
                        "rank stores into the decode rank's cache")
    return p.parse_args()


# ---- clocks -------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi samples of this rank's GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.uuid}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---- distributed plumbing -------------------------------------------------------
class Dist:
    def __init__(self, world: int, rank: int, local_rank: int):
        self.world, self.rank, self.local_rank = world, rank, local_rank

    @classmethod
    def init(cls, use_pg: bool):
        import torch

        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        if world > 1 and use_pg:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        return cls(world, rank, local)

    @property
    def active(self) -> bool:
        import torch.distributed as dist

        return self.world > 1 and dist.is_initialized()

    def barrier(self):
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        if self.active:
            dist.barrier()

    def max(self, x: float) -> float:
        import torch
        import torch.distributed as dist

        if not self.active:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        import torch
        import torch.distributed as dist

        if not self.active:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def gather_obj(self, obj):
        import torch.distributed as dist

        if not self.active:
            return [obj]
        out = [None] * self.world
        dist.all_gather_object(out, obj)
        return out

    def finish(self):
        import torch.distributed as dist

        if self.active:
            dist.barrier()
            dist.destroy_process_group()


def gpu_uuid(dev) -> str:
    import torch

    u = str(torch.cuda.get_device_properties(dev).uuid)
    return u if u.startswith("GPU-") else "GPU-" + u


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def host_link_peaks(dev, dist_=None) -> dict:
    """Copy-engine peaks of the host links of all GPUs of the run together:
    every rank copies 2 GiB of page-locked memory per direction as 256 MiB
    pieces back to back (single multi-GiB copies run slower on this link),
    H2D alone, D2H alone, and both at once.  All ranks start each window after
    a barrier; a window's box figure is (bytes of all ranks) / (slowest
    rank's device time).  Best of 10 windows after a warm-up (the host memory
    is shared with other jobs, and a few short windows can all land in a busy
    spell); values returned per GPU (box / N) plus the box figure of both
    directions."""
    import torch

    world = dist_.world if dist_ is not None else 1
    n = 2 * GIB
    piece = 256 << 20
    h1 = torch.empty(n, dtype=torch.uint8).pin_memory()
    h2 = torch.empty(n, dtype=torch.uint8).pin_memory()
    d1 = torch.empty(n, dtype=torch.uint8, device=dev)
    d2 = torch.empty(n, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def h2d():
        with torch.cuda.stream(s1):
            for o in range(0, n, piece):
                d1[o:o + piece].copy_(h1[o:o + piece], non_blocking=True)

    def d2h():
        with torch.cuda.stream(s2):
            for o in range(0, n, piece):
                h2[o:o + piece].copy_(d2[o:o + piece], non_blocking=True)

    def both():
        h2d()
        d2h()

    def timed(fn, nbytes):
        fn()  # warm-up: first touch of the pages by the copy engines
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(10):
            if dist_ is not None:
                dist_.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            cur = torch.cuda.current_stream()
            a.record(cur)
            s1.wait_stream(cur)
            s2.wait_stream(cur)
            fn()
            cur.wait_stream(s1)
            cur.wait_stream(s2)
            b.record(cur)
            b.synchronize()
            t = a.elapsed_time(b) / 1e3
            if dist_ is not None:
                t = dist_.max(t)
            best = max(best, nbytes * world / t / 1e9)
        return best

    box_h2d = timed(h2d, n)
    box_d2h = timed(d2h, n)
    box_bidir = timed(both, 2 * n)
    del h1, h2, d1, d2
    return {"h2d_gbs": box_h2d / world, "d2h_gbs": box_d2h / world,
            "bidir_gbs": box_bidir / world, "box_bidir_gbs": box_bidir}


# ---- configuration 2 state ---------------------------------------------------------
class SwapBench:
    def __init__(self, dev, blocks_per_dir: int, cache_blocks: int):
        import dataclasses

        import torch

        from aegaeon_b200 import swapper, workloads

        self.torch = torch
        self.shape = dataclasses.replace(workloads.CFG2, num_blocks=cache_blocks)
        sh = self.shape
        self.dev = dev
        self.per_dir = blocks_per_dir
        gen = torch.Generator(device=dev).manual_seed(0)
        self.pages = []
        for _ in range(sh.num_segments):
            t = torch.empty(sh.num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
            workloads.fill_segment(t, sh, gen)
            self.pages.append(t)
        segments, comp = swapper.make_segments(
            [((f"layer{i // 2}.{'kv'[i % 2]}",), sh.num_blocks * sh.page_bytes)
             for i in range(sh.num_segments)], sh.num_blocks)
        self.comp = comp
        self.segments = segments
        self.rows = 2 * blocks_per_dir
        self.pool = torch.empty(self.rows * comp, dtype=torch.uint8).pin_memory()
        # rows [per_dir, 2*per_dir) hold earlier swapped-out blocks (random bytes)
        fill = torch.empty(min(GIB, blocks_per_dir * comp), dtype=torch.uint8, device=dev)
        fill.random_(0, 256, generator=gen)
        tail = self.pool[blocks_per_dir * comp:]
        for o in range(0, tail.numel(), fill.numel()):
            n = min(fill.numel(), tail.numel() - o)
            tail[o:o + n].copy_(fill[:n])
        del fill
        self.sw = swapper.KVSwapper(dev.index, segments, self.pages,
                                    [frozenset({0})] * sh.num_segments, [1], kv_swap=self.pool)
        self.s_out = self.sw.swap_out_stream
        self.s_in = self.sw.swap_in_stream
        self.bytes_per_step = 2 * blocks_per_dir * comp

    def step_lists(self, step: int):
        from aegaeon_b200 import workloads

        out_ids, in_ids = workloads.swap_step_ids(self.shape.num_blocks, self.per_dir, step)
        rows_out = list(range(self.per_dir))
        rows_in = list(range(self.per_dir, 2 * self.per_dir))
        return out_ids, rows_out, rows_in, in_ids

    def issue(self, lists, mode):
        out_ids, rows_out, rows_in, in_ids = lists
        n = self.per_dir
        z, one = [0] * n, [1] * n
        e_out = self.sw.swap_blocks([0], out_ids, rows_out, z, z, one, [None], False,
                                    mode=mode, stream=self.s_out)
        e_in = self.sw.swap_blocks([1], rows_in, in_ids, z, z, one, [None], True,
                                   mode=mode, stream=self.s_in)
        return e_out, e_in

    def timed_device(self, steps: int, mode: str, lists_for):
        torch = self.torch
        cur = torch.cuda.current_stream(self.dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(cur)
        self.s_out.wait_event(a)
        self.s_in.wait_event(a)
        for k in range(steps):
            e_out, e_in = self.issue(lists_for(k), mode)
            # next step's swap-out may start once this step's swap-in is done
            # with its rows and vice versa: keep the two streams in lock-step
            self.s_out.wait_event(e_in)
            self.s_in.wait_event(e_out)
        cur.wait_stream(self.s_out)
        cur.wait_stream(self.s_in)
        b.record(cur)
        b.synchronize()
        return a.elapsed_time(b) / 1e3

    def live_one_direction(self, lists, mode: str) -> tuple:
        """Swap-out steps alone (nothing on the swap-in stream), with kernel
        timing on: the staging kernel's live launch duration without the other
        direction's kernels and copy-engine DMA beside it.  Returns
        kvx_kernel_timing_read's (launches, total ms, busy ms, bytes)."""
        from aegaeon_b200 import _lib

        n = self.per_dir
        z, one = [0] * n, [1] * n
        self.s_out.synchronize()
        self.s_in.synchronize()
        _lib.kernel_timing_read()
        _lib.kernel_timing(True)
        for out_ids, rows_out, _, _ in lists:
            self.sw.swap_blocks([0], out_ids, rows_out, z, z, one, [None], False, mode=mode,
                                stream=self.s_out)
        self.s_out.synchronize()
        _lib.kernel_timing(False)
        return _lib.kernel_timing_read()

    def timed_e2e(self, steps: int, mode: str):
        """Wall clock through the public API from block tables: the
        move_requests list building (plan_move_requests) for the outgoing and
        the incoming requests, then KVSwapper.swap_blocks per direction."""
        from aegaeon_b200 import block_table as bt

        group = (bt.CacheGroupConfig("attention", 16, 16),)
        per_req = 16  # 256-token requests: 16 full pages each

        class Req:
            def __init__(self, rid):
                self.request_id = rid

            def get_first_new_token_index(self):
                return 256

        t0 = time.perf_counter()
        for k in range(steps):
            out_ids, rows_out, rows_in, in_ids = self.step_lists(1000 + k)
            n_req = self.per_dir // per_req
            tables = {r: bt.BlockTable(0, (1,), group, [out_ids[r * per_req:(r + 1) * per_req]])
                      for r in range(n_req)}
            tables.update({n_req + r: bt.BlockTable(-1, (1,), group,
                                                    [rows_in[r * per_req:(r + 1) * per_req]])
                           for r in range(n_req)})
            lo = bt.plan_move_requests(tables, [Req(r) for r in range(n_req)], -1,
                                       {0: group}, lambda n, loc, shape: rows_out[:n])
            li = bt.plan_move_requests(tables, [Req(n_req + r) for r in range(n_req)], 0,
                                       {0: group}, lambda n, loc, shape: in_ids[:n])
            e_out = self.sw.swap_blocks(lo.swapped_request_ids, lo.source_block_ids,
                                        lo.target_block_ids, lo.group_ids,
                                        lo.first_kernel_blocks, lo.valid_kernel_blocks,
                                        [None] * n_req, lo.is_swap_in, mode=mode,
                                        stream=self.s_out)
            e_in = self.sw.swap_blocks(li.swapped_request_ids, li.source_block_ids,
                                       li.target_block_ids, li.group_ids,
                                       li.first_kernel_blocks, li.valid_kernel_blocks,
                                       [None] * n_req, li.is_swap_in, mode=mode,
                                       stream=self.s_in)
            self.s_out.wait_event(e_in)
            self.s_in.wait_event(e_out)
        self.s_out.synchronize()
        self.s_in.synchronize()
        return time.perf_counter() - t0

    def kernel_roofline(self, mode_bulk: bool) -> dict:
        """Device-side gather kernel alone: the 1024 blocks of a step copied
        HBM->HBM into another cache (the kernel the copy-engine mode uses to
        gather into / scatter from staging)."""
        torch = self.torch
        from aegaeon_b200 import _lib, swapper

        sh = self.shape
        n = self.per_dir
        dst_pages = [torch.empty(n * sh.page_bytes, dtype=torch.uint8, device=self.dev)
                     for _ in range(sh.num_segments)]
        segs, _ = swapper.make_segments([((f"d{i}",), n * sh.page_bytes)
                                         for i in range(sh.num_segments)], n)
        dst = swapper.KVSwapper(self.dev.index, segs, dst_pages,
                                [frozenset({0})] * sh.num_segments, [1])
        src_ep, dst_ep = self.sw.local_endpoint(), dst.local_endpoint()
        ids = self.step_lists(0)[0]
        arr = swapper._entry_arrays(ids, list(range(n)), [0] * n, [0] * n, [1] * n)
        mode = _lib.mode_of("sm_bulk" if mode_bulk else "sm")
        cur = torch.cuda.current_stream(self.dev)

        def run():
            _lib.check(_lib.lib().kvx_migrate_blocks(src_ep.handle, dst_ep.handle, *arr, mode,
                                                     cur.cuda_stream, None, None))

        for _ in range(3):
            run()
        torch.cuda.synchronize()
        times = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # keep the GPU busy while the host plans, so the window holds the kernel only
            torch.cuda._sleep(200_000_000)
            a.record(cur)
            run()
            b.record(cur)
            b.synchronize()
            times.append(a.elapsed_time(b) / 1e3)
        dst.close()
        del dst_pages
        t = statistics.median(times)
        payload = n * self.comp
        return {"kernel": "kvx_copy_bulk" if mode_bulk else "kvx_copy_vec<device>",
                "seconds": t, "payload_bytes": payload, "algorithmic_bytes": 2 * payload}

    def close(self):
        self.sw.close()


def host_facts() -> dict:
    """Host-side limits that bound the box aggregate of the swap: memory,
    NUMA nodes, page-locking limit and CPU model."""
    import resource

    facts = {"cpus": len(os.sched_getaffinity(0))}
    try:
        mem = {l.split(":")[0]: int(l.split()[1]) for l in open("/proc/meminfo")
               if l.startswith(("MemTotal", "MemAvailable"))}
        facts["mem_total_gib"] = round(mem["MemTotal"] / (1 << 20), 1)
        facts["mem_available_gib"] = round(mem["MemAvailable"] / (1 << 20), 1)
    except (OSError, KeyError, ValueError, IndexError):
        pass
    try:
        nodes = [d for d in os.listdir("/sys/devices/system/node") if d.startswith("node")]
        facts["numa_nodes"] = len(nodes)
    except OSError:
        pass
    soft, _ = resource.getrlimit(resource.RLIMIT_MEMLOCK)
    facts["memlock"] = "unlimited" if soft == resource.RLIM_INFINITY else soft
    try:
        facts["cpu"] = [l for l in open("/proc/cpuinfo")
                        if l.startswith("model name")][0].split(":")[1].strip()
    except (OSError, IndexError):
        pass
    return facts


def host_dram_copy_gbs(nbytes: int = 4 * GIB) -> float:
    """Host DRAM copy bandwidth on all host threads (torch's parallel CPU
    copy between two page-locked buffers): bytes copied per second, each byte
    read once and written once.  Best of 5 after a warm-up."""
    import torch

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    a = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    b = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    a.fill_(1)
    b.copy_(a)
    best = 0.0
    for _ in range(5):
        t0 = time.perf_counter()
        b.copy_(a)
        best = max(best, nbytes / (time.perf_counter() - t0) / 1e9)
    del a, b
    return best


def cpu_baseline(seconds: float) -> dict:
    """The reference's CPU path over the configuration-2 mapping: per K/V
    tensor, swap-out as torch.index_select of the 1024 out-going blocks into a
    host slot tensor and swap-in as index_copy_ of 1024 slots into the cache,
    on all host threads.  Bounded sample: 4 of the 64 [4096,16,32,128] fp16
    tensors (2 GiB of host cache) and the step-0 block ids, repeated for about
    `seconds`.  The builder's threaded C gather (oracle/) is reported beside
    it."""
    import torch

    from aegaeon_b200 import workloads

    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    sh = workloads.CFG2
    n_t = 4
    g = torch.Generator().manual_seed(0)
    shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
    caches = [torch.empty(shape, dtype=sh.dtype).uniform_(-2.0, 2.0, generator=g)
              for _ in range(n_t)]
    out_ids, in_ids = workloads.swap_step_ids(sh.num_blocks, 1024, 0)
    oi = torch.tensor(out_ids, dtype=torch.int64)
    ii = torch.tensor(in_ids, dtype=torch.int64)
    slots = torch.empty((1024,) + shape[1:], dtype=sh.dtype)
    incoming = torch.empty((1024,) + shape[1:], dtype=sh.dtype).uniform_(-2.0, 2.0, generator=g)

    def once():
        for c in caches:
            torch.index_select(c, 0, oi, out=slots)
            c.index_copy_(0, ii, incoming)

    once()  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        once()
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    moved = reps * n_t * 2 * 1024 * sh.page_bytes
    # exactness of the sample: the last swap-out holds the out-going blocks
    exact = bool(torch.equal(slots, caches[-1][oi]))
    del caches, slots, incoming
    port = None
    try:
        port = _c_port_gather(min(seconds, 5.0), threads)
    except Exception:  # noqa: BLE001 - the side figure is optional
        pass
    facts = host_facts()
    return {"value": moved / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "path": "torch.index_select (swap-out) + index_copy_ (swap-in) per K/V tensor "
                    "over the cfg2 block mapping: the reference CPU path north_star names",
            "bit_exact": exact, "c_port_gather_gbs": port,
            "sample": f"{reps} x (4 of 64 cfg2 tensors x [1024 out + 1024 in] x 128 KiB "
                      f"blocks), {threads} threads, {dt:.1f} s; cpu {facts.get('cpu')}"}


def _c_port_gather(seconds: float, threads: int) -> float:
    """The builder's threaded C block gather (test-infrastructure oracle) on
    the same kind of mapping: GB/s."""
    import numpy as np
    import torch

    from oracle import oracle as orc

    page, nsrc, ngather = 131072, 16384, 4096
    src = np.empty(nsrc * page, np.uint8)
    src[::4096] = 1
    dst = np.empty(ngather * page, np.uint8)
    ids = torch.randperm(nsrc, generator=torch.Generator().manual_seed(0))[:ngather].tolist()
    slots = list(range(ngather))
    orc.copy_blocks_mt(ids, slots, src, dst, page, threads)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < seconds:
        orc.copy_blocks_mt(ids, slots, src, dst, page, threads)
        reps += 1
    return reps * ngather * page / (time.perf_counter() - t0) / 1e9


MIGRATION_SMALL_BLOCKS = (1, 4, 16, 64)
# Measured peer copy per direction on this pool's 8xB200 nodes, as published
# with the pool's profiling notes; reported beside the nominal 900 GB/s.
POOL_PEER_COPY_GBS = 770.0


def _pair_exact(dist_, dev, pages, page: int, ids, is_src: bool, partner: int) -> bool:
    """Position-keyed comparison of the moved blocks across a pair: each side
    gathers its blocks in plan order (entry i = all segments of its i-th
    block; torch indexing, independent of the copy path), the prefill rank
    sends its gather over NCCL and the decode rank compares byte for byte.
    Returns, on every rank, whether every pair matched."""
    import torch
    import torch.distributed as dist

    idx = torch.tensor(ids, device=dev)
    mine = torch.cat([p.view(-1, page)[idx] for p in pages], dim=1).contiguous()
    ok = True
    if is_src:
        dist.send(mine, dst=partner)
    else:
        theirs = torch.empty_like(mine)
        dist.recv(theirs, src=partner)
        ok = bool(torch.equal(mine, theirs))
        del theirs
    del mine
    torch.cuda.synchronize()
    return all(x for x in dist_.gather_obj(ok))


def _peer_copy_peak(dist_, sw, partner: int, direction: str, active: bool, stream, blocks: int,
                    segments: int, page: int, streams: int = 1) -> dict:
    """Copy-engine peer copy between the pair, same direction and same
    mapped caches as the migration: blocks [0, blocks) of every segment, which
    coalesce into one plain cudaMemcpyAsync per segment (mode ce_extent), in
    barrier-started windows; best of 5, slowest rank.  With streams > 1 the
    block range is split into that many parts, each on its own stream (each
    stream may feed another copy engine)."""
    import torch

    dev = torch.device("cuda", sw.device_index)
    parts = [list(range(k * blocks // streams, (k + 1) * blocks // streams))
             for k in range(streams)]
    extra = [stream] + [torch.cuda.Stream(dev) for _ in range(streams - 1)]

    def run():
        if not active:
            return
        ev = torch.cuda.Event()
        ev.record(stream)
        for q, ids in zip(extra, parts):
            q.wait_event(ev)
            sw.migrate_blocks([0], partner, ids, ids, None, direction=direction,
                              mode="ce_extent", stream=q)
        for q in extra[1:]:
            stream.wait_stream(q)

    run()
    torch.cuda.synchronize(dev)
    nbytes = blocks * segments * page
    best = 0.0
    for _ in range(5):
        dist_.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        run()
        run()
        b.record(stream)
        b.synchronize()
        t = dist_.max(a.elapsed_time(b) / 1e3)
        best = max(best, 2 * nbytes / t / 1e9)
    return {"per_pair_gbs": best, "bytes": nbytes,
            "how": f"copy engine: one cudaMemcpyAsync per segment ({segments} x "
                   f"{blocks * page} B) between the mapped caches, issued by the active rank "
                   f"on {streams} stream(s), best of 5 windows"}


def _ipc_event_ordering(dist_, dev, sw, pages, page: int, plan, is_src: bool, partner: int,
                        pair: int, stream) -> bool:
    """worker.py:2351-2394 across processes: the prefill rank swaps new
    bytes into the plan's source blocks from host rows and ships the swap's
    interprocess event handle at once (before the swap has finished); the
    decode rank pulls the blocks after waiting on that event.  The pulled
    blocks must equal the swapped-in ones (position-keyed exact check)."""
    import torch

    from aegaeon_b200 import swapper

    n = plan.num_blocks
    handle = None
    if is_src:
        comp = len(pages) * page
        pool = torch.empty(n * comp, dtype=torch.uint8, pin_memory=True)
        g = torch.Generator(device=dev).manual_seed(4242 + pair)
        fill = torch.empty(min(n * comp, GIB), dtype=torch.uint8, device=dev)
        for o in range(0, pool.numel(), fill.numel()):
            fill.random_(0, 256, generator=g)
            pool[o:o + fill.numel()].copy_(fill[:pool.numel() - o])
        del fill
        segs, _ = swapper.make_segments([((f"l{i}",), p.numel()) for i, p in enumerate(pages)],
                                        pages[0].numel() // page)
        writer = swapper.KVSwapper(dev.index, segs, pages, [frozenset({0})] * len(pages), [1],
                                   kv_swap=pool)
        torch.cuda.synchronize()
        dist_.barrier()
        rows = list(range(n))
        handle = writer.swap_blocks([pair], rows, plan.source_ids, [0] * n, [0] * n, [1] * n,
                                    [None], True, return_handle=True)
    else:
        dist_.barrier()
    handles = dist_.gather_obj(handle)
    if not is_src:
        sw.migrate_blocks([pair], partner, plan.source_ids, plan.target_ids, [handles[partner]],
                          direction="pull", stream=stream)
    torch.cuda.synchronize()
    ok = _pair_exact(dist_, dev, pages, page, plan.source_ids if is_src else plan.target_ids,
                     is_src, partner)
    if is_src:
        writer.close()
        del pool
    return ok


def migration_bench(dist_, dev, steps: int, warmup: int, direction: str = "pull",
                    ipc_check: bool = False, mode: str = "auto", extras: bool = True,
                    split: float = 0.5) -> dict:
    """Configuration 3 at N >= 2: pairs (i, i + N/2), rank i the prefill side.
    pull: the decode rank maps the prefill rank's cache and copies the blocks
    in (loads over NVLink); push: the prefill rank stores them into the
    decode rank's mapped cache; split: both at once on disjoint entries, the
    prefill rank pushing the first `split` fraction and the decode rank
    pulling the rest."""
    import torch

    from aegaeon_b200 import swapper, workloads

    sh = workloads.CFG3
    half = dist_.world // 2
    gen = torch.Generator(device=dev).manual_seed(100 + dist_.rank)
    pages = []
    for _ in range(sh.num_segments):
        t = torch.empty(sh.num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
        workloads.fill_segment(t, sh, gen)
        pages.append(t)
    segs, _ = swapper.make_segments([((f"l{i}",), sh.num_blocks * sh.page_bytes)
                                     for i in range(sh.num_segments)], sh.num_blocks)
    sw = swapper.KVSwapper(dev.index, segs, pages, [frozenset({0})] * sh.num_segments, [1])
    handles = dist_.gather_obj(sw.export_kvcache_mem_handles())
    is_src = dist_.rank < half
    partner = dist_.rank + half if is_src else dist_.rank - half
    pair = min(dist_.rank, partner)
    plan = workloads.migration_plan(sh, requests=8, seed=0, pair=pair)
    nbytes = plan.num_blocks * sh.composite_bytes
    active = (is_src if direction == "push" else not is_src) or direction == "split"
    # both sides map the partner: the pull of the event-ordering check and the
    # push both need it
    sw.register_kvcache_mem_handles(partner, None, handles[partner])
    stream = torch.cuda.Stream(dev)
    peer_dir = "push" if direction == "push" else "pull"
    peer_peak = _peer_copy_peak(dist_, sw, partner, peer_dir,
                                is_src if peer_dir == "push" else not is_src, stream, 2048,
                                sh.num_segments, sh.page_bytes)
    cut = int(round(plan.num_blocks * split))

    def run():
        if direction == "split":
            if is_src:
                sw.migrate_blocks([pair], partner, plan.source_ids[:cut], plan.target_ids[:cut],
                                  None, direction="push", stream=stream, mode=mode)
            else:
                sw.migrate_blocks([pair], partner, plan.source_ids[cut:], plan.target_ids[cut:],
                                  None, direction="pull", stream=stream, mode=mode)
        elif active:
            sw.migrate_blocks([pair], partner, plan.source_ids, plan.target_ids, None,
                              direction=direction, stream=stream, mode=mode)

    for _ in range(warmup):
        run()
    stream.synchronize()
    dist_.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        run()
    b.record(stream)
    b.synchronize()
    t = dist_.max(a.elapsed_time(b) / 1e3)
    dist_.barrier()
    # Exact parity of the timed migrations, position-keyed across the pair.
    parity = _pair_exact(dist_, dev, pages, sh.page_bytes,
                         plan.source_ids if is_src else plan.target_ids, is_src, partner)
    if not extras:
        sw.close()
        del pages
        torch.cuda.empty_cache()
        per_pair = nbytes * steps / t / 1e9
        return {"per_pair_gbs": per_pair, "frac_of_nominal_900": per_pair / 900.0,
                "peer_copy_gbs": peer_peak["per_pair_gbs"],
                "frac_of_measured_peer_copy": per_pair / peer_peak["per_pair_gbs"],
                "bit_exact": parity}
    # Small calls: the plan's first n blocks (all 56 segments), as a decode
    # rank pulls a short request; µs per call, device time, max over ranks.
    small = {}
    for n in MIGRATION_SMALL_BLOCKS:
        sub_src, sub_dst = plan.source_ids[:n], plan.target_ids[:n]

        def one():
            if active:
                sw.migrate_blocks([pair], partner, sub_src, sub_dst, None,
                                  direction=direction, stream=stream)

        for _ in range(20):
            one()
        stream.synchronize()
        dist_.barrier()
        a.record(stream)
        for _ in range(200):
            one()
        b.record(stream)
        b.synchronize()
        small[str(n)] = dist_.max(a.elapsed_time(b) * 1e3 / 200)
        dist_.barrier()
    ipc_ok = None
    if ipc_check:
        ipc_ok = _ipc_event_ordering(dist_, dev, sw, pages, sh.page_bytes, plan, is_src,
                                     partner, pair, stream)
    nccl = nccl_comparison(dist_, dev, sw, plan, is_src, partner, steps, warmup)
    sw.close()
    del pages
    torch.cuda.empty_cache()
    total = half * nbytes * steps
    per_pair = nbytes * steps / t / 1e9
    out = {"config": "cfg3 Qwen2.5-7B P->D migration: 28 layers, 4 kv heads, 128 dim, bf16, "
                     "block 16; 8 requests/pair, prompts U{512..8192}; pairs (i, i+N/2); "
                     f"{direction}: " + ("decode rank loads from the prefill rank's mapped "
                                         "cache over NVLink" if direction == "pull" else
                                         "prefill rank stores into the decode rank's mapped "
                                         "cache over NVLink"),
           "pairs": half, "bytes_per_pair": nbytes, "value": total / t / 1e9, "unit": "GB/s",
           "per_pair_gbs": per_pair, "frac_of_nominal_900": per_pair / 900.0,
           "frac_of_pool_peer_copy_770": per_pair / POOL_PEER_COPY_GBS,
           "pool_peer_copy_source": "the pool's published measured peer copy, 770 GB/s per "
                                    "direction (not measured by this run)",
           "peer_copy_peak": peer_peak,
           "frac_of_measured_peer_copy": per_pair / peer_peak["per_pair_gbs"],
           "ms_per_step": t / steps * 1e3, "bit_exact": parity,
           "bit_exact_how": "every moved block, all 56 segments, compared byte for byte across "
                            "the pair in plan order (prefill gather sent over NCCL)",
           "small_calls_us": small,
           "small_calls_how": "per n: one migrate_blocks call moving n blocks x 56 segments "
                              f"({sh.composite_bytes // 1024} KiB per block), 200 calls "
                              "after 20 warm-up, CUDA events, max over ranks",
           "nccl_sendrecv": {"value": half * nbytes / nccl / 1e9, "unit": "GB/s",
                             "per_pair_gbs": nbytes / nccl / 1e9,
                             "how": "gather blocks into a contiguous buffer (kvx kernel), "
                                    "torch.distributed send/recv (NCCL), scatter on the "
                                    "decode rank; CUDA events, max over ranks"}}
    if ipc_check:
        out["ipc_event_ordering"] = ipc_ok
        out["ipc_event_ordering_how"] = (
            "prefill swaps new bytes into the source blocks and ships the swap's IPC event "
            "handle before it completes; decode pulls after waiting on it; exact check")
    return out


def nccl_comparison(dist_, dev, sw, plan, is_src, partner, steps, warmup) -> float:
    """Seconds per migration through NCCL send/recv of a gathered buffer."""
    import torch
    import torch.distributed as dist

    from aegaeon_b200 import _lib, swapper

    n = plan.num_blocks
    segs = sw.segments
    buf = torch.empty(n * sw.composite_page, dtype=torch.uint8, device=dev)
    # segment-major staging: segment s holds the n moved pages back to back
    staging_pages = [buf[i * n * s.page_size_bytes:(i + 1) * n * s.page_size_bytes]
                     for i, s in enumerate(segs)]
    st_segs, _ = swapper.make_segments([((f"st{i}",), n * s.page_size_bytes)
                                        for i, s in enumerate(segs)], n)
    staging = swapper.KVSwapper(dev.index, st_segs, staging_pages,
                                [frozenset({0})] * len(segs), [1])
    local, st_ep = sw.local_endpoint(), staging.local_endpoint()
    cur = torch.cuda.current_stream(dev)
    idx = list(range(n))

    def move(src_ep, dst_ep, src_ids, dst_ids):
        arr = swapper._entry_arrays(src_ids, dst_ids, [0] * n, [0] * n, [1] * n)
        _lib.check(_lib.lib().kvx_migrate_blocks(src_ep.handle, dst_ep.handle, *arr,
                                                 _lib.MODE_SM, cur.cuda_stream, None, None))

    def once():
        if is_src:
            move(local, st_ep, plan.source_ids, idx)
            dist.send(buf, dst=partner)
        else:
            dist.recv(buf, src=partner)
            move(st_ep, local, idx, plan.target_ids)

    for _ in range(warmup):
        once()
    dist_.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(cur)
    for _ in range(steps):
        once()
    b.record(cur)
    b.synchronize()
    t = dist_.max(a.elapsed_time(b) / 1e3)
    staging.close()
    return t / steps


def traffic_from_profile() -> float | None:
    """DRAM bytes (read + write) per launch of the gather kernel from the
    committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    try:
        with open(path) as f:
            return float(json.load(f)["traffic_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


# ---- arms --------------------------------------------------------------------------
def blocks_per_direction(requested: int, world: int, cache_blocks: int) -> int:
    """Blocks each way per step: `requested`, unless 2 x that many 8 MiB
    page-locked host rows per rank would not fit in 45% of the host's
    available memory (then fewer, a multiple of 16; stated in the config)."""
    from aegaeon_b200 import workloads

    per_dir = requested
    try:
        avail = int([l for l in open("/proc/meminfo")
                     if l.startswith("MemAvailable")][0].split()[1]) * 1024
        rows_fit = int(0.45 * avail / world / workloads.CFG2.composite_bytes)
        if 2 * per_dir > rows_fit:
            per_dir = max(64, rows_fit // 2 // 16 * 16)
    except (OSError, IndexError, ValueError):
        pass
    return min(per_dir, cache_blocks // 2)


def cfg2_config(per_dir: int, cache_blocks: int, world: int) -> dict:
    """The `config` object of both arms (identical, so the lines compare)."""
    from aegaeon_b200 import workloads

    return {
        "workload": "cfg2 Llama-2-7B-shaped per-GPU swap: 32 layers x separate K/V "
                    f"[{cache_blocks},16,32,128] fp16 U(-2,2) seed 0; per step {per_dir} "
                    f"random blocks out to host and {per_dir} other random blocks in from "
                    "host, out and in on two streams concurrently; every GPU independent",
        "blocks_per_direction": per_dir,
        "bytes_per_step_per_gpu": 2 * per_dir * workloads.CFG2.composite_bytes,
        "l2": "no flush needed: 8 GiB per direction per step, far larger than the 126 MB L2",
        "parallelism": f"independent swap per GPU x{world}",
    }


def run_kvx(args):
    import torch

    from aegaeon_b200 import _lib, workloads

    dist_ = Dist.init(use_pg=True)
    dev = torch.device("cuda", dist_.local_rank)
    per_dir = blocks_per_direction(args.blocks, dist_.world, args.cache_blocks)
    peaks = host_link_peaks(dev, dist_)  # all ranks at once: the box's concurrent peak
    box_peak = peaks["box_bidir_gbs"]
    # host DRAM copy bandwidth: a property of the box, measured by rank 0 alone
    dram = host_dram_copy_gbs() if dist_.rank == 0 else None
    dist_.barrier()
    bench = SwapBench(dev, per_dir, args.cache_blocks)
    bench.host_peaks = peaks
    lists = [bench.step_lists(k) for k in range(args.warmup + args.steps)]
    for k in range(args.warmup):
        bench.issue(lists[k], args.mode)
    torch.cuda.synchronize()
    mode_used = _lib.last_mode_name()
    clocks = ClockSampler(gpu_uuid(dev))
    dist_.barrier()
    clocks.start()
    l0 = _lib.lib().kvx_kernel_launches()
    _lib.kernel_timing_read()  # drop anything recorded before
    _lib.kernel_timing(True)
    t_dev = bench.timed_device(args.steps, args.mode, lambda k: lists[args.warmup + k])
    _lib.kernel_timing(False)
    launches = _lib.lib().kvx_kernel_launches() - l0
    clk = clocks.stop()
    k_launches, k_ms, k_busy_ms, k_bytes = _lib.kernel_timing_read()
    dist_.barrier()
    t_dev = dist_.max(t_dev)
    launches = int(dist_.sum(launches))
    # end-to-end through the public API from block tables
    bench.timed_e2e(1, args.mode)  # warm the planner path
    dist_.barrier()
    t_e2e = dist_.max(bench.timed_e2e(args.steps, args.mode))
    kr = bench.kernel_roofline(mode_bulk=True)
    kr_vec = bench.kernel_roofline(mode_bulk=False)
    one_dir = bench.live_one_direction(lists[args.warmup:args.warmup + 2], args.mode)
    bytes_total = bench.bytes_per_step * args.steps * dist_.world
    value = bytes_total / t_dev / 1e9
    e2e = bytes_total / t_e2e / 1e9
    extras = None
    if dist_.world == 1 and not args.no_extras:
        extras = baseline_configs(dev, bench)
    bench.close()
    del bench
    torch.cuda.empty_cache()
    mig = mig_push = None
    if dist_.world >= 2 and not args.no_migration:
        mig = migration_bench(dist_, dev, steps=args.steps, warmup=args.warmup,
                              direction="pull", ipc_check=True)
        mig_push = migration_bench(dist_, dev, steps=args.steps, warmup=args.warmup,
                                   direction="push")
    cpu = None
    if dist_.rank == 0 and dist_.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)
    mp = measured_peaks()
    hbm_peak = mp.get("hbm_gbs", 6650.0)
    per_gpu = value / dist_.world
    line = None
    if dist_.rank == 0:
        # algorithmic bytes per launch / mean launch duration
        achieved_k = k_bytes / (k_ms / 1e3) / 1e9 if k_ms > 0 else None
        traffic = traffic_from_profile()
        k_name = ("kvx_copy_bulk<GridList>" if mode_used == "ce" else "kvx_copy_vec<GridList>")
        facts = host_facts()
        host_link = {
            "bound": "host_link", "achieved_box_gbs": value, "box_peak_gbs": box_peak,
            "frac": value / box_peak, "per_gpu_gbs": per_gpu,
            "per_gpu_peak_h2d_gbs": peaks["h2d_gbs"], "per_gpu_peak_d2h_gbs": peaks["d2h_gbs"],
            "host_dram_copy_gbs": dram,
            "host": {k: facts.get(k) for k in ("cpus", "numa_nodes", "mem_total_gib", "memlock")},
            "limiter": ("PCIe link of the one GPU" if dist_.world == 1 else
                        "host memory shared by all GPUs' copy engines: every payload byte is "
                        "written to (swap-out) or read from (swap-in) host DRAM"),
        }
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "GB/s",
            "n_gpus": dist_.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": t_dev / args.steps * 1e3,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u8",
            "data": "synthetic: fp16 U(-2,2) from seed 0, block ids from seeded randperm "
                    "(no real checkpoint or trace)",
            "config": cfg2_config(per_dir, args.cache_blocks, dist_.world),
            "api": "KVSwapper.swap_blocks (Worker.swap_blocks replacement) -> kvx_swap_blocks; "
                   f"transfer mode {args.mode} -> {mode_used}",
            "roofline": {
                "bound": "hbm",
                "kernel": k_name,
                "achieved": achieved_k,
                "peak": hbm_peak,
                "unit": "GB/s",
                "frac": (achieved_k / hbm_peak) if achieved_k else None,
                "traffic": traffic,
                "host_link": host_link,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (burst copy, read+write), of measured"
                               if "hbm_gbs" in mp else "fallback 6650 GB/s, of fallback",
                "how": "live: CUDA events around every launch of the copy kernel on its stream "
                       "inside the timed region; achieved = algorithmic bytes per launch (read "
                       "+ write of one staging chunk gather/scatter) / mean launch duration. "
                       "Each launch runs beside the other direction's copy-engine DMA",
                "launches": k_launches,
                "algorithmic_bytes_per_launch": (k_bytes // k_launches) if k_launches else None,
                "mean_launch_ms": (k_ms / k_launches) if k_launches else None,
                "busy_ms": k_busy_ms,
                "one_direction_live": {
                    "how": "2 swap-out steps with nothing on the swap-in stream, same events "
                           "and byte count: the launches without the other direction beside "
                           "them",
                    "launches": one_dir[0],
                    "mean_launch_ms": (one_dir[1] / one_dir[0]) if one_dir[0] else None,
                    "achieved": (one_dir[3] / (one_dir[1] / 1e3) / 1e9) if one_dir[1] else None,
                    "frac": (one_dir[3] / (one_dir[1] / 1e3) / 1e9 / hbm_peak)
                    if one_dir[1] else None,
                },
                "isolated_bulk_gbs": kr["algorithmic_bytes"] / kr["seconds"] / 1e9,
                "isolated_vec_gbs": kr_vec["algorithmic_bytes"] / kr_vec["seconds"] / 1e9,
                "ncu": "profiles/kvx_copy_bulk_grid_cfg2_small.md",
            },
            "host_link_roofline": {
                "bound": "host_link",
                "achieved": per_gpu,
                "peak": box_peak / dist_.world,
                "unit": "GB/s",
                "frac": value / box_peak,
                "peak_source": "measured live: every GPU of the run copies 2 GiB of "
                               "page-locked memory each way (256 MiB pieces) in the same "
                               "barrier-started windows, best of 10; box = all bytes / "
                               "slowest rank; "
                               "per-GPU share shown (the step is bidirectional)",
                "box_peak_gbs": box_peak,
                "peak_h2d_gbs": peaks["h2d_gbs"],
                "peak_d2h_gbs": peaks["d2h_gbs"],
                "nominal_gbs_per_direction": 63.0,
                "host": facts,
            },
            "e2e": {
                "value": e2e,
                "unit": "GB/s",
                "h2d_bytes_per_step": per_dir * workloads.CFG2.composite_bytes * dist_.world,
                "d2h_bytes_per_step": per_dir * workloads.CFG2.composite_bytes * dist_.world,
                "api": "block tables -> plan_move_requests (move_requests list building) -> "
                       "KVSwapper.swap_blocks -> stream sync",
                "seconds": t_e2e,
            },
            "gpu_launches": launches,
        }
        if mig is not None:
            line["migration"] = mig
            line["migration_push"] = mig_push
        if cpu is not None:
            line["cpu_baseline"] = cpu
        line["clocks"] = clk
        # Compact summaries last: they stay in the tail of the line.
        line["host_link"] = {k: (round(v, 3) if isinstance(v, float) else v)
                             for k, v in host_link.items() if k not in ("host", "limiter")}
        if mig is not None:
            line["migration_summary"] = {
                d: {"per_pair_gbs": round(m["per_pair_gbs"], 1),
                    "frac_of_900": round(m["frac_of_nominal_900"], 3),
                    "frac_of_pool_770": round(m["frac_of_pool_peer_copy_770"], 3),
                    "ce_peer_copy_gbs": round(m["peer_copy_peak"]["per_pair_gbs"], 1),
                    "bit_exact": m["bit_exact"], "ipc_event_ordering": m.get("ipc_event_ordering")}
                for d, m in (("pull", mig), ("push", mig_push))}
        if extras is not None:
            line["baseline_configs"] = extras
    dist_.finish()
    if line is not None:
        emit(line)


def run_reference(args):
    """The reference's own swap op (ops/swap.cu, built unmodified from the
    reference sources into oracle/_ref) on configuration 2: one call per K/V
    tensor, one cudaMemcpyAsync per block, out and in on two streams, issued
    from one host thread per GPU.  At N > 1 every rank swaps its own cache, as
    one reference Worker per GPU does (aegaeon/llm.py:992-1017); the box
    aggregate uses the slowest rank's time."""
    import torch

    from aegaeon_b200 import workloads

    try:
        from oracle import build_ref

        ref = build_ref.load_module()
    except Exception as e:  # noqa: BLE001
        if int(os.environ.get("RANK", "0")) == 0:
            emit({"impl": "reference", "unavailable": f"reference op not built: {e}"})
        return
    dist_ = Dist.init(use_pg=True)
    dev = torch.device("cuda", dist_.local_rank)
    sh = workloads.CFG2
    per_dir = blocks_per_direction(args.blocks, dist_.world, args.cache_blocks)
    nb = args.cache_blocks
    gen = torch.Generator(device=dev).manual_seed(0)
    caches = []
    for _ in range(sh.num_segments):
        t = torch.empty((nb, 16, sh.kv_heads, sh.head_dim), dtype=sh.dtype, device=dev)
        t.uniform_(-2.0, 2.0, generator=gen)
        caches.append(t)
    out_host = [torch.empty((per_dir, 16, sh.kv_heads, sh.head_dim), dtype=sh.dtype,
                            pin_memory=True) for _ in range(sh.num_segments)]
    in_host = [torch.empty_like(h, pin_memory=True) for h in out_host]
    s_out, s_in = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    slots = list(range(per_dir))
    live = args.ref_variant == "live-loop"
    if live:
        # composite host rows: row r holds every segment's page of one block
        page = sh.page_bytes
        pool_out = torch.empty((per_dir, sh.num_segments * page), dtype=torch.uint8,
                               pin_memory=True)
        pool_in = torch.empty((per_dir, sh.num_segments * page), dtype=torch.uint8,
                              pin_memory=True)
        gpu_pages = [c.view(torch.uint8).view(nb, page) for c in caches]

    def live_loop(pool, ids, is_swap_in):
        # worker.py:2272-2329 restated: per segment, per entry, one copy_
        for s, pages in enumerate(gpu_pages):
            off = s * page
            for row, blk in enumerate(ids):
                cpu_page = pool[row].narrow(0, off, page)
                if is_swap_in:
                    pages[blk].narrow(0, 0, page).copy_(cpu_page, non_blocking=True)
                else:
                    cpu_page.copy_(pages[blk].narrow(0, 0, page), non_blocking=True)

    def step(k):
        out_ids, in_ids = workloads.swap_step_ids(nb, per_dir, k)
        with torch.cuda.stream(s_out):
            if live:
                live_loop(pool_out, out_ids, False)
            else:
                for c, h in zip(caches, out_host):
                    ref.swap(out_ids, slots, False, c, h)
        with torch.cuda.stream(s_in):
            if live:
                live_loop(pool_in, in_ids, True)
            else:
                for c, h in zip(caches, in_host):
                    ref.swap(slots, in_ids, True, c, h)
        ev_o, ev_i = torch.cuda.Event(), torch.cuda.Event()
        ev_o.record(s_out)
        ev_i.record(s_in)
        s_out.wait_event(ev_i)
        s_in.wait_event(ev_o)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    clocks = ClockSampler(gpu_uuid(dev))
    dist_.barrier()
    clocks.start()
    cur = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record(cur)
    s_out.wait_event(a)
    s_in.wait_event(a)
    for k in range(args.steps):
        step(args.warmup + k)
    cur.wait_stream(s_out)
    cur.wait_stream(s_in)
    b.record(cur)
    b.synchronize()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    t = dist_.max(a.elapsed_time(b) / 1e3)
    wall = dist_.max(wall)
    # the last step's swap-out must hold its blocks (checked on every rank)
    last_out, _ = workloads.swap_step_ids(nb, per_dir, args.warmup + args.steps - 1)
    oi = torch.tensor(last_out, device=dev)
    exact = all(torch.equal(h.to(dev).view(torch.uint8), c[oi].view(torch.uint8))
                for c, h in zip(caches[:4], out_host[:4])) if not live else None
    exact_all = dist_.gather_obj(exact)
    dist_.finish()
    if dist_.rank != 0:
        return
    per_step = per_dir * sh.composite_bytes * dist_.world
    nbytes = 2 * per_step * args.steps
    value = nbytes / t / 1e9
    emit({
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": dist_.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic: fp16 U(-2,2) from seed 0, block ids from seeded randperm "
                "(no real checkpoint or trace)",
        "config": cfg2_config(per_dir, nb, dist_.world),
        "api": ("restated Worker.swap_blocks hot loop (worker.py:2270-2329): one torch "
                "copy_(non_blocking=True) per segment and block into composite host rows"
                if live else
                "reference aegaeon.ops.swap (ops/swap.cu, built unmodified from the reference "
                "sources): one call per K/V tensor, one cudaMemcpyAsync per block"),
        "bit_exact_last_swap_out": exact_all if not live else None,
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": dist_.world,
                         "kind": "reference",
                         "sample": f"full workload, {args.steps} steps; one host thread per GPU "
                                   f"issues {2 * per_dir * sh.num_segments} copies per step"},
        "e2e": {"value": nbytes / wall / 1e9, "unit": "GB/s", "h2d_bytes_per_step": per_step,
                "d2h_bytes_per_step": per_step,
                "how": "the op takes host buffers: every payload byte crosses the host link "
                       "inside the timed region; wall clock, slowest rank"},
        "gpu_launches": 0,
        "clocks": clk,
    })


# ---- configurations 1, 4 and 5 (one JSON line each, N=1 unless stated) ---------
def _ref_module():
    from oracle import build_ref

    return build_ref.load_module()


def _timed(stream_list, fn, steps, dev):
    """Device time of `steps` calls of fn (which issues on the given streams)."""
    import torch

    cur = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(cur)
    for st in stream_list:
        st.wait_event(a)
    for k in range(steps):
        fn(k)
    for st in stream_list:
        cur.wait_stream(st)
    b.record(cur)
    b.synchronize()
    return a.elapsed_time(b) / 1e3


def _bytes_equal_chunked(dev, host_u8, device_u8_fn, rows: int, row_bytes: int,
                         chunk_rows: int) -> bool:
    """host_u8 (page-locked, rows x row_bytes) equals device_u8_fn(r0, r1)
    (a (r1-r0) x row_bytes uint8 device tensor) for every chunk of rows;
    compared on the device."""
    import torch

    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        h = host_u8[r0 * row_bytes:r1 * row_bytes].to(dev, non_blocking=False)
        if not torch.equal(h.view(r1 - r0, row_bytes), device_u8_fn(r0, r1)):
            return False
    return True


class Cfg1:
    """Configuration 1 (Qwen3-4B round trip) through the per-tensor op: 72
    tensors [1024,16,8,128] bf16 N(0,1) from seed 0; 256 blocks out to slots
    0..255, then back in to a fresh permutation of a zeroed cache.  Either
    arm: this build's ops.swap or the reference's compiled op."""

    N = 256

    def __init__(self, dev):
        import torch

        from aegaeon_b200 import workloads

        self.dev = dev
        self.sh = sh = workloads.CFG1
        gen = torch.Generator(device=dev).manual_seed(0)
        self.shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
        self.caches = [torch.empty(self.shape, dtype=sh.dtype, device=dev).normal_(generator=gen)
                       for _ in range(sh.num_segments)]
        self.back = [torch.zeros_like(c) for c in self.caches]
        self.hosts = [torch.empty((self.N,) + self.shape[1:], dtype=sh.dtype, pin_memory=True)
                      for _ in self.caches]
        self.out_ids = workloads.randperm(sh.num_blocks, 0)[:self.N]
        self.in_ids = workloads.randperm(sh.num_blocks, 1)[:self.N]
        self.slots = list(range(self.N))
        self.step_bytes = 2 * sh.num_segments * self.N * sh.page_bytes

    def run(self, impl: str, steps: int, warmup: int, mode: str = "auto", ref=None) -> dict:
        import torch

        from aegaeon_b200 import ops

        for b in self.back:
            b.zero_()
        for h in self.hosts:
            h.zero_()

        def swap(src, dst, is_in, cache, host):
            if impl == "reference":
                ref.swap(src, dst, is_in, cache, host)
            else:
                ops.swap(src, dst, is_in, cache, host, mode=mode)

        def step_out(_k):
            for c, h in zip(self.caches, self.hosts):
                swap(self.out_ids, self.slots, False, c, h)

        def step_in(_k):
            for c, h in zip(self.back, self.hosts):
                swap(self.slots, self.in_ids, True, c, h)

        def step(k):
            step_out(k)
            step_in(k)

        for k in range(warmup):
            step(k)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        t = _timed([], step, steps, self.dev)
        wall = time.perf_counter() - t0
        # device time per call of each direction on its own (repeating a
        # direction rewrites the same bytes, so the checks below still hold)
        per_call = {}
        if steps:
            for name, fn in (("out", step_out), ("in", step_in)):
                per_call[f"{name}_us_per_call"] = (_timed([], fn, steps, self.dev) * 1e6
                                                   / steps / len(self.caches))
        oi = torch.tensor(self.out_ids, device=self.dev)
        ii = torch.tensor(self.in_ids, device=self.dev)
        exact = all(torch.equal(b[ii].view(torch.uint8), c[oi].view(torch.uint8)) and
                    torch.equal(h.to(self.dev).view(torch.uint8), c[oi].view(torch.uint8))
                    for b, c, h in zip(self.back, self.caches, self.hosts))
        return {"seconds": t, "wall": wall, "gbs": self.step_bytes * steps / t / 1e9,
                "e2e_gbs": self.step_bytes * steps / wall / 1e9, "bit_exact": bool(exact),
                **per_call}

    def close(self):
        del self.caches, self.back, self.hosts


class Cfg4:
    """Configuration 4 (model-switch overlap): swap-in of 2048 cfg2 blocks
    (16 GiB) while a Qwen1.5-14B TP-2 weight shard (14.17 GB bf16, four
    safetensors-sized storages) is uploaded from page-locked host memory on a
    second stream.  The cfg2 cache (64 segments) and its 2048-row host pool
    are reused from the headline run when given.

    kvx arm: switch_in (KV swap-in through kvx_swap_blocks, weights through
    kvx_upload_weights in 64 MiB chunks).  Reference arm: the reference op per
    K/V tensor for the KV (host slots carved from the same pool, one
    contiguous region per tensor) and one copy_(non_blocking=True) per weight
    storage (quick_loader.py:340)."""

    N = 2048
    FILES = 4

    def __init__(self, dev, pages=None, pool=None, segments=None):
        import torch

        from aegaeon_b200 import swapper, workloads

        self.dev = dev
        self.sh = sh = workloads.CFG2
        if pages is None:
            gen = torch.Generator(device=dev).manual_seed(0)
            pages = []
            for _ in range(sh.num_segments):
                t = torch.empty(sh.num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
                workloads.fill_segment(t, sh, gen)
                pages.append(t)
            segments, _ = swapper.make_segments(
                [((f"l{i}",), sh.num_blocks * sh.page_bytes) for i in range(sh.num_segments)],
                sh.num_blocks)
            pool = torch.empty(self.N * sh.composite_bytes, dtype=torch.uint8, pin_memory=True)
            fill = torch.empty(GIB, dtype=torch.uint8, device=dev).random_(0, 256, generator=gen)
            for o in range(0, pool.numel(), fill.numel()):
                pool[o:o + fill.numel()].copy_(fill[:pool.numel() - o])
            del fill
        self.pages, self.pool, self.segments = pages, pool, segments
        self.ws = workloads.WeightShard()
        gen = torch.Generator(device=dev).manual_seed(4)
        self.w_dev = torch.empty(self.ws.nbytes, dtype=torch.uint8, device=dev)
        self.w_host = torch.empty(self.ws.nbytes, dtype=torch.uint8, pin_memory=True)
        fill = torch.empty(GIB, dtype=torch.uint8, device=dev).random_(0, 256, generator=gen)
        for o in range(0, self.ws.nbytes, fill.numel()):
            self.w_host[o:o + fill.numel()].copy_(fill[:self.ws.nbytes - o])
        del fill
        self.in_ids = workloads.randperm(sh.num_blocks, 7)[:self.N]
        self.kv_bytes = self.N * sh.composite_bytes
        self.s_kv, self.s_w = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        # storages of the reference arm: the shard cut into FILES pieces
        cut = -(-self.ws.nbytes // self.FILES)
        self.files = [(o, min(self.ws.nbytes, o + cut)) for o in range(0, self.ws.nbytes, cut)]

    def _check(self, impl) -> bool:
        import torch

        sh, page = self.sh, self.sh.page_bytes
        ii = torch.tensor(self.in_ids, device=self.dev)
        if impl == "reference":
            # tensor s's host slots are the contiguous region s of the pool
            for s, p in enumerate(self.pages):
                region = self.pool[s * self.N * page:(s + 1) * self.N * page]
                cache = p.view(-1, page)
                if not _bytes_equal_chunked(self.dev, region, lambda r0, r1: cache[ii[r0:r1]],
                                            self.N, page, 1024):
                    return False
        else:
            comp = sh.composite_bytes

            def gathered(r0, r1):
                return torch.cat([p.view(-1, page)[ii[r0:r1]] for p in self.pages], dim=1)

            if not _bytes_equal_chunked(self.dev, self.pool, gathered, self.N, comp, 128):
                return False
        return _bytes_equal_chunked(self.dev, self.w_host, lambda r0, r1: self.w_dev[
            r0 * GIB:r1 * GIB].view(r1 - r0, GIB), self.ws.nbytes // GIB, GIB, 1) and \
            torch.equal(self.w_dev[self.ws.nbytes // GIB * GIB:],
                        self.w_host[self.ws.nbytes // GIB * GIB:].to(self.dev))

    def run(self, impl: str, steps: int, warmup: int, mode: str = "auto", ref=None,
            sw=None) -> dict:
        import torch

        from aegaeon_b200 import swapper, switch

        sh, n = self.sh, self.N
        self.w_dev.zero_()
        if impl == "reference":
            page = sh.page_bytes
            shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
            caches = [p.view(sh.dtype).view(shape) for p in self.pages]
            hosts = [self.pool[s * n * page:(s + 1) * n * page].view(sh.dtype).view(
                (n,) + shape[1:]) for s in range(sh.num_segments)]
            slots = list(range(n))

            def step(_k):
                with torch.cuda.stream(self.s_kv):
                    for c, h in zip(caches, hosts):
                        ref.swap(slots, self.in_ids, True, c, h)
                with torch.cuda.stream(self.s_w):
                    for a, b in self.files:
                        self.w_dev[a:b].copy_(self.w_host[a:b], non_blocking=True)
        else:
            own = sw is None
            if own:
                sw = swapper.KVSwapper(self.dev.index, self.segments, self.pages,
                                       [frozenset({0})] * sh.num_segments, [1], kv_swap=self.pool)
            rows = list(range(n))
            z, one = [0] * n, [1] * n

            def step(_k):
                switch.switch_in(sw, [(self.w_dev, self.w_host)], [0], rows, self.in_ids, z, z,
                                 one, [None], chunk_bytes=64 << 20, kv_stream=self.s_kv,
                                 weight_stream=self.s_w, mode=mode)

        for k in range(warmup):
            step(k)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        t = _timed([self.s_kv, self.s_w], step, steps, self.dev)
        wall = time.perf_counter() - t0
        exact = self._check(impl)
        if impl != "reference" and own:
            sw.close()
        per = t / steps
        return {"seconds": t, "wall": wall, "switch_ms": per * 1e3,
                "gbs": (self.kv_bytes + self.ws.nbytes) / per / 1e9,
                "e2e_gbs": (self.kv_bytes + self.ws.nbytes) * steps / wall / 1e9,
                "bit_exact": bool(exact)}

    def close(self):
        del self.w_dev, self.w_host, self.pages, self.pool


class Cfg5:
    """Configuration 5 (fragmented swap-out): Qwen1.5-MoE-A2.7B pages (16 kv
    heads x 128 dim bf16, 64 KiB per K or V page), a 16,384-entry mapping with
    half the entries in contiguous device runs of 1..32 blocks and half
    isolated; host slots sequential; one call per step.  `layers` may be
    below 24 to bound the host memory and time of a run (stated in the
    output)."""

    def __init__(self, dev, layers: int = 24, entries: int = 16384, seed: int = 0):
        import dataclasses

        import torch

        from aegaeon_b200 import swapper, workloads

        self.dev = dev
        self.sh = sh = dataclasses.replace(workloads.CFG5, layers=layers)
        self.n = entries
        self.ids, self.slots = workloads.fragmented_mapping(entries, sh.num_blocks, seed=seed)
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.pages = []
        for _ in range(sh.num_segments):
            t = torch.empty(sh.num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
            workloads.fill_segment(t, sh, gen)
            self.pages.append(t)
        self.segments, self.comp = swapper.make_segments(
            [((f"l{i}",), sh.num_blocks * sh.page_bytes) for i in range(sh.num_segments)],
            sh.num_blocks)
        self.pool = torch.empty(entries * self.comp, dtype=torch.uint8, pin_memory=True)
        self.s = torch.cuda.Stream(dev)
        self.call_bytes = entries * self.comp

    def _check(self, impl) -> bool:
        import torch

        page, n = self.sh.page_bytes, self.n
        idx = torch.tensor(self.ids, device=self.dev)
        if impl == "reference":
            for s, p in enumerate(self.pages):
                region = self.pool[s * n * page:(s + 1) * n * page]
                cache = p.view(-1, page)
                if not _bytes_equal_chunked(self.dev, region, lambda r0, r1: cache[idx[r0:r1]],
                                            n, page, 4096):
                    return False
            return True

        def gathered(r0, r1):
            return torch.cat([p.view(-1, page)[idx[r0:r1]] for p in self.pages], dim=1)

        return _bytes_equal_chunked(self.dev, self.pool, gathered, n, self.comp,
                                    max(1, GIB // self.comp))

    def run(self, impl: str, steps: int, warmup: int, mode: str = "auto", ref=None) -> dict:
        import torch

        from aegaeon_b200 import swapper

        sh, n = self.sh, self.n
        self.pool.zero_()
        if impl == "reference":
            page = sh.page_bytes
            shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
            caches = [p.view(sh.dtype).view(shape) for p in self.pages]
            hosts = [self.pool[s * n * page:(s + 1) * n * page].view(sh.dtype).view(
                (n,) + shape[1:]) for s in range(sh.num_segments)]

            def step(_k):
                with torch.cuda.stream(self.s):
                    for c, h in zip(caches, hosts):
                        ref.swap(self.ids, self.slots, False, c, h)
        else:
            sw = swapper.KVSwapper(self.dev.index, self.segments, self.pages,
                                   [frozenset({0})] * sh.num_segments, [1], kv_swap=self.pool)
            z, one = [0] * n, [1] * n

            def step(_k):
                sw.swap_blocks([0], self.ids, self.slots, z, z, one, [None], False, mode=mode,
                               stream=self.s)

        for k in range(warmup):
            step(k)
        torch.cuda.synchronize()
        if steps == 0:
            if impl != "reference":
                sw.close()
            return {}
        lat = []
        t0 = time.perf_counter()
        for k in range(steps):
            lat.append(_timed([self.s], step, 1, self.dev))
        wall = time.perf_counter() - t0
        exact = self._check(impl)
        if impl != "reference":
            sw.close()
        t = sum(lat)
        return {"seconds": t, "wall": wall, "gbs": self.call_bytes * steps / t / 1e9,
                "e2e_gbs": self.call_bytes * steps / wall / 1e9,
                "call_ms": sorted(x * 1e3 for x in lat), "bit_exact": bool(exact)}

    def close(self):
        del self.pages, self.pool


def _ref_or_none():
    try:
        return _ref_module()
    except Exception:  # noqa: BLE001 - reported as a missing arm
        return None


def baseline_configs(dev, bench, cfg5_layers: int = 4) -> dict:
    """Configurations 1, 4 and 5 of BASELINE.json, both arms in this
    process, for the default N=1 line: a few timed steps each, every arm's
    output checked byte for byte afterwards."""
    import torch

    from aegaeon_b200 import workloads

    ref = _ref_or_none()
    out = {}

    def pair(name, obj, steps, warmup, extra=None, **kw):
        k = obj.run("kvx", steps, warmup, **kw)
        r = obj.run("reference", steps, warmup, ref=ref) if ref is not None else None
        rec = {"kvx_gbs": round(k["gbs"], 2),
               "reference_gbs": round(r["gbs"], 2) if r else None,
               "ratio": round(k["gbs"] / r["gbs"], 2) if r else None,
               "bit_exact": k["bit_exact"] and (r["bit_exact"] if r else True),
               "steps": steps}
        if extra:
            rec.update(extra(k, r))
        out[name] = rec

    c1 = Cfg1(dev)
    pair("cfg1", c1, 5, 2)
    c1.close()
    del c1
    torch.cuda.empty_cache()
    reuse = bench.rows >= Cfg4.N and bench.shape.num_blocks == workloads.CFG2.num_blocks
    c4 = Cfg4(dev, bench.pages, bench.pool, bench.segments) if reuse else Cfg4(dev)
    pair("cfg4", c4, 3, 1, extra=lambda k, r: {
        "kvx_switch_ms": round(k["switch_ms"], 1),
        "reference_switch_ms": round(r["switch_ms"], 1) if r else None},
        sw=bench.sw if reuse else None)
    c4.close()
    del c4
    torch.cuda.empty_cache()
    # scattered host slots, both directions at once (AUTO picks the mode):
    # the headline 8 MiB rows (the cfg2 cache and pool of the headline run) and
    # 896 KiB rows (the Qwen2.5-7B shape)
    bidir = bench.host_peaks["bidir_gbs"]
    frag = FragSwap(dev, bench.shape, bench.per_dir, bench.rows, bench.pages, bench.pool,
                    bench.segments, bench.sw)
    r = frag.run(3, 1, "auto", "auto", group=1)
    out["frag_8mib_rows"] = {"gbs": round(r["gbs"], 2), "frac_of_bidir_peak": round(r["gbs"] / bidir, 3),
                             "modes": r["modes_used"], "bit_exact": r["bit_exact"]}
    frag = FragSwap(dev, workloads.CFG3, 1024, 4096)
    # a new page-locked pool: warm up like --config 9 before timing
    r = frag.run(6, 3, "auto", "auto", group=1)
    out["frag_896kib_rows"] = {"gbs": round(r["gbs"], 2),
                               "frac_of_bidir_peak": round(r["gbs"] / bidir, 3),
                               "modes": r["modes_used"], "bit_exact": r["bit_exact"]}
    frag.close()
    del frag
    torch.cuda.empty_cache()
    c5 = Cfg5(dev, layers=cfg5_layers)
    pair("cfg5", c5, 3, 1, extra=lambda k, r: {
        "layers": cfg5_layers, "kvx_call_ms": round(statistics.median(k["call_ms"]), 1),
        "reference_call_ms": round(statistics.median(r["call_ms"]), 1) if r else None})
    c5.close()
    del c5
    torch.cuda.empty_cache()
    out["how"] = ("both arms here, same inputs; cfg1 72 tensors x 256 blocks out+in; cfg4 "
                  "2048-block swap-in + 14.17 GB weights; cfg5 16384 fragmented entries, "
                  f"{cfg5_layers} of 24 layers; frag_*: 1024 blocks out and 1024 in at once "
                  "over shuffled host rows, AUTO mode; outputs compared byte for byte")
    return out


def _line_for(args, r: dict, workload: str, impl: str, extra: dict = None) -> dict:
    line = {"impl": impl, "metric": METRIC, "value": r["gbs"], "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["seconds"] / args.steps * 1e3, "higher_is_better": True,
            "dtype": "u8", "data": "synthetic, seeded", "config": {"workload": workload},
            "bit_exact": r["bit_exact"],
            "e2e": {"value": r["e2e_gbs"], "unit": "GB/s"}}
    line.update(extra or {})
    return line


def run_config1(args):
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = Cfg1(dev)
    r = c.run(args.impl, args.steps, args.warmup, args.mode,
              ref=_ref_module() if args.impl == "reference" else None)
    line = _line_for(args, r, "cfg1 Qwen3-4B round trip: 36 layers x separate K/V "
                     "[1024,16,8,128] bf16 N(0,1) seed 0; 256 blocks out to slots 0..255 then "
                     "in to a fresh permutation, 72 swap calls per direction", args.impl,
                     {k: r[k] for k in ("out_us_per_call", "in_us_per_call") if k in r})
    line["e2e"].update({"h2d_bytes_per_step": c.step_bytes // 2,
                        "d2h_bytes_per_step": c.step_bytes // 2})
    return line


def run_config4(args):
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = Cfg4(dev)
    r = c.run(args.impl, args.steps, args.warmup, args.mode,
              ref=_ref_module() if args.impl == "reference" else None)
    peaks = host_link_peaks(dev)
    line = _line_for(args, r, "cfg4 switch overlap: swap-in of 2048 Llama-2-7B-shaped blocks "
                     f"({c.kv_bytes} B) concurrent with a Qwen1.5-14B TP-2 bf16 weight shard "
                     f"({c.ws.nbytes} B) uploaded on a second stream", args.impl,
                     {"switch_ms": r["switch_ms"],
                      "roofline": {"bound": "host_link", "achieved": r["gbs"],
                                   "peak": peaks["h2d_gbs"], "unit": "GB/s",
                                   "frac": r["gbs"] / peaks["h2d_gbs"],
                                   "peak_source": "measured live: 2 GiB page-locked H2D copy "
                                                  "in 256 MiB pieces"}})
    line["e2e"].update({"h2d_bytes_per_step": c.kv_bytes + c.ws.nbytes, "d2h_bytes_per_step": 0})
    return line


def run_config5(args):
    """Configuration 5 standalone: every rank (torchrun; one GPU alone
    without it) swaps out its own 16,384-entry fragmented mapping at the same
    time, either arm.  All 24 layers unless the host cannot page-lock 48 GiB
    per rank (then fewer, stated).  Box aggregate GB/s over the slowest rank;
    per-call latency of rank 0; every rank's output checked byte for byte."""
    import torch

    from aegaeon_b200 import workloads

    dist_ = Dist.init(use_pg=True)
    dev = torch.device("cuda", dist_.local_rank)
    layers = 24
    try:
        avail = int([l for l in open("/proc/meminfo")
                     if l.startswith("MemAvailable")][0].split()[1]) * 1024
        per_layer = 2 * 16384 * workloads.CFG5.page_bytes
        layers = max(1, min(24, int(0.4 * avail / dist_.world // per_layer)))
    except (OSError, IndexError, ValueError):
        pass
    layers = int(dist_.max(float(-layers)) * -1)  # the smallest over ranks
    c = Cfg5(dev, layers=layers, seed=dist_.rank)
    ref = _ref_module() if args.impl == "reference" else None
    # warm-up outside the window, then barrier-started timed calls
    c.run(args.impl, 0, args.warmup, args.mode, ref=ref)
    dist_.barrier()
    r = c.run(args.impl, args.steps, 0, args.mode, ref=ref)
    t = dist_.max(r["seconds"])
    wall = dist_.max(r["wall"])
    exact = dist_.gather_obj(r["bit_exact"])
    c.close()
    dist_.finish()
    if dist_.rank != 0:
        return None
    total = c.call_bytes * args.steps * dist_.world
    line = _line_for(args, {"gbs": total / t / 1e9, "seconds": t, "e2e_gbs": total / wall / 1e9,
                            "bit_exact": all(exact)},
                     f"cfg5 Qwen1.5-MoE-A2.7B fragmented swap-out: {layers} of 24 layers x K/V "
                     "64 KiB pages, 16384 entries per GPU (half in contiguous device runs of "
                     "1..32 blocks, half isolated), host slots sequential; one call per step, "
                     "every GPU at once", args.impl,
                     {"n_gpus": dist_.world, "scaling": "weak",
                      "call_latency_ms_rank0": r["call_ms"]})
    line["e2e"].update({"h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": c.call_bytes * dist_.world})
    return line


def run_config3_reference(args):
    """The reference's prefill->decode route (prefill_scheduler.py:84-99,
    decode_scheduler.py:336-347): the prefill GPU swaps the request's blocks
    out to page-locked host memory with the reference op, then the decode GPU
    swaps them in.  One process drives cuda:0 (prefill) and cuda:1 (decode);
    the time is the sum of the two hops (the decode side starts after the
    prefill side finished)."""
    import torch

    from aegaeon_b200 import workloads

    if torch.cuda.device_count() < 2:
        return {"impl": "reference", "unavailable": "config 3 needs two visible GPUs"}
    ref = _ref_module()
    sh = workloads.CFG3
    plan = workloads.migration_plan(sh, requests=8, seed=0, pair=0)
    n = plan.num_blocks
    shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    g = torch.Generator(device=d0).manual_seed(100)
    src = [torch.empty(shape, dtype=sh.dtype, device=d0).normal_(generator=g)
           for _ in range(sh.num_segments)]
    dst = [torch.zeros(shape, dtype=sh.dtype, device=d1) for _ in range(sh.num_segments)]
    host = [torch.empty((n,) + shape[1:], dtype=sh.dtype).pin_memory() for _ in src]
    slots = list(range(n))

    def hop(dev, fn):
        with torch.cuda.device(dev):
            s = torch.cuda.current_stream(dev)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            fn()
            b.record(s)
            b.synchronize()
            return a.elapsed_time(b) / 1e3

    def out_hop():
        for c, h in zip(src, host):
            ref.swap(plan.source_ids, slots, False, c, h)

    def in_hop():
        for c, h in zip(dst, host):
            ref.swap(slots, plan.target_ids, True, c, h)

    for _ in range(args.warmup):
        hop(d0, out_hop)
        hop(d1, in_hop)
    t = 0.0
    for _ in range(args.steps):
        t += hop(d0, out_hop) + hop(d1, in_hop)
    exact = all(torch.equal(b[plan.target_ids].cpu().view(torch.uint8),
                            a[plan.source_ids].cpu().view(torch.uint8)) for a, b in zip(src, dst))
    nbytes = n * sh.composite_bytes
    value = nbytes * args.steps / t / 1e9
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 2,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3,
            "higher_is_better": True, "dtype": "u8", "bit_exact": exact,
            "config": {"workload": "cfg3 P->D handoff of 8 requests (prompts U{512..8192}, "
                                   f"{n} blocks, {nbytes} B) on the reference route: "
                                   "swap-out on the prefill GPU to host, swap-in on the decode "
                                   "GPU, reference op (one cudaMemcpyAsync per block and tensor)"},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def run_config6(args):
    """The reference's own swap micro-benchmark workload
    (benchmark/benchmark_composite_swap.py:117-187): 8 segments of one
    17,301,504-byte physical page, 528-token physical blocks of 16-token
    kernel blocks, 3 fixed (full) pages plus the attention pages of a sequence
    of each length in [1, 128, 256, 512, 528, 529, 1057]; "full" copies every
    page whole, "optimized" only the live prefix of the last attention page.
    p50 / p95 of the swap time over `--steps` samples (CUDA events), H2D and
    D2H, for this build (kvx_swap_blocks, one call) or, with --impl
    reference, the harness's own copy loop restated (one torch copy_ per
    segment and page, benchmark_composite_swap.py:67-87)."""
    import math

    import torch

    from aegaeon_b200 import cache_transfer as ct
    from aegaeon_b200 import swapper

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    segments_n, fixed, phys_bytes, pbs, kbs = 8, 3, 17_301_504, 528, 16
    seg_page = phys_bytes // segments_n
    ratio = pbs // kbs
    results = {}
    for length in (1, 128, 256, 512, 528, 529, 1057):
        attn = math.ceil(length / pbs)
        total = fixed + attn
        extents = {"full": [(0, ratio)] * total, "optimized": [(0, ratio)] * fixed}
        for b in range(attn):
            extents["optimized"].append(
                ct.kernel_block_extent_for_attention_page(length, b, pbs, kbs, None))
        cpu_pages = torch.empty((total, phys_bytes), dtype=torch.uint8).pin_memory()
        gpu = [torch.empty((total, seg_page), dtype=torch.uint8, device=dev)
               for _ in range(segments_n)]
        # The first transfers over freshly page-locked memory run slower and
        # this buffer is new for every length: one untimed round trip of the
        # whole buffer first, the same for both arms.
        scratch = cpu_pages.to(dev)
        cpu_pages.copy_(scratch)
        torch.cuda.synchronize()
        del scratch
        segs = [swapper.CacheSegment(f"s{i}", (f"s{i}",), i * seg_page, seg_page)
                for i in range(segments_n)]
        sw = None
        if args.impl != "reference":
            sw = swapper.KVSwapper(0, segs, [g.view(-1) for g in gpu], [frozenset({0})] * segments_n,
                                   [ratio], kv_swap=cpu_pages.view(-1))
        stream = torch.cuda.Stream(dev)
        row = {}
        for kind, ext in extents.items():
            ids = list(range(total))
            first = [f for f, _ in ext]
            valid = [v for _, v in ext]
            for direction, is_in in (("H2D", True), ("D2H", False)):
                def submit():
                    if sw is not None:
                        sw.swap_blocks([0], ids, ids, [0] * total, first, valid, [None], is_in,
                                       stream=stream)
                        return
                    with torch.cuda.stream(stream):
                        for si, gp in enumerate(gpu):
                            for page, (f, v) in enumerate(ext):
                                off, ln = ct.byte_extent_for_kernel_blocks(seg_page, ratio, f, v)
                                if ln == 0:
                                    continue
                                c = cpu_pages[page].narrow(0, si * seg_page + off, ln)
                                g = gp[page].narrow(0, off, ln)
                                if is_in:
                                    g.copy_(c, non_blocking=True)
                                else:
                                    c.copy_(g, non_blocking=True)

                for _ in range(args.warmup):
                    submit()
                stream.synchronize()
                samples = []
                for _ in range(args.steps):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    submit()
                    b.record(stream)
                    b.synchronize()
                    samples.append(a.elapsed_time(b))
                samples.sort()
                nbytes = sum(ct.byte_extent_for_kernel_blocks(seg_page, ratio, f, v)[1]
                             for f, v in ext) * segments_n
                row[f"{kind}_{direction}"] = {
                    "p50_ms": samples[len(samples) // 2],
                    "p95_ms": samples[math.ceil(0.95 * len(samples)) - 1],
                    "bytes": nbytes,
                    "gbs_at_p50": nbytes / (samples[len(samples) // 2] / 1e3) / 1e9}
        results[str(length)] = row
        if sw is not None:
            sw.close()
        del gpu, cpu_pages
        torch.cuda.empty_cache()
    head = results["1057"]["optimized_H2D"]
    return {"impl": args.impl, "metric": METRIC, "value": head["gbs_at_p50"], "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "u8",
            "config": {"workload": "benchmark_composite_swap.py defaults: 8 segments, 3 fixed "
                                   "pages, 17,301,504-byte physical page, 528-token physical / "
                                   "16-token kernel blocks; value = optimized H2D at length 1057",
                       "api": "kvx_swap_blocks (one call per swap)" if args.impl != "reference"
                       else "restated harness loop: one torch copy_ per segment and page"},
            "per_length": results}


def run_config8(args):
    """Transfer forms of the configuration-3 migration at N >= 2 (pairs
    (i, i+N/2)): pull and push through the vector kernel (KVX_MODE_SM at
    several CTA counts) and through the TMA bulk kernel (KVX_MODE_SM_BULK),
    each timed like the default run's migration object and checked byte for
    byte across the pair.  One JSON line on rank 0."""
    import torch

    from aegaeon_b200 import _lib

    dist_ = Dist.init(use_pg=True)
    if dist_.world < 2:
        emit({"impl": args.impl, "note": "config 8 needs torchrun with 2 or more ranks"})
        return
    dev = torch.device("cuda", dist_.local_rank)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    variants = [("pull", "sm", 2, None), ("pull", "sm", 16, None), ("pull", "sm", 32, None),
                ("pull", "sm_bulk", None, None), ("push", "sm", 2, None),
                ("push", "sm", 16, None), ("push", "sm", 32, None), ("push", "sm_bulk", None, None)]
    variants += [("split", "sm", 16, f) for f in (0.3, 0.5)]
    out = {}
    # copy-engine peer copies of contiguous blocks over 1..8 streams, both directions
    from aegaeon_b200 import swapper, workloads

    sh = workloads.CFG3
    pages = [torch.empty(sh.num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
             for _ in range(sh.num_segments)]
    segs, _ = swapper.make_segments([((f"l{i}",), sh.num_blocks * sh.page_bytes)
                                     for i in range(sh.num_segments)], sh.num_blocks)
    sw = swapper.KVSwapper(dev.index, segs, pages, [frozenset({0})] * sh.num_segments, [1])
    handles = dist_.gather_obj(sw.export_kvcache_mem_handles())
    half = dist_.world // 2
    is_src = dist_.rank < half
    partner = dist_.rank + half if is_src else dist_.rank - half
    sw.register_kvcache_mem_handles(partner, None, handles[partner])
    st = torch.cuda.Stream(dev)
    for direction in ("pull", "push"):
        active = is_src if direction == "push" else not is_src
        for k in (1, 2, 4, 8):
            r = _peer_copy_peak(dist_, sw, partner, direction, active, st, 4096,
                                sh.num_segments, sh.page_bytes, streams=k)
            out[f"{direction}_copy_engine_{k}streams"] = {
                "per_pair_gbs": round(r["per_pair_gbs"], 3),
                "frac_of_nominal_900": round(r["per_pair_gbs"] / 900.0, 3)}
    dist_.barrier()
    sw.close()
    del pages
    torch.cuda.empty_cache()
    for direction, mode, per_sm, frac in variants:
        if per_sm:
            _lib.configure(sm_ctas_dev=per_sm * sms)
        r = migration_bench(dist_, dev, steps=args.steps, warmup=args.warmup,
                            direction=direction, mode=mode, extras=False, split=frac or 0.5)
        key = (f"{direction}_{mode}" + (f"_{per_sm * sms}ctas" if per_sm else "")
               + (f"_push{frac}" if frac else ""))
        out[key] = {k: (round(v, 3) if isinstance(v, float) else v) for k, v in r.items()}
    _lib.set_option("sm_ctas_dev", 0)  # back to the library default
    if dist_.rank == 0:
        best = max(out, key=lambda k: out[k]["per_pair_gbs"])
        emit({"impl": args.impl, "metric": "P->D migration GB/s per GPU pair (cfg3)",
              "value": out[best]["per_pair_gbs"], "unit": "GB/s", "n_gpus": dist_.world,
              "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
              "dtype": "u8", "config": {"workload": "cfg3 Qwen2.5-7B P->D migration, pairs "
                                                    "(i, i+N/2), 8 requests per pair"},
              "best": best, "variants": out})
    dist_.finish()


class FragSwap:
    """Swap-out and swap-in at once with scattered host slots.  The
    reference's CPU slab allocator hands out host slots from a free list
    (block_manager.py:942-1031), so after some churn the slots of one swap
    are scattered rows of the pool.  Per step `n` random blocks go out to `n`
    rows and `n` other blocks come in from `n` other rows of a `rows_total`-row
    pool; the rows are shuffled in groups of `group` consecutive rows (host
    runs of about `group` rows).  The cache and pool may be borrowed (the
    headline run's), else they are made here for `shape`."""

    def __init__(self, dev, shape, n: int, rows_total: int, pages=None, pool=None,
                 segments=None, sw=None):
        import torch

        from aegaeon_b200 import swapper, workloads

        self.dev, self.sh, self.n, self.rows_total = dev, shape, n, rows_total
        sh = shape
        self.own = sw is None
        if pages is None:
            gen = torch.Generator(device=dev).manual_seed(0)
            pages = []
            for _ in range(sh.num_segments):
                t = torch.empty(sh.num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
                workloads.fill_segment(t, sh, gen)
                pages.append(t)
            segments, _ = swapper.make_segments(
                [((f"l{i}",), sh.num_blocks * sh.page_bytes) for i in range(sh.num_segments)],
                sh.num_blocks)
            pool = torch.empty(rows_total * sh.composite_bytes, dtype=torch.uint8,
                               pin_memory=True)
            fill = torch.empty(GIB, dtype=torch.uint8, device=dev)
            for o in range(0, pool.numel(), GIB):
                fill.random_(0, 256, generator=gen)
                pool[o:o + GIB].copy_(fill[:pool.numel() - o])
            del fill
        if sw is None:
            sw = swapper.KVSwapper(dev.index, segments, pages, [frozenset({0})] * sh.num_segments,
                                   [1], kv_swap=pool)
        self.pages, self.pool, self.sw = pages, pool, sw
        self.comp = sh.composite_bytes

    def lists(self, k: int, group: int, shuffled: bool = True):
        from aegaeon_b200 import workloads

        n = self.n
        blocks = workloads.randperm(self.sh.num_blocks, 900 + k)
        if shuffled:
            order = workloads.randperm(self.rows_total // group, 500 + k)
            rows = [q * group + j for q in order for j in range(group)]
        else:
            rows = list(range(self.rows_total))
        return blocks[:n], rows[:n], rows[n:2 * n], blocks[n:2 * n]

    def run(self, steps: int, warmup: int, m_out, m_in, group: int = 1,
            shuffled: bool = True, host_bulk=(False, False), ctas=None) -> dict:
        """Times `steps` steps (either direction may be None); returns GB/s
        of both directions together, the modes AUTO resolved to and whether
        the last step's host rows and swapped-in blocks are exact.  `ctas`,
        when given, sets `sm_ctas_host` for the swap-out and the swap-in
        calls (and puts back the library's split by direction after each
        step)."""
        import torch

        from aegaeon_b200 import _lib

        sw, n = self.sw, self.n
        z, one = [0] * n, [1] * n

        def step(k):
            out_b, out_r, in_r, in_b = self.lists(k, group, shuffled)
            mo = mi = "-"
            e_out = e_in = None
            if m_out:
                _lib.set_option("host_bulk", int(host_bulk[0]))
                if ctas:
                    _lib.set_option("sm_ctas_host", ctas[0])
                e_out = sw.swap_blocks([0], out_b, out_r, z, z, one, [None], False,
                                       mode="sm" if m_out == "smb" else m_out,
                                       stream=sw.swap_out_stream)
                mo = _lib.last_mode_name() + ("+bulk" if host_bulk[0] else "")
            if m_in:
                _lib.set_option("host_bulk", int(host_bulk[1]))
                if ctas:
                    _lib.set_option("sm_ctas_host", ctas[1])
                e_in = sw.swap_blocks([1], in_r, in_b, z, z, one, [None], True,
                                      mode="sm" if m_in == "smb" else m_in,
                                      stream=sw.swap_in_stream)
                mi = _lib.last_mode_name() + ("+bulk" if host_bulk[1] else "")
            _lib.set_option("host_bulk", 0)
            if ctas:
                _lib.set_option("sm_ctas_host", 0)
            if e_in is not None:
                sw.swap_out_stream.wait_event(e_in)
            if e_out is not None:
                sw.swap_in_stream.wait_event(e_out)
            return mo, mi

        for k in range(warmup):
            step(k)
        torch.cuda.synchronize()
        cur = torch.cuda.current_stream(self.dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(cur)
        sw.swap_out_stream.wait_event(a)
        sw.swap_in_stream.wait_event(a)
        used = ("-", "-")
        for k in range(steps):
            used = step(warmup + k)
        cur.wait_stream(sw.swap_out_stream)
        cur.wait_stream(sw.swap_in_stream)
        b.record(cur)
        b.synchronize()
        t = a.elapsed_time(b) / 1e3
        moved = n * self.comp * ((1 if m_out else 0) + (1 if m_in else 0))
        exact = self._check(warmup + steps - 1, group, shuffled, bool(m_out), bool(m_in))
        return {"gbs": moved * steps / t / 1e9, "modes_used": "/".join(used), "bit_exact": exact}

    def run_split(self, steps: int, warmup: int, frac_ce: float) -> dict:
        """Both directions at once over scattered rows (groups of 1), each
        direction's entries split in two calls running together: the first
        part through the SM mode, the last `frac_ce` through the copy-engine
        mode, on four streams.  GB/s of both directions together and whether
        the last step is exact."""
        import torch

        sw, n = self.sw, self.n
        m = n - int(round(n * frac_ce))
        streams = [torch.cuda.Stream(self.dev) for _ in range(4)]

        def call(src, dst, lo, hi, is_in, mode, st):
            if hi <= lo:
                return None
            z, one = [0] * (hi - lo), [1] * (hi - lo)
            return sw.swap_blocks([1 if is_in else 0], src[lo:hi], dst[lo:hi], z, z, one, [None],
                                  is_in, mode=mode, stream=st)

        def step(k):
            out_b, out_r, in_r, in_b = self.lists(k, 1, True)
            evs = [call(in_r, in_b, 0, m, True, "sm", streams[0]),
                   call(out_b, out_r, 0, m, False, "sm", streams[1]),
                   call(in_r, in_b, m, n, True, "ce", streams[2]),
                   call(out_b, out_r, m, n, False, "ce", streams[3])]
            for st in streams:
                for e in evs:
                    if e is not None:
                        st.wait_event(e)

        for k in range(warmup):
            step(k)
        torch.cuda.synchronize()
        t = _timed(streams, lambda k: step(warmup + k), steps, self.dev)
        exact = self._check(warmup + steps - 1, 1, True, True, True)
        return {"gbs": 2 * n * self.comp * steps / t / 1e9, "bit_exact": exact}

    def _check(self, k, group, shuffled, check_out, check_in) -> bool:
        import torch

        sh, n, page = self.sh, self.n, self.sh.page_bytes
        out_b, out_r, in_r, in_b = self.lists(k, group, shuffled)
        rows = self.pool.view(self.rows_total, self.comp)
        ob = torch.tensor(out_b, device=self.dev)
        ib = torch.tensor(in_b, device=self.dev)
        for r0 in range(0, n, 256):
            r1 = min(n, r0 + 256)
            got = rows[torch.tensor(out_r[r0:r1])].to(self.dev).view(r1 - r0, sh.num_segments, page)
            src = rows[torch.tensor(in_r[r0:r1])].to(self.dev).view(r1 - r0, sh.num_segments, page)
            for si, p in enumerate(self.pages):
                pv = p.view(-1, page)
                if check_out and not torch.equal(got[:, si], pv[ob[r0:r1]]):
                    return False
                if check_in and not torch.equal(src[:, si], pv[ib[r0:r1]]):
                    return False
        return True

    def close(self):
        if self.own:
            self.sw.close()


def run_config9(args):
    """Fragmented host slots with both directions active, every transfer
    mode: a Qwen2.5-7B-shaped cache (28 layers x K/V, 16 KiB pages: 896 KiB
    host rows), 1024 blocks out to shuffled rows and 1024 in from other
    shuffled rows of a 4096-row pool per step, rows shuffled in groups of g
    (host runs of about g rows), each direction alone and both at once, and
    contiguous rows for comparison.  GB/s against the live copy-engine peaks
    of the same direction(s); every variant's last step checked byte for
    byte."""
    import torch

    from aegaeon_b200 import _lib, workloads

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    fs = FragSwap(dev, workloads.CFG3, 1024, 4096)
    peaks = host_link_peaks(dev)
    variants = [(True, 1, "auto", "auto", 0)]
    for g in (1, 2, 4, 8):
        for m in ("ce", "sm"):
            variants += [(True, g, m, m, 1), (True, g, m, None, 1), (True, g, None, m, 1)]
    variants += [(False, 1, "ce", "ce", 1), (False, 1, "sm", "sm", 1), (True, 1, "ce", "ce", 2)]
    # one mechanism per direction
    variants += [(True, 1, "ce", "sm", 1), (True, 1, "sm", "ce", 1)]
    # SM mode through the TMA bulk kernel (16 KiB bulk copies to / from host rows)
    variants += [(True, 1, "smb", "smb", 1), (True, 1, "smb", None, 1), (True, 1, None, "smb", 1),
                 (True, 1, "smb", "sm", 1), (True, 1, "sm", "smb", 1),
                 (False, 1, "smb", "smb", 1)]
    out = {}
    for shuffled, group, m_out, m_in, streams in variants:
        if streams:
            _lib.set_option("ce_streams", streams)
        bulk_modes = {"smb"}
        # "smb": SM mode with host_bulk set for that direction's calls
        r = fs.run(args.steps, args.warmup, m_out, m_in, group, shuffled,
                   host_bulk=(m_out in bulk_modes, m_in in bulk_modes))
        both = m_out is not None and m_in is not None
        peak = peaks["bidir_gbs"] if both else (peaks["d2h_gbs"] if m_out else peaks["h2d_gbs"])
        key = (("shuffled" + str(group)) if shuffled else "contiguous") + \
            f":{m_out or '-'}/{m_in or '-'}" + (f"/{streams}streams" if streams else "")
        out[key] = {"gbs": round(r["gbs"], 2), "frac": round(r["gbs"] / peak, 3),
                    "modes_used": r["modes_used"], "bit_exact": r["bit_exact"]}
    _lib.set_option("ce_streams", 1)
    # both directions on the SMs, scattered rows: CTAs of the swap-out (host
    # writes) and swap-in (host reads) kernels
    for co, ci in ((148, 148), (74, 148), (96, 148), (111, 148), (96, 185), (111, 185),
                   (80, 222), (48, 148), (74, 74)):
        r = fs.run(args.steps, args.warmup, "sm", "sm", 1, True, ctas=(co, ci))
        out[f"shuffled1:sm/sm:ctas{co}/{ci}"] = {
            "gbs": round(r["gbs"], 2), "frac": round(r["gbs"] / peaks["bidir_gbs"], 3),
            "modes_used": r["modes_used"], "bit_exact": r["bit_exact"]}
    # each direction split between the SM path and the copy engines at once
    for f in (0.1, 0.3, 0.5):
        r = fs.run_split(args.steps, args.warmup, f)
        out[f"shuffled1:split_ce{f}"] = {"gbs": round(r["gbs"], 2),
                                         "frac": round(r["gbs"] / peaks["bidir_gbs"], 3),
                                         "modes_used": "sm+ce/sm+ce", "bit_exact": r["bit_exact"]}
    # the TMA bulk kernel both ways, sized so both directions stay resident
    _lib.set_option("bulk_ctas_per_sm", 1)
    _lib.set_option("bulk_waves", 1)
    r = fs.run(args.steps, args.warmup, "smb", "smb", 1, True, host_bulk=(True, True))
    _lib.set_option("bulk_ctas_per_sm", 2)
    _lib.set_option("bulk_waves", 16)
    out["shuffled1:smb/smb:1cta_per_sm_1wave"] = {
        "gbs": round(r["gbs"], 2), "frac": round(r["gbs"] / peaks["bidir_gbs"], 3),
        "modes_used": r["modes_used"], "bit_exact": r["bit_exact"]}
    fs.close()
    return {"impl": args.impl, "metric": METRIC, "value": out["shuffled1:auto/auto"]["gbs"],
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "u8", "data": "synthetic, seeded",
            "config": {"workload": "fragmented host slots: Qwen2.5-7B-shaped cache "
                                   f"({workloads.CFG3.num_segments} x 16 KiB pages, "
                                   f"{workloads.CFG3.composite_bytes} B host rows), 1024 blocks "
                                   "out and 1024 in per step over a 4096-row pool"},
            "bidir_peak_gbs": peaks["bidir_gbs"], "h2d_peak_gbs": peaks["h2d_gbs"],
            "d2h_peak_gbs": peaks["d2h_gbs"], "modes": out}


def run_config10(args):
    """The headline configuration-2 step under the copy-engine mode's knobs:
    the staged copies cut into pieces of at most P bytes (`ce_max_copy`), and
    the staging gather/scatter kernel (TMA bulk at 1 or 2 CTAs per SM, or the
    vector kernel at several CTA counts).  Per variant: GB/s of both
    directions together, and the live gather/scatter kernel's fraction of
    the HBM peak (mean launch, and over the union of launch intervals)."""
    import torch

    from aegaeon_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    per_dir = blocks_per_direction(args.blocks, 1, args.cache_blocks)
    peaks = host_link_peaks(dev)
    bench = SwapBench(dev, per_dir, args.cache_blocks)
    lists = [bench.step_lists(k) for k in range(args.warmup + args.steps)]
    hbm = measured_peaks().get("hbm_gbs", 6650.0)

    def timed(tag, out, staging_bulk=True):
        for k in range(args.warmup):
            bench.issue(lists[k], args.mode)
        torch.cuda.synchronize()
        _lib.kernel_timing_read()
        _lib.kernel_timing(True)
        t = bench.timed_device(args.steps, args.mode, lambda k: lists[args.warmup + k])
        _lib.kernel_timing(False)
        n_l, ms, busy, nbytes = _lib.kernel_timing_read()
        iso = bench.kernel_roofline(mode_bulk=staging_bulk)
        out.setdefault(tag, []).append({
            "gbs": round(bench.bytes_per_step * args.steps / t / 1e9, 2),
            "kernel_frac": round(nbytes / (ms / 1e3) / 1e9 / hbm, 3) if ms else None,
            "kernel_frac_union": round(nbytes / (busy / 1e3) / 1e9 / hbm, 3) if busy else None,
            "isolated_frac": round(iso["algorithmic_bytes"] / iso["seconds"] / 1e9 / hbm, 3),
            "launches": n_l})


    pieces = {}
    for piece_mib in (0, 256):
        _lib.set_option("ce_max_copy", piece_mib << 20)
        timed(f"{piece_mib}MiB" if piece_mib else "unlimited", pieces)
    _lib.set_option("ce_max_copy", 0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    kernels = {}
    for tag, opts in (("bulk_1wave", {"staging_bulk": 1, "bulk_waves": 1}),
                      ("bulk_8waves", {"staging_bulk": 1, "bulk_waves": 8}),
                      ("bulk_16waves", {"staging_bulk": 1, "bulk_waves": 16}),
                      ("bulk_32waves", {"staging_bulk": 1, "bulk_waves": 32}),
                      ("bulk_1perSM_16waves", {"staging_bulk": 1, "bulk_ctas_per_sm": 1,
                                               "bulk_waves": 32}),
                      ("vec32_32perSM", {"staging_bulk": 0, "sm_ctas_dev": 32 * sms}),
                      ("bulk_16waves_again", {"staging_bulk": 1, "bulk_ctas_per_sm": 2,
                                              "bulk_waves": 16})):
        for k, v in opts.items():
            _lib.set_option(k, v)
        timed(tag, kernels, staging_bulk=bool(opts["staging_bulk"]))
    _lib.set_option("staging_bulk", 1)
    _lib.set_option("bulk_ctas_per_sm", 2)
    _lib.set_option("bulk_waves", 16)
    _lib.set_option("sm_ctas_dev", 0)
    bench.close()
    best = max(x["gbs"] for v in list(pieces.values()) + list(kernels.values()) for x in v)
    return {"impl": args.impl, "metric": METRIC, "value": best,
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "u8",
            "config": cfg2_config(per_dir, args.cache_blocks, 1),
            "bidir_peak_gbs": peaks["bidir_gbs"], "by_piece": pieces,
            "by_staging_kernel": kernels}


def run_config11(args):
    """Weight upload of a model switch from pageable host memory: the
    Qwen1.5-14B TP-2 shard (14.17 GB bf16) as four safetensors-sized
    storages in ordinary (pageable) host memory, uploaded to the GPU.  Both
    arms run here on the same bytes and are checked byte for byte:
    * kvx: switch.upload_weights (kvx_upload_weights: 64 MiB pieces through
      two page-locked bounce buffers, host threads filling one while the
      copy engine drains the other);
    * reference: pipeline_storage_transfer restated
      (quick_model_loader/quick_model_loader/model_loader.py:348-369): per
      storage a page-locked buffer of its size (allocated once, before the
      timing, as the loader's pinned allocator does), 16 cuts, each copied
      host -> page-locked, then the stream synchronized, then copied to the
      device non-blocking; one final synchronize.
    Wall-clock GB/s (the host copies are part of the work)."""
    import torch

    from aegaeon_b200 import switch, workloads

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    ws = workloads.WeightShard()
    cut = -(-ws.nbytes // 4)
    sizes = [min(cut, ws.nbytes - o) for o in range(0, ws.nbytes, cut)]
    gen = torch.Generator().manual_seed(11)
    hosts = [torch.randint(0, 256, (n,), dtype=torch.uint8, generator=gen) for n in sizes]
    devs = [torch.empty(n, dtype=torch.uint8, device=dev) for n in sizes]
    stream = torch.cuda.Stream(dev)
    pinned = [torch.empty(n, dtype=torch.uint8, pin_memory=True) for n in sizes]

    def kvx_once():
        switch.upload_weights(list(zip(devs, hosts)), chunk_bytes=64 << 20, stream=stream)
        stream.synchronize()

    def create_cuts(size, cuts_num):
        base, extra = divmod(size, cuts_num)
        out, start = [], 0
        for i in range(cuts_num):
            end = start + base + (1 if i < extra else 0)
            out.append((start, end))
            start = end
        return out

    def ref_once():
        with torch.cuda.stream(stream):
            for d, h, pb in zip(devs, hosts, pinned):
                size = h.numel()
                for a, b in create_cuts(size, 1 if size <= GIB else 16):
                    pb[a:b].copy_(h[a:b], non_blocking=True)
                    stream.synchronize()
                    d[a:b].copy_(pb[a:b], non_blocking=True)
            stream.synchronize()

    out = {}
    for name, fn in (("kvx", kvx_once), ("reference", ref_once)):
        for d in devs:
            d.zero_()
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            fn()
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        exact = all(torch.equal(d.cpu(), h) for d, h in zip(devs, hosts))
        t = statistics.median(times)
        out[name] = {"seconds": round(t, 4), "gbs": round(ws.nbytes / t / 1e9, 2),
                     "bit_exact": exact}
    return {"impl": "kvx+reference", "metric": METRIC, "value": out["kvx"]["gbs"], "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "dtype": "u8", "data": "synthetic, seeded",
            "config": {"workload": f"Qwen1.5-14B TP-2 shard ({ws.nbytes} B) as 4 pageable "
                                   "storages uploaded to the GPU"},
            "arms": out, "ratio": round(out["kvx"]["gbs"] / out["reference"]["gbs"], 2)}


SMALL_CALL_BLOCKS = (1, 2, 4, 16, 64, 256)


def run_config7(args):
    """Small swap calls, as a decode turn issues them: latency of one
    ``swap`` call (the reference op's interface) moving n scattered blocks of
    one cfg2 K tensor ([4096,16,32,128] fp16, 128 KiB blocks) to host slots,
    and one moving them back in to other blocks, for n in SMALL_CALL_BLOCKS.
    Per n: warm-up calls, then steps x 20 calls per direction timed with CUDA
    events on the current stream and with the host clock (these calls are
    bound by host-side issue cost, so the two agree).  Afterwards the moved
    blocks are compared byte for byte."""
    import torch

    from aegaeon_b200 import _lib, ops, workloads

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    sh = workloads.CFG2
    shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
    gen = torch.Generator(device=dev).manual_seed(0)
    cache = torch.empty(shape, dtype=sh.dtype, device=dev).uniform_(-2, 2, generator=gen)
    host = torch.zeros((max(SMALL_CALL_BLOCKS),) + shape[1:], dtype=sh.dtype).pin_memory()
    ref = _ref_module() if args.impl == "reference" else None
    torch.cuda.synchronize()

    def swap(src, dst, is_in):
        if ref is not None:
            ref.swap(src, dst, is_in, cache, host)
        else:
            ops.swap(src, dst, is_in, cache, host, mode=args.mode)

    perm = workloads.randperm(sh.num_blocks, 7)
    calls = max(args.steps, 1) * 20
    cur = torch.cuda.current_stream(dev)
    per_n, exact = {}, True
    for n in SMALL_CALL_BLOCKS:
        out_ids, in_ids, slots = perm[:n], perm[n:2 * n], list(range(n))
        row = {}
        for name, src, dst, is_in in (("out", out_ids, slots, False),
                                      ("in", slots, in_ids, True)):
            for _ in range(max(args.warmup, 3) * 20):
                swap(src, dst, is_in)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            a.record(cur)
            for _ in range(calls):
                swap(src, dst, is_in)
            b.record(cur)
            wall = time.perf_counter() - t0
            b.synchronize()
            row[f"{name}_us"] = a.elapsed_time(b) * 1e3 / calls
            row[f"{name}_host_us"] = wall * 1e6 / calls
            if ref is None:
                row[f"{name}_mode"] = _lib.last_mode_name()
        exact &= torch.equal(cache[in_ids].view(torch.uint8), cache[out_ids].view(torch.uint8))
        exact &= torch.equal(host[:n].to(dev).view(torch.uint8), cache[out_ids].view(torch.uint8))
        per_n[str(n)] = row
    value = (per_n["1"]["out_us"] + per_n["1"]["in_us"]) / 2
    return {"impl": args.impl, "metric": "us per small swap call (n=1 block; table for n up "
                                         "to 256)",
            "value": value, "unit": "us", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": value / 1e3, "higher_is_better": False,
            "dtype": "u8", "data": "synthetic: fp16 U(-2,2) from seed 0, seeded block ids",
            "config": {"workload": "cfg2 K tensor [4096,16,32,128] fp16 (128 KiB blocks); "
                                   "per n: one call moving n scattered blocks out to host "
                                   "slots 0..n-1, one moving them back in to other blocks",
                       "blocks_per_call": list(SMALL_CALL_BLOCKS),
                       "calls_per_direction_and_n": calls,
                       "api": "aegaeon.ops.swap (reference op)" if ref is not None
                       else "aegaeon_b200.ops.swap -> kvx_swap",
                       "transfer_mode": None if ref is not None else args.mode},
            "per_n": per_n, "bit_exact": bool(exact),
            "e2e": {"value": (per_n["1"]["out_host_us"] + per_n["1"]["in_host_us"]) / 2,
                    "unit": "us", "h2d_bytes_per_step": sh.page_bytes,
                    "d2h_bytes_per_step": sh.page_bytes}}


def main():
    # Exactly one JSON line on stdout: libraries (NCCL prints its version)
    # write to fd 1 too, so fd 1 points at stderr while the benchmark runs and
    # the line goes to a private copy of the original stdout.
    out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    global _OUT
    _OUT = out
    args = parse_args()
    if args.set:
        from aegaeon_b200 import _lib

        for item in args.set:
            name, _, value = item.partition("=")
            _lib.set_option(name.strip(), int(value, 0))
    if args.config != 2:
        rank = int(os.environ.get("RANK", "0"))
        if args.config in (1, 4, 7, 9, 10, 11) and rank != 0:
            return
        if args.config == 3:
            if args.impl != "reference":
                emit({"impl": "kvx", "note": "config 3 (migration) is measured by the default "
                      "run at N >= 2 (its 'migration' object)"})
                return
            if rank == 0:
                emit(run_config3_reference(args))
            return
        if args.config == 8:
            run_config8(args)
            return
        if args.config == 6:
            if rank == 0:
                emit(run_config6(args))
            return
        fn = {1: run_config1, 4: run_config4, 5: run_config5, 7: run_config7,
              9: run_config9, 10: run_config10, 11: run_config11}[args.config]
        line = fn(args)
        if line is not None:
            emit(line)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_kvx(args)


if __name__ == "__main__":
    main()
