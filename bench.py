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
(plan_swap_lists -> KVSwapper.swap_blocks -> wait), with the payload crossing
the host link inside the timed region.  ``roofline`` is the binding host link
(measured copy-engine peak, both directions together); ``kernel_roofline`` the
device-side gather kernel against the measured HBM copy peak.  At N >= 2 a
``migration`` object adds configuration 3 (NVLink P->D migration, pairs
(i, i+N/2)).

``--impl reference`` times the reference's own swap op (ops/swap.cu, built
from the reference sources into oracle/_ref) on the same configuration: one
call per K or V tensor, one cudaMemcpyAsync per block, out and in on two
streams.  Under torchrun only rank 0 runs it.
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
    p.add_argument("--config", type=int, choices=[1, 2, 3, 4, 5, 6, 7], default=2,
                   help="BASELINE.json configuration (2 = the headline line; 3 is the "
                        "migration object of the N>=2 line; 7 = latency of small swap calls)")
    p.add_argument("--mode", default="auto", help="transfer mode: auto|sm|ce|ce_extent")
    p.add_argument("--blocks", type=int, default=1024, help="blocks per direction per step")
    p.add_argument("--cache-blocks", type=int, default=4096,
                   help="blocks per K/V tensor (4096 in the configuration; smaller only for "
                        "profiling captures)")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-migration", action="store_true")
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
    rank's device time).  Best of 5 windows after a warm-up; values returned
    per GPU (box / N) plus the box figure of both directions."""
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
        for _ in range(5):
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
        """Wall clock through the public API from block tables."""
        from aegaeon_b200 import block_table as bt

        torch = self.torch
        group = (bt.CacheGroupConfig("attention", 16, 16),)
        per_req = 16  # 256-token requests: 16 full pages each
        t0 = time.perf_counter()
        for k in range(steps):
            out_ids, rows_out, rows_in, in_ids = self.step_lists(1000 + k)
            n_req = self.per_dir // per_req
            out_plans = [(bt.BlockTable(0, (1,), group, [out_ids[r * per_req:(r + 1) * per_req]]),
                          256) for r in range(n_req)]
            in_plans = [(bt.BlockTable(-1, (1,), group, [rows_in[r * per_req:(r + 1) * per_req]]),
                         256) for r in range(n_req)]
            lo = bt.plan_swap_lists(out_plans, rows_out)
            li = bt.plan_swap_lists(in_plans, in_ids)
            e_out = self.sw.swap_blocks(list(range(n_req)), lo.source_block_ids,
                                        lo.target_block_ids, lo.group_ids,
                                        lo.first_kernel_blocks, lo.valid_kernel_blocks,
                                        [None] * n_req, False, mode=mode, stream=self.s_out)
            e_in = self.sw.swap_blocks(list(range(n_req)), li.source_block_ids,
                                       li.target_block_ids, li.group_ids,
                                       li.first_kernel_blocks, li.valid_kernel_blocks,
                                       [None] * n_req, True, mode=mode, stream=self.s_in)
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


def cpu_baseline(seconds: float) -> dict:
    """The same block gather on the host cores (CPU restatement of the copy,
    multi-threaded), on a bounded sample."""
    import numpy as np

    from oracle import oracle as orc

    threads = len(os.sched_getaffinity(0))
    page = 131072
    nsrc, ngather = 16384, 4096
    src = np.empty(nsrc * page, np.uint8)
    src[::4096] = 1  # touch pages
    dst = np.empty(ngather * page, np.uint8)
    import torch

    ids = torch.randperm(nsrc, generator=torch.Generator().manual_seed(0))[:ngather].tolist()
    slots = list(range(ngather))
    orc.copy_blocks_mt(ids, slots, src, dst, page, threads)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        orc.copy_blocks_mt(ids, slots, src, dst, page, threads)
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    # The same gather with torch.index_select over a block-shaped host tensor,
    # on all host threads (the CPU path named by the configuration).
    import torch

    torch.set_num_threads(threads)
    src_t = torch.from_numpy(src).view(nsrc, page)
    idx = torch.tensor(ids, dtype=torch.int64)
    out_t = torch.index_select(src_t, 0, idx)
    t1 = time.perf_counter()
    reps_t = 0
    while time.perf_counter() - t1 < min(seconds, 5.0):
        torch.index_select(src_t, 0, idx, out=out_t)
        reps_t += 1
    torch_gbs = reps_t * ngather * page / (time.perf_counter() - t1) / 1e9
    cpu = "unknown"
    try:
        cpu = [l for l in open("/proc/cpuinfo") if l.startswith("model name")][0].split(":")[1].strip()
    except (OSError, IndexError):
        pass
    return {"value": reps * ngather * page / dt / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port", "torch_index_select_gbs": torch_gbs,
            "sample": f"{reps} x gather of {ngather} random 128 KiB blocks (512 MiB) from a "
                      f"2 GiB host cache, {threads} threads, {dt:.1f} s; cpu {cpu}"}


MIGRATION_SMALL_BLOCKS = (1, 4, 16, 64)


def migration_bench(dist_, dev, steps: int, warmup: int, direction: str = "pull") -> dict:
    """Configuration 3 at N >= 2: pairs (i, i + N/2), rank i the prefill side.
    pull: the decode rank maps the prefill rank's cache and copies the blocks
    in (loads over NVLink); push: the prefill rank stores them into the
    decode rank's mapped cache."""
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
    active = is_src if direction == "push" else not is_src
    if active:
        sw.register_kvcache_mem_handles(partner, None, handles[partner])
    stream = torch.cuda.Stream(dev)

    def run():
        if active:
            sw.migrate_blocks([pair], partner, plan.source_ids, plan.target_ids, None,
                              direction=direction, stream=stream)

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
    # Small calls: the plan's first n blocks (all 56 segments), as a decode
    # rank pulls a short request; µs per call, device time, max over ranks.
    # The same source/target pairs as the plan, so the parity check below
    # still holds.
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
    # Parity of the timed push: the decode rank's blocks equal the prefill
    # rank's (checked on a digest of the moved pages, both sides on device).
    moved = [p.view(-1, sh.page_bytes)[plan.source_ids if is_src else plan.target_ids]
             for p in pages]
    digest = torch.stack([m.view(torch.int32).sum(dtype=torch.int64) for m in moved]).cpu().tolist()
    digests = dist_.gather_obj(digest)
    parity = all(digests[r] == digests[r + half] for r in range(half))
    del moved
    nccl = nccl_comparison(dist_, dev, sw, plan, is_src, partner, steps, warmup)
    sw.close()
    del pages
    total = half * nbytes * steps
    per_pair = nbytes * steps / t / 1e9
    return {"config": "cfg3 Qwen2.5-7B P->D migration: 28 layers, 4 kv heads, 128 dim, bf16, "
                      "block 16; 8 requests/pair, prompts U{512..8192}; pairs (i, i+N/2); "
                      f"{direction}: " + ("decode rank loads from the prefill rank's mapped "
                                          "cache over NVLink" if direction == "pull" else
                                          "prefill rank stores into the decode rank's mapped "
                                          "cache over NVLink"),
            "pairs": half, "bytes_per_pair": nbytes, "value": total / t / 1e9, "unit": "GB/s",
            "per_pair_gbs": per_pair, "nvlink_peer_copy_gbs": 770.0,
            "frac_of_measured_peer_copy": per_pair / 770.0, "frac_of_nominal_900": per_pair / 900.0,
            "ms_per_step": t / steps * 1e3, "bit_exact": parity,
            "small_calls_us": small,
            "small_calls_how": "per n: one migrate_blocks call moving n blocks x 56 segments "
                               f"({sh.composite_bytes // 1024} KiB per block), 200 calls "
                               "after 20 warm-up, CUDA events, max over ranks",
            "nccl_sendrecv": {"value": half * nbytes / nccl / 1e9, "unit": "GB/s",
                              "per_pair_gbs": nbytes / nccl / 1e9,
                              "how": "gather blocks into a contiguous buffer (kvx kernel), "
                                     "torch.distributed send/recv (NCCL), scatter on the "
                                     "decode rank; CUDA events, max over ranks"}}


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
def run_kvx(args):
    import torch

    from aegaeon_b200 import _lib, workloads

    dist_ = Dist.init(use_pg=True)
    dev = torch.device("cuda", dist_.local_rank)
    per_dir = args.blocks
    # Host RAM guard: 2 * per_dir rows of 8 MiB page-locked per rank.
    try:
        avail = int([l for l in open("/proc/meminfo") if l.startswith("MemAvailable")][0].split()[1]) * 1024
        rows_fit = int(0.45 * avail / dist_.world / workloads.CFG2.composite_bytes)
        if 2 * per_dir > rows_fit:
            per_dir = max(64, rows_fit // 2 // 16 * 16)
    except (OSError, IndexError, ValueError):
        pass
    peaks = host_link_peaks(dev, dist_)  # all ranks at once: the box's concurrent peak
    box_peak = peaks["box_bidir_gbs"]
    per_dir = min(per_dir, args.cache_blocks // 2)
    bench = SwapBench(dev, per_dir, args.cache_blocks)
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
    bench.close()
    del bench
    torch.cuda.empty_cache()
    mig = None
    if dist_.world >= 2 and not args.no_migration:
        mig = migration_bench(dist_, dev, steps=args.steps, warmup=args.warmup,
                              direction=args.migration_direction)
    mp = measured_peaks()
    hbm_peak = mp.get("hbm_gbs", 6650.0)
    per_gpu = value / dist_.world
    line = None
    if dist_.rank == 0:
        # algorithmic bytes per launch / mean launch duration
        achieved_k = k_bytes / (k_ms / 1e3) / 1e9 if k_ms > 0 else None
        traffic = traffic_from_profile()
        k_name = ("kvx_copy_bulk<GridList>" if mode_used == "ce" else "kvx_copy_vec<GridList>")
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
            "config": {
                "workload": "cfg2 Llama-2-7B-shaped per-GPU swap: 32 layers x separate K/V "
                            f"[{args.cache_blocks},16,32,128] fp16; per step "
                            f"{per_dir} random blocks out (host rows 0..{per_dir - 1}) and "
                            f"{per_dir} other random blocks in, on the swap-out / swap-in "
                            "streams concurrently",
                "blocks_per_direction": per_dir,
                "bytes_per_step_per_gpu": bench_bytes(per_dir),
                "api": "KVSwapper.swap_blocks (Worker.swap_blocks replacement) -> "
                       "kvx_swap_blocks",
                "transfer_mode": f"{args.mode} -> {mode_used}",
                "l2": "no flush needed: 8 GiB per direction per step, far larger than the "
                      "126 MB L2",
                "parallelism": f"independent swap per GPU x{dist_.world}",
            },
            "roofline": {
                "bound": "hbm",
                "kernel": k_name,
                "achieved": achieved_k,
                "peak": hbm_peak,
                "unit": "GB/s",
                "frac": (achieved_k / hbm_peak) if achieved_k else None,
                "traffic": traffic,
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
                               "barrier-started windows; box = all bytes / slowest rank; "
                               "per-GPU share shown (the step is bidirectional)",
                "box_peak_gbs": box_peak,
                "peak_h2d_gbs": peaks["h2d_gbs"],
                "peak_d2h_gbs": peaks["d2h_gbs"],
                "nominal_gbs_per_direction": 63.0,
                "note": "the binding roofline of the swap: payload crosses PCIe Gen5 x16",
            },
            "e2e": {
                "value": e2e,
                "unit": "GB/s",
                "h2d_bytes_per_step": per_dir * workloads.CFG2.composite_bytes * dist_.world,
                "d2h_bytes_per_step": per_dir * workloads.CFG2.composite_bytes * dist_.world,
                "api": "block tables -> plan_swap_lists -> KVSwapper.swap_blocks -> stream sync",
                "seconds": t_e2e,
            },
            "gpu_launches": launches,
            "clocks": clk,
        }
        if mig is not None:
            line["migration"] = mig
    if dist_.rank == 0 and dist_.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    dist_.finish()
    if line is not None:
        emit(line)


def bench_bytes(per_dir: int) -> int:
    from aegaeon_b200 import workloads

    return 2 * per_dir * workloads.CFG2.composite_bytes


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from aegaeon_b200 import workloads

    try:
        from oracle import build_ref

        ref = build_ref.load_module()
    except Exception as e:  # noqa: BLE001
        emit({"impl": "reference", "unavailable": f"reference op not built: {e}"})
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sh = workloads.CFG2
    per_dir = args.blocks
    gen = torch.Generator(device=dev).manual_seed(0)
    caches = []
    for _ in range(sh.num_segments):
        t = torch.empty((sh.num_blocks, 16, sh.kv_heads, sh.head_dim), dtype=sh.dtype, device=dev)
        t.uniform_(-2.0, 2.0, generator=gen)
        caches.append(t)
    out_host = [torch.empty((per_dir, 16, sh.kv_heads, sh.head_dim), dtype=sh.dtype).pin_memory()
                for _ in range(sh.num_segments)]
    in_host = [torch.empty_like(h).pin_memory() for h in out_host]
    s_out, s_in = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    slots = list(range(per_dir))
    live = args.ref_variant == "live-loop"
    if live:
        # composite host rows: row r holds every segment's page of one block
        page = sh.page_bytes
        pool_out = torch.empty((per_dir, sh.num_segments * page), dtype=torch.uint8).pin_memory()
        pool_in = torch.empty((per_dir, sh.num_segments * page), dtype=torch.uint8).pin_memory()
        gpu_pages = [c.view(torch.uint8).view(sh.num_blocks, page) for c in caches]

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
        out_ids, in_ids = workloads.swap_step_ids(sh.num_blocks, per_dir, k)
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
    t = a.elapsed_time(b) / 1e3
    nbytes = 2 * per_dir * sh.composite_bytes * args.steps
    value = nbytes / t / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic: fp16 U(-2,2) from seed 0, block ids from seeded randperm",
        "config": {
            "workload": "cfg2 Llama-2-7B-shaped per-GPU swap: 32 layers x separate K/V "
                        f"[4096,16,32,128] fp16; per step {per_dir} random blocks out and "
                        f"{per_dir} in, out and in on two streams",
            "blocks_per_direction": per_dir,
            "api": ("restated Worker.swap_blocks hot loop (worker.py:2270-2329): one torch "
                    "copy_(non_blocking=True) per segment and block into composite host rows"
                    if live else
                    "reference aegaeon.ops.swap (ops/swap.cu, built unmodified from the "
                    "reference sources): one call per K/V tensor, one cudaMemcpyAsync per block"),
            "l2": "no flush needed: 8 GiB per direction per step",
        },
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": 1, "kind": "reference",
                         "sample": f"full workload, {args.steps} steps; one host thread issues "
                                   f"{2 * per_dir * sh.num_segments} copies per step"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0, "wall_clock_gbs": nbytes / wall / 1e9},
        "gpu_launches": 0,
        "clocks": clk,
    }
    emit(line)


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


def run_config1(args):
    """Qwen3-4B round trip through the per-tensor op: 72 tensors [1024,16,8,128]
    bf16 N(0,1); 256 blocks out to slots 0..255, then back in to a fresh
    permutation of a zeroed cache; bit-exact check of the round trip."""
    import torch

    from aegaeon_b200 import ops, workloads

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    sh = workloads.CFG1
    gen = torch.Generator(device=dev).manual_seed(0)
    shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
    caches = [torch.empty(shape, dtype=sh.dtype, device=dev).normal_(generator=gen)
              for _ in range(sh.num_segments)]
    back = [torch.zeros_like(c) for c in caches]
    n = 256
    hosts = [torch.empty((n,) + shape[1:], dtype=sh.dtype).pin_memory() for _ in caches]
    out_ids = workloads.randperm(sh.num_blocks, 0)[:n]
    in_ids = workloads.randperm(sh.num_blocks, 1)[:n]
    slots = list(range(n))
    ref = _ref_module() if args.impl == "reference" else None

    def swap(src, dst, is_in, cache, host):
        if ref is not None:
            ref.swap(src, dst, is_in, cache, host)
        else:
            ops.swap(src, dst, is_in, cache, host, mode=args.mode)

    def step(_k):
        for c, h in zip(caches, hosts):
            swap(out_ids, slots, False, c, h)
        for c, h in zip(back, hosts):
            swap(slots, in_ids, True, c, h)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    t = _timed([], step, args.steps, dev)
    wall = time.perf_counter() - t0
    exact = all(torch.equal(b[in_ids].view(torch.uint8), c[out_ids].view(torch.uint8))
                for b, c in zip(back, caches))
    nbytes = 2 * sh.num_segments * n * sh.page_bytes * args.steps
    value = nbytes / t / 1e9
    return {"impl": args.impl, "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "dtype": "u8",
            "config": {"workload": "cfg1 Qwen3-4B round trip: 36 layers x separate K/V "
                                   "[1024,16,8,128] bf16 N(0,1) seed 0; 256 blocks out to "
                                   "slots 0..255 then in to a fresh permutation, 72 swap "
                                   "calls per direction",
                       "api": "aegaeon.ops.swap (reference op)" if ref is not None
                       else "aegaeon_b200.ops.swap -> kvx_swap",
                       "transfer_mode": None if ref is not None else args.mode},
            "bit_exact_round_trip": exact,
            "e2e": {"value": nbytes / wall / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": nbytes // 2 // args.steps,
                    "d2h_bytes_per_step": nbytes // 2 // args.steps}}


def run_config4(args):
    """Model-switch overlap: swap-in of 2048 cfg2 blocks (16 GiB) while a
    Qwen1.5-14B TP-2 weight shard (14.17 GB bf16) is uploaded from
    page-locked host memory in 64 MiB chunks on a second stream."""
    import torch

    from aegaeon_b200 import _lib, swapper, workloads

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    sh = workloads.CFG2
    n = 2048
    gen = torch.Generator(device=dev).manual_seed(0)
    ws = workloads.WeightShard()
    w_dev = torch.empty(ws.nbytes, dtype=torch.uint8, device=dev)
    w_host = torch.empty(ws.nbytes, dtype=torch.uint8).pin_memory()
    w_host[:: 1 << 20].fill_(1)
    in_ids = workloads.randperm(sh.num_blocks, 7)[:n]
    s_kv, s_w = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ref = _ref_module() if args.impl == "reference" else None
    if ref is None:
        pages = [torch.empty(sh.num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
                 for _ in range(sh.num_segments)]
        segs, comp = swapper.make_segments([((f"l{i}",), sh.num_blocks * sh.page_bytes)
                                            for i in range(sh.num_segments)], sh.num_blocks)
        pool = torch.empty(n * comp, dtype=torch.uint8).pin_memory()
        pool[:: 1 << 20].fill_(2)
        sw = swapper.KVSwapper(0, segs, pages, [frozenset({0})] * sh.num_segments, [1],
                               kv_swap=pool)
        rows = list(range(n))

        def step(_k):
            sw.swap_blocks([0], rows, in_ids, [0] * n, [0] * n, [1] * n, [None], True,
                           mode=args.mode, stream=s_kv)
            _lib.check(_lib.lib().kvx_upload_chunked(w_dev.data_ptr(), w_host.data_ptr(),
                                                     ws.nbytes, 64 << 20, s_w.cuda_stream))
    else:
        shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
        caches = [torch.empty(shape, dtype=sh.dtype, device=dev) for _ in range(sh.num_segments)]
        hosts = [torch.empty((n,) + shape[1:], dtype=sh.dtype).pin_memory() for _ in caches]
        slots = list(range(n))
        offs = [0]
        for t in ws.tensors:
            offs.append(offs[-1] + 2 * t)

        def step(_k):
            with torch.cuda.stream(s_kv):
                for c, h in zip(caches, hosts):
                    ref.swap(slots, in_ids, True, c, h)
            with torch.cuda.stream(s_w):  # one copy per weight tensor (quick_loader.py:413)
                for a, b in zip(offs[:-1], offs[1:]):
                    w_dev[a:b].copy_(w_host[a:b], non_blocking=True)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    t = _timed([s_kv, s_w], step, args.steps, dev)
    wall = time.perf_counter() - t0
    kv_bytes = n * sh.composite_bytes
    per = t / args.steps
    value = (kv_bytes + ws.nbytes) / per / 1e9
    peaks = host_link_peaks(dev)
    line = {"impl": args.impl, "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3,
            "switch_ms": per * 1e3, "higher_is_better": True, "dtype": "u8",
            "config": {"workload": "cfg4 switch overlap: swap-in of 2048 Llama-2-7B-shaped "
                                   f"blocks ({kv_bytes} B) concurrent with a Qwen1.5-14B TP-2 "
                                   f"bf16 weight shard ({ws.nbytes} B) uploaded on a second "
                                   "stream",
                       "weights": "64 MiB chunks, kvx_upload_chunked" if ref is None else
                                  "one copy per weight tensor (quick_loader.py:413)"},
            "roofline": {"bound": "host_link", "achieved": value, "peak": peaks["h2d_gbs"],
                         "unit": "GB/s", "frac": value / peaks["h2d_gbs"],
                         "peak_source": "measured live: 2 GiB page-locked H2D copy in 256 MiB "
                                        "pieces"},
            "e2e": {"value": (kv_bytes + ws.nbytes) * args.steps / wall / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": kv_bytes + ws.nbytes, "d2h_bytes_per_step": 0}}
    return line


def run_config5(args):
    """Fragmented swap-out: Qwen1.5-MoE shape (24 layers x K/V, 64 KiB pages),
    16384 entries, half in contiguous device runs of 1..32 blocks, half
    isolated; host slots sequential.  One call per step; per-call latency."""
    import torch

    from aegaeon_b200 import ops, swapper, workloads

    dist_ = Dist.init(use_pg=args.impl == "kvx")
    if args.impl == "reference" and dist_.rank != 0:
        return None
    dev = torch.device("cuda", dist_.local_rank)
    sh = workloads.CFG5
    n = 16384
    avail = int([l for l in open("/proc/meminfo") if l.startswith("MemAvailable")][0].split()[1]) * 1024
    fit = int(0.45 * avail / max(1, dist_.world if args.impl == "kvx" else 1) / sh.composite_bytes)
    if fit < n:
        n = max(1024, fit // 1024 * 1024)
    ids, slots = workloads.fragmented_mapping(n, sh.num_blocks, seed=dist_.rank)
    gen = torch.Generator(device=dev).manual_seed(dist_.rank)
    ref = _ref_module() if args.impl == "reference" else None
    s = torch.cuda.Stream(dev)
    if ref is None:
        pages = []
        for _ in range(sh.num_segments):
            t = torch.empty(sh.num_blocks * sh.page_bytes, dtype=torch.uint8, device=dev)
            workloads.fill_segment(t, sh, gen)
            pages.append(t)
        segs, comp = swapper.make_segments([((f"l{i}",), sh.num_blocks * sh.page_bytes)
                                            for i in range(sh.num_segments)], sh.num_blocks)
        pool = torch.empty(n * comp, dtype=torch.uint8).pin_memory()
        sw = swapper.KVSwapper(dev.index, segs, pages, [frozenset({0})] * sh.num_segments, [1],
                               kv_swap=pool)

        def step(_k):
            sw.swap_blocks([0], ids, slots, [0] * n, [0] * n, [1] * n, [None], False,
                           mode=args.mode, stream=s)
    else:
        shape = (sh.num_blocks, sh.block_size, sh.kv_heads, sh.head_dim)
        caches = [torch.empty(shape, dtype=sh.dtype, device=dev).normal_(generator=gen)
                  for _ in range(sh.num_segments)]
        hosts = [torch.empty((n,) + shape[1:], dtype=sh.dtype).pin_memory() for _ in caches]

        def step(_k):
            with torch.cuda.stream(s):
                for c, h in zip(caches, hosts):
                    ref.swap(ids, slots, False, c, h)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    dist_.barrier()
    lat = []
    t0 = time.perf_counter()
    for k in range(args.steps):
        lat.append(_timed([s], step, 1, dev))
    wall = time.perf_counter() - t0
    t = dist_.max(sum(lat))
    nbytes = n * sh.composite_bytes
    world = dist_.world if ref is None else 1
    value = nbytes * args.steps * world / t / 1e9
    line = None
    if dist_.rank == 0:
        line = {"impl": args.impl, "metric": METRIC, "value": value, "unit": "GB/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": t / args.steps * 1e3, "call_latency_ms": sorted(x * 1e3 for x in lat),
                "higher_is_better": True, "dtype": "u8", "scaling": "weak",
                "config": {"workload": f"cfg5 Qwen1.5-MoE-A2.7B fragmented swap-out: 24 layers x "
                                       f"K/V 64 KiB pages, {n} entries (half in contiguous "
                                       "device runs of 1..32 blocks, half isolated), host "
                                       "slots sequential; one call per step",
                           "entries": n,
                           "api": "KVSwapper.swap_blocks -> kvx_swap_blocks" if ref is None
                           else "aegaeon.ops.swap (reference op), 48 calls per step"},
                "e2e": {"value": nbytes * args.steps * world / wall / 1e9, "unit": "GB/s",
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": nbytes * world}}
    dist_.finish()
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
    if args.config != 2:
        rank = int(os.environ.get("RANK", "0"))
        if args.config in (1, 4, 7) and rank != 0:
            return
        if args.config == 3:
            if args.impl != "reference":
                emit({"impl": "kvx", "note": "config 3 (migration) is measured by the default "
                      "run at N >= 2 (its 'migration' object)"})
                return
            if rank == 0:
                emit(run_config3_reference(args))
            return
        if args.config == 6:
            if rank == 0:
                emit(run_config6(args))
            return
        fn = {1: run_config1, 4: run_config4, 5: run_config5, 7: run_config7}[args.config]
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
