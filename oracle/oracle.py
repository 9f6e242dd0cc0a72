"""Python face of the CPU oracle (liboracle.so, built from kvx_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py, as the checker of the CUDA path.  Buffers are
numpy uint8 arrays (host memory); the functions mutate the destination array
in place and raise on the status codes the oracle returns.

Restated reference code: ops/swap.cu:25-60 (``swap``),
aegaeon/worker.py:2270-2329 (``swap_blocks``), aegaeon/cache_transfer.py:
113-165 (``byte_extent``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

_lib = None
_STATUS = {1: ValueError, 3: ValueError, 4: ValueError, 5: IndexError}


def build() -> str:
    src = os.path.join(HERE, "kvx_oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        _lib = ctypes.CDLL(LIB)
        i64p = ctypes.POINTER(ctypes.c_int64)
        u64p = ctypes.POINTER(ctypes.c_uint64)
        vp = ctypes.c_void_p
        _lib.oracle_swap.argtypes = [i64p, i64p, ctypes.c_int64, ctypes.c_int, vp,
                                     ctypes.c_uint64, ctypes.c_uint64, vp, ctypes.c_uint64]
        _lib.oracle_byte_extent.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, u64p, u64p]
        _lib.oracle_swap_blocks.argtypes = [
            ctypes.c_int64, ctypes.POINTER(vp), u64p, u64p, u64p, u64p, ctypes.c_int64, i64p, vp,
            ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, i64p, i64p, i64p,
            i64p, i64p, ctypes.c_int, u64p]
        _lib.oracle_copy_blocks_mt.argtypes = [i64p, i64p, ctypes.c_int64, vp, vp,
                                               ctypes.c_uint64, ctypes.c_int]
    return _lib


def _check(rc: int) -> None:
    if rc:
        raise _STATUS.get(rc, RuntimeError)(f"oracle status {rc}")


def _i64(values) -> ctypes.Array:
    a = np.ascontiguousarray(np.asarray(values, dtype=np.int64))
    return (ctypes.c_int64 * max(a.size, 1)).from_buffer_copy(a if a.size else np.zeros(1, np.int64))


def _ptr(a: np.ndarray) -> int:
    assert a.dtype == np.uint8 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def byte_extent(page: int, ratio: int, first: int, count: int) -> tuple[int, int]:
    off = ctypes.c_uint64()
    ln = ctypes.c_uint64()
    _check(lib().oracle_byte_extent(page, ratio, first, count, ctypes.byref(off),
                                    ctypes.byref(ln)))
    return off.value, ln.value


def swap(source_ids, target_ids, is_swap_in: bool, cache: np.ndarray, swap_buf: np.ndarray,
         block_bytes: int) -> None:
    """ops/swap.cu:25-60 on host byte arrays."""
    n = len(source_ids)
    assert len(target_ids) == n
    _check(lib().oracle_swap(_i64(source_ids), _i64(target_ids), n, int(bool(is_swap_in)),
                             _ptr(cache), cache.size, block_bytes, _ptr(swap_buf), swap_buf.size))


def swap_blocks(seg_pages: list, page_bytes, cpu_offsets, owner_masks, group_ratios,
                pool: np.ndarray, row_bytes: int, row_offset: int, source_ids, target_ids,
                group_ids, first_blocks, valid_blocks, is_swap_in: bool) -> int:
    """worker.py:2270-2329 on host byte arrays; returns copied bytes.
    seg_pages[s] is a uint8 array of num_blocks[s] * page_bytes[s] bytes."""
    ns = len(seg_pages)
    P = (ctypes.c_void_p * max(ns, 1))(*[_ptr(p) for p in seg_pages])
    U = lambda v: (ctypes.c_uint64 * max(len(v), 1))(*v)  # noqa: E731
    nb = [p.size // pb for p, pb in zip(seg_pages, page_bytes)]
    copied = ctypes.c_uint64()
    n = len(source_ids)
    _check(lib().oracle_swap_blocks(
        ns, P, U(page_bytes), U(nb), U(cpu_offsets), U(owner_masks), len(group_ratios),
        _i64(group_ratios), _ptr(pool), pool.size // row_bytes, row_bytes, row_offset, n,
        _i64(source_ids), _i64(target_ids), _i64(group_ids), _i64(first_blocks),
        _i64(valid_blocks), int(bool(is_swap_in)), ctypes.byref(copied)))
    return copied.value


def copy_blocks_mt(src_ids, dst_ids, from_buf: np.ndarray, to_buf: np.ndarray,
                   block_bytes: int, threads: int) -> None:
    """to[dst[i]] = from[src[i]] over `threads` host threads (CPU baseline)."""
    n = len(src_ids)
    _check(lib().oracle_copy_blocks_mt(_i64(src_ids), _i64(dst_ids), n, _ptr(from_buf),
                                       _ptr(to_buf), block_bytes, threads))


def swap_numpy(source_ids, target_ids, is_swap_in: bool, cache: np.ndarray,
               swap_buf: np.ndarray, block_bytes: int) -> None:
    """Independent numpy restatement of ops/swap.cu:36-58 (in-order copies)."""
    c = cache.reshape(-1)[: cache.size // block_bytes * block_bytes].reshape(-1, block_bytes)
    s = swap_buf.reshape(-1)[: swap_buf.size // block_bytes * block_bytes].reshape(-1, block_bytes)
    for a, b in zip(source_ids, target_ids):
        if is_swap_in:
            c[b] = s[a]
        else:
            s[b] = c[a]
