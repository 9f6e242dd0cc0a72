"""The C ABI library loads without a GPU and exports every declared symbol."""

import ctypes
import os
import re

import pytest
from conftest import ROOT


def declared_functions():
    text = open(os.path.join(ROOT, "include", "kvx.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kvx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("kvx_swap", "kvx_swap_blocks", "kvx_migrate_blocks", "kvx_layout_create",
                     "kvx_ipc_export", "kvx_ipc_import", "kvx_upload_chunked"):
        assert required in names


def test_library_exports_every_declared_symbol(kvx):
    for name in declared_functions():
        assert hasattr(kvx, name), name


def test_binding_covers_header():
    from aegaeon_b200 import _lib

    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_status_strings(kvx):
    assert kvx.kvx_status_string(0) == b"ok"
    assert kvx.kvx_status_string(5) == b"block id out of range"
    assert kvx.kvx_version() >= 10000


def test_extent_call_without_gpu(kvx):
    off, ln = ctypes.c_uint64(), ctypes.c_uint64()
    assert kvx.kvx_byte_extent(65536, 4, 1, 2, ctypes.byref(off), ctypes.byref(ln)) == 0
    assert (off.value, ln.value) == (16384, 32768)
    assert kvx.kvx_byte_extent(65536, 4, 3, 2, ctypes.byref(off), ctypes.byref(ln)) == 4
    assert b"exceeds page size 4" in kvx.kvx_last_error()


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from aegaeon_b200 import _lib

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="missing"):
        _lib.lib()


def test_id_arrays_from_any_sequence():
    import numpy as np
    import torch

    from aegaeon_b200 import _lib

    for v in ([3, 1, 2], (3, 1, 2), np.array([3, 1, 2], dtype=np.int32), torch.tensor([3, 1, 2])):
        a = _lib.i64_array(v)
        assert list(a) == [3, 1, 2]
    assert len(_lib.i64_array([])) == 0
    assert len(_lib.i64_array(np.zeros(0, dtype=np.int64))) == 0


def test_id_arrays_reject_non_int64_ids():
    """An id that does not fit int64 or is not an integer raises instead of
    wrapping around to some other block."""
    import numpy as np

    from aegaeon_b200 import _lib

    assert list(_lib.i64_array(range(2, 12, 3))) == [2, 5, 8, 11]
    assert list(_lib.i64_array([np.int64(7), 2**63 - 1, -1])) == [7, 2**63 - 1, -1]
    for bad in ([2**63], [0, -2**63 - 1], list(range(20)) + [2**64]):
        with pytest.raises(OverflowError):
            _lib.i64_array(bad)
    for bad in ([1.5], ["3"], [None]):
        with pytest.raises(TypeError):
            _lib.i64_array(bad)


def test_call_shim_converts_ids_and_returns_status():
    """The compiled call shim binds to libkvx.so without a GPU, takes ids as
    lists, tuples or int64 buffers, raises on bad ids before calling the
    library, and returns the library's status (here from its validation,
    which runs before any CUDA call)."""
    import numpy as np

    from aegaeon_b200 import _lib

    sh = _lib.shim()
    assert sh is _lib.shim()
    one_block = (0x10000, 4096, 4096, 0x200000, 4096, 0, 0)  # 1 cache block, 1 slot
    assert sh.swap([], (), False, *one_block) == 0
    for ids in ([3], (3,), np.array([3], dtype=np.int64), _lib.i64_array([3]),
                np.array([3], dtype=np.int32)):
        status = sh.swap(ids, [0], False, *one_block)
        assert status == _lib.KVX_ERR_BLOCK_ID
        with pytest.raises(IndexError, match="block id"):
            _lib.check(status)
    with pytest.raises(ValueError, match="1 ids but target_block_ids has 2"):
        sh.swap([0], [0, 0], False, *one_block)
    with pytest.raises(TypeError):
        sh.swap([0.5], [0], False, *one_block)
    with pytest.raises(OverflowError):
        sh.swap([2**63], [0], False, *one_block)
    big = list(range(100))  # beyond the shim's on-stack id buffer
    assert sh.swap(big, big, True, *one_block) == _lib.KVX_ERR_BLOCK_ID


def test_call_shim_swap_blocks_checks_lengths():
    from aegaeon_b200 import _lib, swapper

    page, blocks = 4096, 8
    lay = swapper._Layout(0, [0x7f0000000000], [page], [blocks], [0], [1], [1],
                          0x100000000, 4 * page, page, 0)
    sh = _lib.shim()
    with pytest.raises(ValueError, match="equal lengths"):
        sh.swap_blocks(lay.handle, [0], [0], [0], [0], [], False, 0, 0)
    status, copied, extents = sh.swap_blocks(lay.handle, [9], [0], [0], [0], [1], False, 0, 0)
    assert status == _lib.KVX_ERR_BLOCK_ID and copied == 0 and extents == 0
    # migration between two layouts: same checks, validation before any CUDA call
    with pytest.raises(ValueError, match="equal lengths"):
        sh.migrate_blocks(lay.handle, lay.handle, [0, 1], [2], [0], [0], [1], 0, 0)
    with pytest.raises(ValueError, match="null layout"):
        sh.migrate_blocks(lay.handle, 0, [0], [2], [0], [0], [1], 0, 0)
    status, _, _ = sh.migrate_blocks(lay.handle, lay.handle, [0], [blocks], [0], [0], [1], 0, 0)
    assert status == _lib.KVX_ERR_BLOCK_ID
    lay.close()
