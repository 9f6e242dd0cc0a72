"""The C ABI library loads without a GPU and exports every declared symbol."""

import ctypes
import os
import re

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
    import pytest

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
