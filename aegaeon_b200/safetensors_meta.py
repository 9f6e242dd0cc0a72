"""Safetensors header metadata, read natively.

``read_safetensors_meta_as_json(file_path)`` has the name, argument, result
and errors of the reference's Rust extension function
(quick_model_loader/rsrc/lib.rs:45-51, used by
quick_model_loader/meta.py:207): a pretty JSON string with ``file_path``,
``size``, ``offset`` and ``tensor_info_map`` (name -> ``dtype``, ``shape``,
``data_offsets``).  An unreadable file raises ``OSError`` (``FileNotFoundError``
when it does not exist); an invalid header raises ``BufferError`` ("Fail to
read the metadata from the given buffer"), as the reference does.
"""

from __future__ import annotations

import ctypes
import errno
import os

from . import _lib


def read_safetensors_meta_as_json(file_path: str) -> str:
    lib = _lib.lib()
    path = os.fsencode(file_path)
    n = ctypes.c_uint64(0)
    rc = lib.kvx_safetensors_meta_json(path, None, 0, ctypes.byref(n))
    if rc == _lib.KVX_ERR_IO:
        msg = lib.kvx_last_error().decode(errors="replace")
        if not os.path.exists(file_path):
            raise FileNotFoundError(errno.ENOENT, msg, file_path)
        raise OSError(msg)
    if rc == _lib.KVX_ERR_FORMAT:
        raise BufferError("Fail to read the metadata from the given buffer")
    _lib.check(rc)
    buf = ctypes.create_string_buffer(n.value + 1)
    _lib.check(lib.kvx_safetensors_meta_json(path, buf, n.value + 1, ctypes.byref(n)))
    return buf.value.decode("utf-8")
