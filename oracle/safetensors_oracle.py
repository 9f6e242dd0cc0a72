"""CPU restatement of the safetensors header check (test infrastructure only).

Restates, in Python, what the reference's Rust function does
(quick_model_loader/rsrc/lib.rs:19-51): map the file, call the `safetensors`
crate 0.4.3 `SafeTensors::read_metadata` (length prefix, UTF-8 JSON header,
Metadata::validate: offsets tile the data from 0 without gaps, each size equals
prod(shape) * dtype size, nothing after the last tensor) and return file_path,
size, offset = 8 + header length and the tensor map.  Only tests/ use it, as
the checker of aegaeon_b200.safetensors_meta.
"""

from __future__ import annotations

import json
import os

DTYPE_SIZES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E5M2": 1, "F8_E4M3": 1, "I16": 2, "U16": 2,
               "F16": 2, "BF16": 2, "I32": 4, "U32": 4, "F32": 4, "F64": 8, "I64": 8, "U64": 8}
MAX_HEADER = 100_000_000


class InvalidHeader(Exception):
    pass


def _uint(x) -> bool:
    return isinstance(x, int) and not isinstance(x, bool) and 0 <= x < 2**64


def read_meta(path: str) -> dict:
    data = open(path, "rb").read()
    size = len(data)
    if size < 8:
        raise InvalidHeader("header too small")
    n = int.from_bytes(data[:8], "little")
    if n > MAX_HEADER:
        raise InvalidHeader("header too large")
    if 8 + n > size:
        raise InvalidHeader("invalid header length")
    try:
        text = data[8:8 + n].decode("utf-8")
        header = json.loads(text)
    except (UnicodeDecodeError, ValueError) as e:
        raise InvalidHeader(str(e))
    if not isinstance(header, dict):
        raise InvalidHeader("not an object")
    tensors = {}
    for name, info in header.items():
        if name == "__metadata__":
            if info is None:
                continue
            if not isinstance(info, dict) or not all(isinstance(v, str) for v in info.values()):
                raise InvalidHeader("bad __metadata__")
            continue
        if not isinstance(info, dict) or not {"dtype", "shape", "data_offsets"} <= set(info):
            raise InvalidHeader("bad tensor entry")
        dt, shape, offs = info["dtype"], info["shape"], info["data_offsets"]
        if not isinstance(dt, str) or dt not in DTYPE_SIZES:
            raise InvalidHeader("dtype")
        if not isinstance(shape, list) or not all(_uint(d) for d in shape):
            raise InvalidHeader("shape")
        if not isinstance(offs, list) or len(offs) != 2 or not all(_uint(o) for o in offs):
            raise InvalidHeader("data_offsets")
        tensors[name] = {"dtype": dt, "shape": shape, "data_offsets": offs}
    start = 0
    for name, t in sorted(tensors.items(), key=lambda kv: tuple(kv[1]["data_offsets"])):
        b, e = t["data_offsets"]
        if b != start or e < b:
            raise InvalidHeader(f"invalid offset {name}")
        start = e
        nel = 1
        for d in t["shape"]:
            nel *= d
        if nel * DTYPE_SIZES[t["dtype"]] >= 2**64:
            raise InvalidHeader("overflow")
        if nel * DTYPE_SIZES[t["dtype"]] != e - b:
            raise InvalidHeader(f"tensor info invalid {name}")
    if start + 8 + n != size:
        raise InvalidHeader("metadata incomplete buffer")
    return {"file_path": path, "size": size, "offset": 8 + n, "tensor_info_map": tensors}
