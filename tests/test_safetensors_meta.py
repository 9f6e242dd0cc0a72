"""Safetensors header reading (the reference's Rust `read_safetensors_meta_as_json`).

Checked against (1) the reference's own test of the path
(quick_model_loader/tests/test_meta.py::test_read_meta, same tensors and the
same expected dtype / shape / data_offsets), (2) the CPU restatement of the
`safetensors` crate's header check (oracle/safetensors_oracle.py) on valid and
invalid files, and (3) the installed `safetensors` package, which must accept
exactly the files the reader accepts.
"""

import json
import os
import struct

import pytest
import torch

from aegaeon_b200.safetensors_meta import read_safetensors_meta_as_json
from oracle import safetensors_oracle as orc

st = pytest.importorskip("safetensors")
from safetensors.torch import save_file  # noqa: E402


def read(path):
    return json.loads(read_safetensors_meta_as_json(str(path)))


def test_read_meta_like_reference(tmp_path):
    """Mirrors quick_model_loader/tests/test_meta.py::test_read_meta."""
    path = tmp_path / "test.safetensors"
    save_file({"tensor0": torch.tensor([0, 1, 2, 3], dtype=torch.float16),
               "tensor1": torch.tensor([4, 5, 6], dtype=torch.float16),
               "tensor2": torch.tensor([7, 8, 9], dtype=torch.float16)}, str(path))
    meta = read(path)
    m = meta["tensor_info_map"]
    assert len(m) == 3
    assert [m[f"tensor{i}"]["dtype"] for i in range(3)] == ["F16"] * 3
    assert [m[f"tensor{i}"]["shape"] for i in range(3)] == [[4], [3], [3]]
    assert [tuple(m[f"tensor{i}"]["data_offsets"]) for i in range(3)] == [(0, 8), (8, 14), (14, 20)]
    assert meta["size"] == os.path.getsize(path)
    assert meta["offset"] == meta["size"] - 20
    assert meta["file_path"] == str(path)


DTYPES = [torch.float16, torch.bfloat16, torch.float32, torch.float64, torch.int8, torch.uint8,
          torch.int16, torch.int32, torch.int64, torch.bool]


@pytest.mark.parametrize("seed", range(6))
def test_random_files_match_oracle_and_safetensors(tmp_path, seed):
    g = torch.Generator().manual_seed(seed)
    tensors = {}
    for i in range(int(torch.randint(1, 12, (1,), generator=g))):
        dt = DTYPES[int(torch.randint(0, len(DTYPES), (1,), generator=g))]
        shape = [int(x) for x in torch.randint(0, 5, (int(torch.randint(0, 4, (1,), generator=g)),),
                                               generator=g)]
        tensors[f"layer.{i}.wé"] = torch.zeros(shape, dtype=dt)
    path = tmp_path / "m.safetensors"
    save_file(tensors, str(path), metadata={"format": "pt"})
    mine = read(path)
    assert mine == orc.read_meta(str(path))
    from safetensors import safe_open

    with safe_open(str(path), framework="pt") as f:
        assert sorted(f.keys()) == sorted(mine["tensor_info_map"])
        for k in f.keys():
            assert list(f.get_slice(k).get_shape()) == mine["tensor_info_map"][k]["shape"]


def craft(tmp_path, header, body: bytes, name="x.safetensors", raw_len=None):
    h = header if isinstance(header, bytes) else json.dumps(header).encode()
    p = tmp_path / name
    p.write_bytes(struct.pack("<Q", len(h) if raw_len is None else raw_len) + h + body)
    return p


INVALID = {
    "gap": ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
             "b": {"dtype": "F32", "shape": [1], "data_offsets": [12, 16]}}, b"\0" * 16),
    "size_mismatch": ({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8),
    "trailing_bytes": ({"a": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]}}, b"\0" * 6),
    "missing_bytes": ({"a": {"dtype": "F16", "shape": [4], "data_offsets": [0, 8]}}, b"\0" * 4),
    "unknown_dtype": ({"a": {"dtype": "F12", "shape": [1], "data_offsets": [0, 2]}}, b"\0" * 2),
    "negative_dim": ({"a": {"dtype": "F16", "shape": [-1], "data_offsets": [0, 2]}}, b"\0" * 2),
    "missing_field": ({"a": {"dtype": "F16", "shape": [1]}}, b"\0" * 2),
    "not_object": ([1, 2], b""),
    "bad_metadata": ({"__metadata__": {"k": 1}}, b""),
    "reversed_offsets": ({"a": {"dtype": "U8", "shape": [0], "data_offsets": [0, 0]},
                          "b": {"dtype": "U8", "shape": [2], "data_offsets": [2, 0]}}, b"\0\0"),
}


@pytest.mark.parametrize("case", sorted(INVALID))
def test_invalid_headers_are_rejected(tmp_path, case):
    header, body = INVALID[case]
    p = craft(tmp_path, header, body)
    with pytest.raises(BufferError, match="Fail to read the metadata"):
        read_safetensors_meta_as_json(str(p))
    with pytest.raises(orc.InvalidHeader):
        orc.read_meta(str(p))
    from safetensors import safe_open

    with pytest.raises(Exception):
        with safe_open(str(p), framework="pt"):
            pass


def test_framing_errors(tmp_path):
    short = tmp_path / "short.safetensors"
    short.write_bytes(b"\x01\x02")
    too_long = craft(tmp_path, {}, b"", name="long.safetensors", raw_len=1000)
    huge = craft(tmp_path, {}, b"", name="huge.safetensors", raw_len=200_000_000)
    bad_utf8 = craft(tmp_path, b'{"\xff": 1}', b"", name="utf.safetensors")
    bad_json = craft(tmp_path, b'{"a": ', b"", name="json.safetensors")
    for p in (short, too_long, huge, bad_utf8, bad_json):
        with pytest.raises(BufferError):
            read_safetensors_meta_as_json(str(p))
        with pytest.raises(orc.InvalidHeader):
            orc.read_meta(str(p))


def test_empty_and_metadata_only(tmp_path):
    p = craft(tmp_path, {"__metadata__": {"format": "pt"}}, b"")
    assert read(p)["tensor_info_map"] == {}
    assert read(p) == orc.read_meta(str(p))
    q = craft(tmp_path, b"{}      ", b"", name="pad.safetensors")  # space-padded header
    assert read(q) == orc.read_meta(str(q))


def test_missing_file(tmp_path):
    with pytest.raises(FileNotFoundError):
        read_safetensors_meta_as_json(str(tmp_path / "nope.safetensors"))
