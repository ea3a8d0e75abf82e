"""Safetensors validation of the native loader (yue2_checkpoint_scan, no device needed):
the header checks of Weights::open (src/checkpoint.rs:315-396) with the reference's error
messages, single files and sharded indexes."""
import ctypes
import json
import os
import struct

import numpy as np
import pytest

from yue2_rs_b200 import _lib, checkpoint


def scan(path):
    n = ctypes.c_uint64()
    rc = _lib.lib().yue2_checkpoint_scan(os.fsencode(str(path)), ctypes.byref(n))
    return rc, (n.value if rc == 0 else _lib.last_error())


def raw_file(path, header_text, data=b""):
    blob = header_text.encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        f.write(data)


def test_single_file_and_metadata(tmp_path):
    named = {"a": ("BF16", (2, 3), np.arange(6, dtype=np.uint16)),
             "b": ("F32", (4,), np.ones(4, dtype=np.float32)),
             "c": ("F16", (1, 2), np.zeros(2, dtype=np.uint16))}
    checkpoint.write(str(tmp_path / "model.safetensors"), named, {"format": "pt"})
    assert scan(tmp_path) == (0, 3)


def test_sharded_index(tmp_path):
    checkpoint.write(str(tmp_path / "s1.safetensors"), {"a": ("BF16", (2,), np.zeros(2, np.uint16))})
    checkpoint.write(str(tmp_path / "s2.safetensors"), {"b": ("BF16", (3,), np.zeros(3, np.uint16)),
                                                        "c": ("F32", (1,), np.zeros(1, np.float32))})
    (tmp_path / "model.safetensors.index.json").write_text(
        json.dumps({"metadata": {}, "weight_map": {"a": "s1.safetensors", "b": "s2.safetensors",
                                                   "c": "s2.safetensors"}}))
    assert scan(tmp_path) == (0, 3)


@pytest.mark.parametrize("header,data,message", [
    ('{"x": {"dtype": "I32", "shape": [1], "data_offsets": [0, 4]}}', b"\0" * 4, "Unsupported dtype I32 for x"),
    ('{"x": {"dtype": "BF16", "shape": [3], "data_offsets": [0, 4]}}', b"\0" * 4, "Invalid tensor extent x"),
    ('{"x": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 8]}}', b"\0" * 4, "Invalid tensor extent x"),
    ('{"x": {"dtype": "BF16", "shape": [2], "data_offsets": [4, 0]}}', b"\0" * 8, "Invalid tensor extent x"),
    ('{"x": {"dtype": "BF16", "shape": [2], "data_offsets": [0]}}', b"\0" * 4, "Invalid tensor offsets"),
    ('{"x": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}, '
     '"y": {"dtype": "BF16", "shape": [2], "data_offsets": [2, 6]}}', b"\0" * 8, "Overlapping safetensors tensors"),
    ('{"x": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}, '
     '"x": {"dtype": "BF16", "shape": [2], "data_offsets": [4, 8]}}', b"\0" * 8, "Duplicate tensor x"),
    ('{"x": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]', b"\0" * 4, "Invalid safetensors header"),
])
def test_header_errors(tmp_path, header, data, message):
    raw_file(tmp_path / "model.safetensors", header, data)
    rc, msg = scan(tmp_path)
    assert rc == -1 and msg == message


def test_header_size_and_short_file(tmp_path):
    with open(tmp_path / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", 1 << 40) + b"{}")
    assert scan(tmp_path) == (-1, "Invalid safetensors header size")
    with open(tmp_path / "model.safetensors", "wb") as f:
        f.write(b"\1\2\3")
    assert scan(tmp_path) == (-1, "Short safetensors file")


def test_shard_paths_stay_in_the_directory(tmp_path):
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"a": "../x.safetensors"}}))
    assert scan(tmp_path) == (-1, "Invalid shard path")


def test_missing_file_is_an_error(tmp_path):
    rc, msg = scan(tmp_path)
    assert rc == -1 and msg.startswith("Cannot open checkpoint shard")
