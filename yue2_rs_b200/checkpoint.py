"""Safetensors reading/writing for checkpoints under the reference's tensor names
(reference: src/checkpoint.rs:481-732 -- memory-mapped, F32/BF16/F16, sharded index)."""
import json
import os
import struct

import numpy as np

DTYPES = {"BF16": (0, np.uint16), "F32": (1, np.float32), "F16": (2, np.uint16)}


def _read_header(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        if n > 100 << 20:
            raise ValueError("Invalid safetensors header")
        header = json.loads(f.read(n))
    return header, 8 + n


def tensors(path):
    """Yields (name, dtype code, shape, numpy view) for every tensor of a file or a
    directory holding model.safetensors or model.safetensors.index.json."""
    files = []
    if os.path.isdir(path):
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                files = sorted(set(json.load(f)["weight_map"].values()))
            files = [os.path.join(path, x) for x in files]
        else:
            files = [os.path.join(path, "model.safetensors")]
    else:
        files = [path]
    for fp in files:
        header, base = _read_header(fp)
        mm = np.memmap(fp, dtype=np.uint8, mode="r")
        for name, info in header.items():
            if name == "__metadata__":
                continue
            code, np_t = DTYPES[info["dtype"]]
            b, e = info["data_offsets"]
            arr = mm[base + b: base + e].view(np_t)
            yield name, code, tuple(info["shape"]), arr


def write(path, named, metadata=None):
    """named: dict name -> (dtype string, shape, numpy array of the raw element type)."""
    header, offset, order = {}, 0, []
    for name, (dt, shape, arr) in named.items():
        nbytes = arr.nbytes
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
        order.append(arr)
    if metadata:
        header["__metadata__"] = metadata
    blob = json.dumps(header).encode()
    blob += b" " * ((8 - len(blob) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for arr in order:
            f.write(np.ascontiguousarray(arr).tobytes())
