"""Minimal .safetensors writer for the tests (8-byte little-endian header
length, JSON header {name: {dtype, shape, data_offsets}}, then the data)."""
import json
import struct

import numpy as np

_DTYPES = {np.dtype(np.uint8): "U8", np.dtype(np.float32): "F32", np.dtype(np.float16): "F16",
           np.dtype(np.float64): "F64", np.dtype(np.uint16): "U16"}


def write_safetensors(path, tensors, metadata=None, dtypes=None):
    """dtypes: optional {name: dtype string} overriding the numpy dtype's
    (e.g. "BF16" for bf16 bit patterns held in a uint16 array)."""
    header, blobs, off = {"__metadata__": metadata or {"format": "pt"}}, [], 0
    for name, arr in tensors.items():
        arr = np.asarray(arr)  # keeps 0-d shapes (ascontiguousarray would make them 1-d)
        dt = (dtypes or {}).get(name, None) or _DTYPES[arr.dtype]
        header[name] = {"dtype": dt, "shape": list(arr.shape),
                        "data_offsets": [off, off + arr.nbytes]}
        blobs.append(arr.tobytes(order="C"))
        off += arr.nbytes
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
