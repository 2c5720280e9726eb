"""Minimal GGUF (version 3) writer for the tests, following the published
format: "GGUF", u32 version, u64 tensor count, u64 key/value count, typed
key/values, tensor infos (name, n_dims, dims innermost first, type, offset),
then the data at multiples of general.alignment.  B1_0 is tensor type 100
(6-byte blocks of 32 weights), the type the reference's convert_to_b1_0.py
writes; names are renamed as that script's map_tensor_name does."""
import struct

import numpy as np

KV_U32, KV_F32, KV_STRING, KV_ARRAY = 4, 6, 8, 9
GGML_F32, GGML_B1_0 = 0, 100


def gguf_name(name: str) -> str:
    return name.replace("single_transformer_blocks.", "blk.").replace("double_stream_modulation", "double_stream")


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key, value):
    if isinstance(value, str):
        return _str(key) + struct.pack("<I", KV_STRING) + _str(value)
    if isinstance(value, float):
        return _str(key) + struct.pack("<If", KV_F32, value)
    if isinstance(value, list):  # array of u32
        return _str(key) + struct.pack("<IIQ", KV_ARRAY, KV_U32, len(value)) + b"".join(
            struct.pack("<I", v) for v in value)
    return _str(key) + struct.pack("<II", KV_U32, value)


def write_gguf(path, tensors, alignment=32, extra_kv=None):
    """tensors: reference name -> float32 array (stored F32) or (packed uint8
    [out][in/32*6], in_dim) (stored B1_0)."""
    kv = {"general.architecture": "flux.diffusion", "flux.vision.hidden_size": 3072,
          "test.list": [1, 2, 3], "test.scale": 0.5}
    if alignment != 32:
        kv["general.alignment"] = alignment
    kv.update(extra_kv or {})
    infos, blobs, off = [], [], 0
    for name, t in tensors.items():
        if isinstance(t, tuple):
            packed, in_dim = t
            dims, typ, data = [in_dim, packed.shape[0]], GGML_B1_0, np.ascontiguousarray(packed).tobytes()
        else:
            arr = np.asarray(t, np.float32)
            dims, typ, data = list(arr.shape[::-1]) or [1], GGML_F32, arr.tobytes(order="C")
        infos.append(_str(gguf_name(name)) + struct.pack("<I", len(dims)) +
                     b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", typ, off))
        pad = -len(data) % alignment
        blobs.append(data + b"\0" * pad)
        off += len(data) + pad
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)) + b"".join(_kv(k, v) for k, v in kv.items())
    head += b"".join(infos)
    head += b"\0" * (-len(head) % alignment)
    with open(path, "wb") as f:
        f.write(head)
        for b in blobs:
            f.write(b)
