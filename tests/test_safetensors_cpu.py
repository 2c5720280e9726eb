"""The .safetensors index reader of the library (host only, no GPU):
the container of the reference's packed checkpoints (src/safetensors.h)."""
import struct

import numpy as np
import pytest

import bonsai_b200 as bb
from st_writer import write_safetensors


def test_index_roundtrip(tmp_path):
    rng = np.random.default_rng(0)
    tensors = {
        "transformer_blocks.0.attn.to_q.weight": rng.integers(0, 256, (64, 12), dtype=np.uint8),
        "x_embedder.weight": rng.standard_normal((32, 16)).astype(np.float32),
        "norm.weight": np.ones(128, np.float16),
        "scalar": np.zeros((), np.float32),
    }
    p = tmp_path / "t.safetensors"
    write_safetensors(p, tensors, metadata={"format": "pt", "note": "nested {braces} [and] \"quotes\""})
    got = {name: (dtype, shape, b, e) for name, dtype, shape, b, e in bb.safetensors_list(p)}
    assert set(got) == set(tensors)
    off = 0
    for name, arr in tensors.items():  # the writer lays tensors out in insertion order
        dtype, shape, b, e = got[name]
        assert dtype == {np.uint8: "U8", np.float32: "F32", np.float16: "F16"}[arr.dtype.type]
        assert shape == arr.shape
        assert (b, e) == (off, off + arr.nbytes)
        off += arr.nbytes
    assert [n for n, *_ in bb.safetensors_list(p)] == sorted(tensors)


def test_empty_index(tmp_path):
    p = tmp_path / "empty.safetensors"
    p.write_bytes(struct.pack("<Q", 8) + b"{}      ")
    assert bb.safetensors_list(p) == []


@pytest.mark.parametrize("payload,what", [
    (struct.pack("<Q", 12) + b"{not json}  ", "header"),
    (struct.pack("<Q", 1000) + b"{}", "header length"),
    (b"\x01\x02", "shorter"),
    (struct.pack("<Q", 64) + b'{"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 1600]}}'.ljust(64),
     "outside the file"),
    (struct.pack("<Q", 48) + b'{"a": {"dtype": "F32", "shape": [4]}}'.ljust(48), "lacks"),
    (struct.pack("<Q", 64) + b'{"a": {"dtype": "F32", "data_offsets": [0, 16, 32]}}'.ljust(64), "two entries"),
])
def test_malformed_files_are_errors(tmp_path, payload, what):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(payload)
    with pytest.raises(bb.BonsaiError, match=what):
        bb.safetensors_list(p)


def test_missing_file(tmp_path):
    with pytest.raises(bb.BonsaiError, match="cannot open"):
        bb.safetensors_list(tmp_path / "absent.safetensors")
