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


@pytest.mark.parametrize("alignment", [32, 64])
def test_gguf_index(tmp_path, alignment):
    """A GGUF file as convert_to_b1_0.py writes it (B1_0 = type 100, renamed
    tensors) is indexed under the reference's safetensors names, B1_0 as U8
    [out][in/32*6] and F32 with row-major shapes."""
    from gguf_writer import write_gguf
    rng = np.random.default_rng(1)
    packed = rng.integers(0, 256, (96, 64 // 32 * 6), dtype=np.uint8)
    tensors = {
        "single_transformer_blocks.0.attn.to_out.weight": (packed, 64),
        "double_stream_modulation_img.linear.weight": rng.standard_normal((18, 6)).astype(np.float32),
        "transformer_blocks.0.attn.norm_q.weight": rng.standard_normal(128).astype(np.float32),
        "x_embedder.weight": rng.standard_normal((32, 16)).astype(np.float32),
    }
    p = tmp_path / "m.gguf"
    write_gguf(p, tensors, alignment=alignment)
    got = {n: (d, s, b, e) for n, d, s, b, e in bb.safetensors_list(p)}
    assert set(got) == set(tensors)
    assert got["single_transformer_blocks.0.attn.to_out.weight"][:2] == ("U8", (96, 12))
    assert got["double_stream_modulation_img.linear.weight"][:2] == ("F32", (18, 6))
    assert got["transformer_blocks.0.attn.norm_q.weight"][:2] == ("F32", (128,))
    for n, (d, s, b, e) in got.items():
        assert b % alignment == 0
        assert e - b == int(np.prod(s)) * (1 if d == "U8" else 4)
    # the bytes at the reported offsets are the tensors' bytes
    raw = p.read_bytes()
    start = len(raw) - sum(-(-(e - b) // alignment) * alignment for _, _, b, e in got.values())
    b, e = got["x_embedder.weight"][2:]
    assert raw[start + b:start + e] == tensors["x_embedder.weight"].tobytes()


def test_gguf_errors(tmp_path):
    p = tmp_path / "v1.gguf"
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 1, 0, 0))
    with pytest.raises(bb.BonsaiError, match="version"):
        bb.safetensors_list(p)
    p = tmp_path / "trunc.gguf"
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + b"\x05")
    with pytest.raises(bb.BonsaiError, match="gguf"):
        bb.safetensors_list(p)
