"""The checkpoint files the engine's loader tests read are byte-for-byte the
files the reference's own converters write.

tests/golden/klein_ckpt.json holds the size and SHA-256 of what
convert_to_b1_0_packed.py and convert_to_b1_0.py (run unmodified by
tests/golden/make_checkpoint_golden.py) wrote from the seeded checkpoint of
tests/klein_ckpt.py.  Writing the same checkpoint with tests/klein_ckpt.py's
restatement of the two converters must give the same bytes; the GPU loader
tests then load exactly these files.  The files are also indexed by the
library's container reader (host code, no GPU): every tensor the reference's
loader requires (src/diffuser.cpp:88-186) is listed with the dtype and shape
it expects.
"""
import json
from pathlib import Path

import pytest

import klein_ckpt as kc

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "klein_ckpt.json").read_text())


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    d = tmp_path_factory.mktemp("klein")
    sd = kc.make_state_dict(GOLD["seed"])
    st, gg = d / "flux2_4b_1bit.safetensors", d / "flux2_4b_1bit.gguf"
    kc.write_packed_safetensors(sd, st)
    kc.write_gguf(sd, gg)
    return {"safetensors": st, "gguf": gg}


@pytest.mark.parametrize("kind", ["safetensors", "gguf"])
def test_written_file_is_the_reference_converters_output(files, kind):
    p = files[kind]
    want = GOLD["files"][kind]
    assert p.stat().st_size == want["bytes"]
    assert kc.sha256(p) == want["sha256"]


@pytest.mark.parametrize("kind", ["safetensors", "gguf"])
def test_container_index_lists_the_reference_loader_tensors(files, kind):
    import bonsai_b200 as bb
    idx = {name: (dt, shape) for name, dt, shape, _, _ in bb.safetensors_list(files[kind])}
    H = 3072
    assert idx["transformer_blocks.0.attn.to_q.weight"] == ("U8", (H, H // 32 * 6))
    assert idx["transformer_blocks.0.ff.linear_in.weight"] == ("U8", (2 * 9216, H // 32 * 6))
    assert idx["single_transformer_blocks.0.attn.to_out.weight"] == ("U8", (H, (H + 9216) // 32 * 6))
    assert idx["transformer_blocks.0.attn.norm_q.weight"] == ("F32", (128,))
    assert idx["context_embedder.weight"] == ("F32", (H, 7680))
    assert idx["double_stream_modulation_img.linear.weight"] == ("F32", (6 * H, H))
    assert idx["proj_out.weight"] == ("F32", (128, H))
