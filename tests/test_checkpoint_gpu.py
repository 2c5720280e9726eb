"""Weights in and out of a model, the reference's checkpoint layout, and the
reference's sampling loop run on the device.

* bonsai_dit_weight / bonsai_dit_set_weight round-trip every kind of tensor
  (plain B1_0, SwiGLU-interleaved B1_0, stacked per-block modulation views,
  f32).
* bonsai_dit_load_safetensors reads a file written here in the layout the
  reference's loader expects (src/diffuser.cpp:88-186: names, U8 packed
  B1_0 [out][in/32*6], F32 [out][in], separate q/k/v) and gives a model the
  same weights -- and the same prediction -- as the model the file was
  written from.
* bonsai_dit_sample equals the reference's loop (src/diffuser.cpp:251-294)
  driven from the host: forward, then lat += dt * pred in f32.
"""
import struct

import numpy as np
import pytest

import bonsai_b200 as bb
from st_writer import write_safetensors

pytestmark = pytest.mark.gpu

GH = GW = 8
TXT = 32


def _klein(seed, depth=1, single=1):
    return bb.Dit(bb.PRESET_KLEIN4B, GH * GW, TXT, GH, GW, depth=depth, depth_single=single, seed=seed)


def reference_checkpoint(m):
    """The model's weights under the reference's tensor names and shapes."""
    H = 3072
    out = {}

    def b1(name, rows):
        return m.weight(name).reshape(rows, -1)

    def f32(name, shape):
        return m.weight_f32(name).reshape(shape)

    out["x_embedder.weight"] = f32("img_in.w", (H, m.in_ch))
    out["context_embedder.weight"] = f32("txt_in.w", (H, m.ctx_dim))
    out["time_guidance_embed.timestep_embedder.linear_1.weight"] = f32("time.w1", (H, 256))
    out["time_guidance_embed.timestep_embedder.linear_2.weight"] = f32("time.w2", (H, H))
    out["double_stream_modulation_img.linear.weight"] = f32("mod_img.w", (6 * H, H))
    out["double_stream_modulation_txt.linear.weight"] = f32("mod_txt.w", (6 * H, H))
    out["single_stream_modulation.linear.weight"] = f32("mod_single.w", (3 * H, H))
    out["norm_out.linear.weight"] = f32("norm_out.w", (2 * H, H))
    out["proj_out.weight"] = f32("proj_out.w", (m.in_ch, H))
    for d in range(m.depth):
        o, r = f"double.{d}.", f"transformer_blocks.{d}."
        for ours, names in (("img_qkv", ("attn.to_q", "attn.to_k", "attn.to_v")),
                            ("txt_qkv", ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"))):
            w = b1(o + ours, 3 * H)
            for i, n in enumerate(names):
                out[r + n + ".weight"] = w[i * H:(i + 1) * H]
        out[r + "attn.to_out.0.weight"] = b1(o + "img_out", H)
        out[r + "attn.to_add_out.weight"] = b1(o + "txt_out", H)
        out[r + "attn.norm_q.weight"] = f32(o + "img_norm_q", (128,))
        out[r + "attn.norm_k.weight"] = f32(o + "img_norm_k", (128,))
        out[r + "attn.norm_added_q.weight"] = f32(o + "txt_norm_q", (128,))
        out[r + "attn.norm_added_k.weight"] = f32(o + "txt_norm_k", (128,))
        out[r + "ff.linear_in.weight"] = b1(o + "img_mlp_in", 2 * m.mlp)
        out[r + "ff.linear_out.weight"] = b1(o + "img_mlp_out", H)
        out[r + "ff_context.linear_in.weight"] = b1(o + "txt_mlp_in", 2 * m.mlp)
        out[r + "ff_context.linear_out.weight"] = b1(o + "txt_mlp_out", H)
    for s in range(m.depth_single):
        o, r = f"single.{s}.", f"single_transformer_blocks.{s}.attn."
        out[r + "to_qkv_mlp_proj.weight"] = b1(o + "proj", 3 * H + 2 * m.mlp)
        out[r + "to_out.weight"] = b1(o + "out", H)
        out[r + "norm_q.weight"] = f32(o + "norm_q", (128,))
        out[r + "norm_k.weight"] = f32(o + "norm_k", (128,))
    return out


def _inputs(m, seed=3):
    import torch
    rng = np.random.default_rng(seed)
    img = torch.from_numpy(rng.standard_normal((m.img, m.in_ch)).astype(np.float32)).cuda()
    txt = torch.from_numpy(rng.standard_normal((m.txt, m.ctx_dim)).astype(np.float32)).cuda()
    return img, txt


def test_weight_roundtrip_every_kind(gpu):
    rng = np.random.default_rng(0)
    m = _klein(seed=4)
    try:
        # plain B1_0, SwiGLU-interleaved B1_0 (double MLP-in, single proj), f32
        for name in ("double.0.img_out", "double.0.img_mlp_in", "single.0.proj", "img_in.w",
                     "single.0.norm_k"):
            cur = m.weight(name)
            new = rng.integers(0, 256, size=cur.shape, dtype=np.uint8)
            if name.endswith(("norm_k", ".w")):
                new = rng.standard_normal(cur.size // 4).astype(np.float32).view(np.uint8)
            m.set_weight(name, new)
            assert np.array_equal(m.weight(name), new), name
        with pytest.raises(bb.BonsaiError, match="takes"):
            m.set_weight("double.0.img_out", np.zeros(10, np.uint8))
        with pytest.raises(bb.BonsaiError, match="unknown tensor"):
            m.set_weight("double.9.img_out", np.zeros(10, np.uint8))
    finally:
        m.close()
    # stacked per-block modulation linears of the Flux.1 preset (views of one weight)
    f = bb.Dit(bb.PRESET_FLUX1, GH * GW, TXT, GH, GW, depth=2, depth_single=1, seed=4)
    try:
        names = ["double.0.img_mod", "double.1.txt_mod", "single.0.mod"]
        before = {n: f.weight(n) for n in names}
        new = rng.integers(0, 256, size=before["double.1.txt_mod"].shape, dtype=np.uint8)
        f.set_weight("double.1.txt_mod", new)
        assert np.array_equal(f.weight("double.1.txt_mod"), new)
        for n in ("double.0.img_mod", "single.0.mod"):  # neighbours untouched
            assert np.array_equal(f.weight(n), before[n]), n
    finally:
        f.close()


def test_load_reference_layout_checkpoint(gpu, tmp_path):
    import torch
    src = _klein(seed=5)
    dst = _klein(seed=9)
    try:
        ckpt = reference_checkpoint(src)
        path = tmp_path / "klein_1bit.safetensors"
        write_safetensors(path, ckpt)
        assert not np.array_equal(dst.weight("double.0.img_qkv"), src.weight("double.0.img_qkv"))
        dst.load_safetensors(path)
        for name in ("double.0.img_qkv", "double.0.txt_mlp_in", "single.0.proj", "mod_single.w",
                     "proj_out.w", "double.0.txt_norm_k"):
            assert np.array_equal(dst.weight(name), src.weight(name)), name
        img, txt = _inputs(src)
        a = torch.empty(src.img, src.in_ch, device="cuda")
        b = torch.empty_like(a)
        src.forward(img, txt, None, 700.0, a)
        dst.forward(img, txt, None, 700.0, b)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
        # a checkpoint with more blocks than the model loads its first blocks
        # (the reference's --max-depth / --max-single)
        small = _klein(seed=11, depth=1, single=1)
        try:
            big = _klein(seed=12, depth=2, single=2)
            try:
                path2 = tmp_path / "deeper.safetensors"
                write_safetensors(path2, reference_checkpoint(big))
                small.load_safetensors(path2)
                assert np.array_equal(small.weight("single.0.proj"), big.weight("single.0.proj"))
            finally:
                big.close()
        finally:
            small.close()
    finally:
        src.close()
        dst.close()


def test_load_errors(gpu, tmp_path):
    m = _klein(seed=6)
    try:
        ckpt = reference_checkpoint(m)
        missing = dict(ckpt)
        del missing["transformer_blocks.0.attn.to_k.weight"]
        p = tmp_path / "missing.safetensors"
        write_safetensors(p, missing)
        with pytest.raises(bb.BonsaiError, match="to_k.weight' not found"):
            m.load_safetensors(p)
        wrong = dict(ckpt)
        wrong["proj_out.weight"] = wrong["proj_out.weight"][:, :100]
        p = tmp_path / "wrong.safetensors"
        write_safetensors(p, wrong)
        with pytest.raises(bb.BonsaiError, match="proj_out.w"):
            m.load_safetensors(p)
        p = tmp_path / "garbage.safetensors"
        p.write_bytes(struct.pack("<Q", 12) + b"{not json}  ")
        with pytest.raises(bb.BonsaiError, match="safetensors"):
            m.load_safetensors(p)
        with pytest.raises(bb.BonsaiError, match="cannot open"):
            m.load_safetensors(tmp_path / "absent.safetensors")
    finally:
        m.close()
    f = bb.Dit(bb.PRESET_FLUX1, GH * GW, TXT, GH, GW, depth=1, depth_single=1, seed=4)
    try:
        with pytest.raises(bb.BonsaiError, match="klein4b preset only"):
            f.load_safetensors(tmp_path / "missing.safetensors")
    finally:
        f.close()


def test_sample_equals_host_euler_loop(gpu):
    import torch
    m = _klein(seed=7)
    try:
        img, txt = _inputs(m, seed=8)
        steps = 3
        lat = img.clone()
        stats = m.sample(lat, txt, None, steps)
        torch.cuda.synchronize()
        # the reference's loop from the host (src/diffuser.cpp:251-291), f32
        ref = img.cpu().numpy().copy()
        pred = torch.empty_like(img)
        ts = [np.float32(1.0) - np.float32(i) / np.float32(steps) for i in range(steps)]
        for s in range(steps):
            t = ts[s]
            dt = np.float32(t - ts[s + 1]) if s < steps - 1 else t
            m.forward(torch.from_numpy(ref).cuda(), txt, None, float(t * np.float32(1000.0)), pred)
            p = pred.cpu().numpy()
            assert stats[s, 0] == np.isnan(p).sum() and stats[s, 1] == np.isinf(p).sum()
            assert stats[s, 2] == p.min() and stats[s, 3] == p.max()
            assert abs(stats[s, 4] - p.mean(dtype=np.float64)) <= 1e-5 * (np.abs(p).mean() + 1e-30)
            ref = (ref + (np.float32(dt) * p).astype(np.float32)).astype(np.float32)
        assert np.array_equal(lat.cpu().numpy(), ref)
    finally:
        m.close()


def test_count_nonfinite(gpu):
    import torch
    x = torch.randn(100003, device="cuda")
    assert bb.count_nonfinite(x) == 0
    x[[5, 777, 100002]] = float("nan")
    x[[9, 50000]] = float("inf")
    x[12] = float("-inf")
    assert bb.count_nonfinite(x) == 6
    assert bb.count_nonfinite(x[:0]) == 0


def test_load_gguf_container(gpu, tmp_path):
    """The same checkpoint in the GGUF container (B1_0 = type 100, the
    reference converter's renaming) loads to the same weights."""
    from gguf_writer import write_gguf
    src = _klein(seed=15)
    dst = _klein(seed=16)
    try:
        ckpt = reference_checkpoint(src)
        gg = {}
        for name, arr in ckpt.items():
            if arr.dtype == np.uint8:
                gg[name] = (arr, arr.shape[1] // 6 * 32)
            else:
                gg[name] = arr
        path = tmp_path / "klein_1bit.gguf"
        write_gguf(path, gg)
        dst.load_safetensors(path)
        for name in ("double.0.img_qkv", "double.0.txt_mlp_out", "single.0.proj", "mod_img.w",
                     "time.w1", "single.0.norm_q"):
            assert np.array_equal(dst.weight(name), src.weight(name)), name
    finally:
        src.close()
        dst.close()


@pytest.fixture(scope="module")
def converter_files(tmp_path_factory):
    """The files the reference's converters write (byte-identical, checked
    against their SHA-256 in tests/golden/klein_ckpt.json)."""
    import json
    from pathlib import Path
    import klein_ckpt as kc
    gold = json.loads((Path(__file__).resolve().parent / "golden" / "klein_ckpt.json").read_text())
    d = tmp_path_factory.mktemp("converted")
    sd = kc.make_state_dict(gold["seed"])
    out = {"safetensors": d / "flux2_4b_1bit.safetensors", "gguf": d / "flux2_4b_1bit.gguf"}
    kc.write_packed_safetensors(sd, out["safetensors"])
    kc.write_gguf(sd, out["gguf"])
    del sd
    for kind, p in out.items():
        assert kc.sha256(p) == gold["files"][kind]["sha256"], f"{kind} differs from the converter's"
    return out


def test_load_reference_converter_outputs(gpu, converter_files):
    """Load the packed safetensors and the GGUF that the reference's
    converters write (convert_to_b1_0_packed.py, convert_to_b1_0.py) and run
    one forward of each; compare with the CPU oracle reading the same file's
    tensors through the safetensors library under the reference loader's
    names (src/diffuser.cpp:88-186), independently of the engine's loader."""
    import torch
    from oracle import pyoracle as O
    import klein_ckpt as kc
    rng = np.random.default_rng(12)
    outs = {}
    for kind in ("safetensors", "gguf"):
        m = _klein(seed=999)  # random weights, all replaced by the load
        try:
            m.load_safetensors(converter_files[kind])
            img, txt = _inputs(m, seed=12)
            out = torch.empty(m.img, m.in_ch, device="cuda")
            m.forward(img, txt, None, 500.0, out)
            outs[kind] = out.cpu().numpy()
            if kind == "safetensors":
                fw = kc.FileWeights(converter_files[kind], m)
                ref = O.dit_forward(fw, img.cpu().numpy(), txt.cpu().numpy(), None, 500.0)
        finally:
            m.close()
    assert bb.device_error() == 0
    np.testing.assert_array_equal(outs["gguf"], outs["safetensors"])
    g, r = outs["safetensors"].astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    cos = float(g @ r / (np.linalg.norm(g) * np.linalg.norm(r)))
    rel = float(np.abs(g - r).max() / np.sqrt(np.mean(r ** 2)))
    assert cos >= 0.9999 and rel <= 1e-2, (cos, rel)
