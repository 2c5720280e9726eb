"""A seeded Flux.2-klein checkpoint in the layout the reference's converters
read (diffusers names, f32, PyTorch [out][in]), and the two packed files
those converters write from it.

make_state_dict(seed): every tensor the reference's loader reads
(src/diffuser.cpp:88-186) for one double and one single block, plus the
edges.  The block linears that get quantized hold values k * 2^-14 with small
integers k: every partial sum of a 32-weight group is exact in f32, so the
converter's scale mean(|w|) is the same whatever order numpy sums in, and the
files below are byte-for-byte reproducible on any host.  Some weights are
exactly 0 (the converter's sign rule is w >= 0 -> bit 1).

write_packed_safetensors / write_gguf restate, step by step, what
convert_to_b1_0_packed.py (quantize_b1_0 :21-43, should_quantize :46-54, the
tensor loop + save_file :57-112) and convert_to_b1_0.py (quantize_b1_0
:15-43, map_tensor_name :45-50, the GGUFWriter calls :52-97) do with a
source checkpoint, in the converters' tensor order (sorted names, the order
safetensors' safe_open lists them).  tests/golden/klein_ckpt.json holds the
SHA-256 of the files the reference's converters themselves wrote from the
same state dict (tests/golden/make_checkpoint_golden.py): a file written here
with that hash is the reference converter's output.
"""
from __future__ import annotations

import hashlib

import numpy as np

H, HD, MLP, IN_CH, CTX = 3072, 128, 9216, 128, 7680
BLOCK = 32


def make_state_dict(seed: int = 2024, depth: int = 1, single: int = 1) -> dict:
    rng = np.random.default_rng(seed)

    def quantizable(rows, cols):
        k = rng.integers(0, 641, size=(rows, cols), dtype=np.int32)
        s = rng.integers(0, 2, size=(rows, cols), dtype=np.int8) * 2 - 1
        return (k * s).astype(np.float32) * np.float32(2.0 ** -14)

    def f32(*shape, std=0.02):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    def norm():
        return (1.0 + 0.1 * rng.standard_normal(HD, dtype=np.float32)).astype(np.float32)

    sd = {
        "x_embedder.weight": f32(H, IN_CH),
        "context_embedder.weight": f32(H, CTX),
        "time_guidance_embed.timestep_embedder.linear_1.weight": f32(H, 256),
        "time_guidance_embed.timestep_embedder.linear_2.weight": f32(H, H),
        "double_stream_modulation_img.linear.weight": f32(6 * H, H),
        "double_stream_modulation_txt.linear.weight": f32(6 * H, H),
        "single_stream_modulation.linear.weight": f32(3 * H, H),
        "norm_out.linear.weight": f32(2 * H, H),
        "proj_out.weight": f32(IN_CH, H),
    }
    for d in range(depth):
        r = f"transformer_blocks.{d}."
        for n in ("attn.to_q", "attn.to_k", "attn.to_v", "attn.to_out.0", "attn.add_q_proj",
                  "attn.add_k_proj", "attn.add_v_proj", "attn.to_add_out"):
            sd[r + n + ".weight"] = quantizable(H, H)
        for n in ("attn.norm_q", "attn.norm_k", "attn.norm_added_q", "attn.norm_added_k"):
            sd[r + n + ".weight"] = norm()
        for n in ("ff", "ff_context"):
            sd[r + n + ".linear_in.weight"] = quantizable(2 * MLP, H)
            sd[r + n + ".linear_out.weight"] = quantizable(H, MLP)
    for s in range(single):
        r = f"single_transformer_blocks.{s}.attn."
        sd[r + "to_qkv_mlp_proj.weight"] = quantizable(3 * H + 2 * MLP, H)
        sd[r + "to_out.weight"] = quantizable(H, H + MLP)
        sd[r + "norm_q.weight"] = norm()
        sd[r + "norm_k.weight"] = norm()
    return sd


def quantize_b1_0(w: np.ndarray) -> np.ndarray:
    """[out][in] f32 -> [out][in/32*6] u8: per 32-weight group an f16
    mean(|w|) (little-endian) then 32 sign bits (w >= 0 -> 1, bit i = input
    32*blk + i, little-endian) -- convert_to_b1_0_packed.py:21-43."""
    out_dim, in_dim = w.shape
    g = w.reshape(out_dim, in_dim // BLOCK, BLOCK)
    scale = np.mean(np.abs(g), axis=-1).astype(np.float16)
    bits = np.packbits((g >= 0).astype(np.uint8), axis=-1, bitorder="little")
    raw = np.zeros((out_dim, in_dim // BLOCK, 6), np.uint8)
    raw[:, :, 0:2] = scale.view(np.uint8).reshape(out_dim, in_dim // BLOCK, 2)
    raw[:, :, 2:6] = bits
    return raw.reshape(out_dim, -1)


def should_quantize(name: str, shape) -> bool:
    """convert_to_b1_0_packed.py:46-54: 2-D tensors under the block prefixes."""
    return name.startswith(("transformer_blocks.", "single_transformer_blocks.")) and len(shape) != 1


def write_packed_safetensors(sd: dict, path) -> None:
    """The packed safetensors convert_to_b1_0_packed.py writes (U8 B1_0 for
    the block linears, F32 for everything else, one save_file call)."""
    from safetensors.numpy import save_file
    out = {}
    for name in sorted(sd):
        t = sd[name]
        out[name] = quantize_b1_0(t) if should_quantize(name, t.shape) else t.astype(np.float32)
    save_file(out, str(path))


def gguf_name(name: str) -> str:
    """convert_to_b1_0.py:45-50."""
    return name.replace("single_transformer_blocks.", "blk.").replace("double_stream_modulation",
                                                                      "double_stream")


def write_gguf(sd: dict, path) -> None:
    """The GGUF convert_to_b1_0.py writes: architecture "flux.diffusion", one
    u32 key, B1_0 as tensor type 100 with 6-byte blocks of 32 weights, F32 for
    1-D tensors, time-embedding tensors and the edge projections."""
    import gguf
    import gguf.quants
    from gguf import GGMLQuantizationType, GGUFWriter
    b1_0 = 100
    gguf.quants.GGML_QUANT_SIZES[b1_0] = (BLOCK, 6)
    w = GGUFWriter(str(path), "flux.diffusion")
    w.add_uint32("flux.vision.hidden_size", 3072)
    for name in sorted(sd):
        t = sd[name].astype(np.float32)
        g = gguf_name(name)
        if t.ndim == 1 or "time" in name:
            w.add_tensor(g, t, raw_dtype=GGMLQuantizationType.F32)
        elif name.startswith(("transformer_blocks.", "single_transformer_blocks.")):
            raw = quantize_b1_0(t).reshape(-1)
            w.add_tensor(g, raw, raw_shape=t.shape[:-1] + (t.shape[-1] // BLOCK * 6,),
                         raw_dtype=b1_0)
        else:
            w.add_tensor(g, t, raw_dtype=GGMLQuantizationType.F32)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def sha256(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


# The reference loader's names (src/diffuser.cpp:88-186) of every tensor the
# engine and the CPU oracle use, by the engine's tensor name.  B1_0 entries
# list the reference tensors whose rows are stacked (the engine fuses the
# q / k / v linears of a stream into one weight).
def engine_to_reference(depth: int = 1, single: int = 1) -> dict:
    m = {
        "img_in.w": ["x_embedder.weight"],
        "txt_in.w": ["context_embedder.weight"],
        "time.w1": ["time_guidance_embed.timestep_embedder.linear_1.weight"],
        "time.w2": ["time_guidance_embed.timestep_embedder.linear_2.weight"],
        "mod_img.w": ["double_stream_modulation_img.linear.weight"],
        "mod_txt.w": ["double_stream_modulation_txt.linear.weight"],
        "mod_single.w": ["single_stream_modulation.linear.weight"],
        "norm_out.w": ["norm_out.linear.weight"],
        "proj_out.w": ["proj_out.weight"],
    }
    for d in range(depth):
        e, r = f"double.{d}.", f"transformer_blocks.{d}."
        m[e + "img_qkv"] = [r + "attn.to_q.weight", r + "attn.to_k.weight", r + "attn.to_v.weight"]
        m[e + "txt_qkv"] = [r + "attn.add_q_proj.weight", r + "attn.add_k_proj.weight",
                            r + "attn.add_v_proj.weight"]
        m[e + "img_out"] = [r + "attn.to_out.0.weight"]
        m[e + "txt_out"] = [r + "attn.to_add_out.weight"]
        m[e + "img_norm_q"] = [r + "attn.norm_q.weight"]
        m[e + "img_norm_k"] = [r + "attn.norm_k.weight"]
        m[e + "txt_norm_q"] = [r + "attn.norm_added_q.weight"]
        m[e + "txt_norm_k"] = [r + "attn.norm_added_k.weight"]
        m[e + "img_mlp_in"] = [r + "ff.linear_in.weight"]
        m[e + "img_mlp_out"] = [r + "ff.linear_out.weight"]
        m[e + "txt_mlp_in"] = [r + "ff_context.linear_in.weight"]
        m[e + "txt_mlp_out"] = [r + "ff_context.linear_out.weight"]
    for s in range(single):
        e, r = f"single.{s}.", f"single_transformer_blocks.{s}.attn."
        m[e + "proj"] = [r + "to_qkv_mlp_proj.weight"]
        m[e + "out"] = [r + "to_out.weight"]
        m[e + "norm_q"] = [r + "norm_q.weight"]
        m[e + "norm_k"] = [r + "norm_k.weight"]
    return m


class FileWeights:
    """A stand-in for a bonsai_b200.Dit that the CPU oracle (oracle.pyoracle)
    reads its weights from: the tensors of a packed checkpoint file, read by
    the safetensors library and looked up by the reference loader's names, so
    the oracle sees the file's contents independently of the engine's own
    loader.  Model dimensions are copied from `like` (a Dit of the same
    preset and token counts)."""

    def __init__(self, path, like):
        from safetensors.numpy import load_file
        self.t = load_file(str(path))
        self.map = engine_to_reference(like.depth, like.depth_single)
        for a in ("preset", "depth", "depth_single", "mlp", "swiglu", "in_ch", "ctx_dim",
                  "pooled", "axes", "theta", "per_block_mod", "img", "txt", "L", "grid_h",
                  "grid_w"):
            setattr(self, a, getattr(like, a))
        self._like = like

    def weight(self, name: str) -> np.ndarray:
        parts = [self.t[n] for n in self.map[name]]
        return np.ascontiguousarray(np.concatenate(parts, axis=0) if len(parts) > 1 else parts[0]
                                    ).view(np.uint8).reshape(-1)

    def weight_f32(self, name: str) -> np.ndarray:
        (n,) = self.map[name]
        return np.ascontiguousarray(self.t[n], dtype=np.float32).reshape(-1)

    def rope_ids(self) -> np.ndarray:
        return self._like.rope_ids()
