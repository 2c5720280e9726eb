"""Seeded synthetic Flux VAE decoder checkpoints in the reference's layout.

vae_tensor_shapes() lists every tensor the reference's loader reads
(load_vae_weights, src/vae_decoder.cpp:123-250, and the BatchNorm statistics
of :353-373) under its safetensors name, with PyTorch shapes: conv weights
[out][in][kh][kw], linear weights [out][in], vectors [n], all f32.

make_state_dict(seed) fills them from numpy's legacy RandomState (a stream
numpy keeps stable across versions), so the golden-fixture script, the CPU
tests and the GPU tests all rebuild the same weights from a seed.
"""
from __future__ import annotations

import numpy as np

UP_CHANNELS = [(512, 512), (512, 512), (512, 256), (256, 128)]


def vae_tensor_shapes() -> list[tuple[str, tuple[int, ...]]]:
    out: list[tuple[str, tuple[int, ...]]] = []

    def conv(p, co, ci, k):
        out.append((p + ".weight", (co, ci, k, k)))
        out.append((p + ".bias", (co,)))

    def vec2(p, c):
        out.append((p + ".weight", (c,)))
        out.append((p + ".bias", (c,)))

    def resnet(p, ci, co):
        vec2(p + ".norm1", ci)
        conv(p + ".conv1", co, ci, 3)
        vec2(p + ".norm2", co)
        conv(p + ".conv2", co, co, 3)
        if ci != co:
            conv(p + ".conv_shortcut", co, ci, 1)

    conv("post_quant_conv", 32, 32, 1)
    conv("decoder.conv_in", 512, 32, 3)
    resnet("decoder.mid_block.resnets.0", 512, 512)
    a = "decoder.mid_block.attentions.0"
    vec2(a + ".group_norm", 512)
    for n in ("to_q", "to_k", "to_v", "to_out.0"):
        out.append((f"{a}.{n}.weight", (512, 512)))
        out.append((f"{a}.{n}.bias", (512,)))
    resnet("decoder.mid_block.resnets.1", 512, 512)
    for i, (ci, co) in enumerate(UP_CHANNELS):
        for j in range(3):
            resnet(f"decoder.up_blocks.{i}.resnets.{j}", ci if j == 0 else co, co)
        if i < 3:
            conv(f"decoder.up_blocks.{i}.upsamplers.0.conv", co, co, 3)
    vec2("decoder.conv_norm_out", 128)
    conv("decoder.conv_out", 3, 128, 3)
    out.append(("bn.running_mean", (128,)))
    out.append(("bn.running_var", (128,)))
    return out


def make_state_dict(seed: int = 0) -> dict[str, np.ndarray]:
    """Conv / linear weights N(0, 1/fan_in), norm scales 1 + N(0, 0.1), biases
    and norm shifts N(0, 0.05), BatchNorm mean N(0, 0.25), var U(0.25, 4)."""
    rs = np.random.RandomState(seed)
    sd = {}
    for name, shape in vae_tensor_shapes():
        if name == "bn.running_var":
            v = rs.uniform(0.25, 4.0, shape)
        elif name == "bn.running_mean":
            v = 0.5 * rs.standard_normal(shape)
        elif name.endswith(".weight") and len(shape) >= 2:
            v = rs.standard_normal(shape) / np.sqrt(np.prod(shape[1:]))
        elif name.endswith(".weight"):
            v = 1.0 + 0.1 * rs.standard_normal(shape)
        else:
            v = 0.05 * rs.standard_normal(shape)
        sd[name] = np.ascontiguousarray(v, dtype=np.float32)
    return sd
