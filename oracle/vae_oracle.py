"""CPU restatement of the reference's Flux VAE decoder.

TEST INFRASTRUCTURE ONLY: imported by tests/ and bench.py's CPU-baseline leg
as the checker, never by the product code path.

Follows, in f32 NCHW like the reference's ggml graph:
  * the latent preprocessing of src/vae_decoder.cpp:353-421 (BatchNorm
    inverse-normalisation x * sqrt(var + 1e-4) + mean, then the 2x2 spatial
    un-tiling (B,128,h,w) -> (B,32,2h,2w), channel 4c + 2di + dj going to
    pixel (2i + di, 2j + dj) of channel c);
  * build_resnet (src/vae_graph.cpp:44-76): GroupNorm(32, eps 1e-6) + affine,
    SiLU, 3x3 conv, GroupNorm, SiLU, 3x3 conv, optional 1x1 shortcut, sum;
  * build_attention (src/vae_graph.cpp:97-166): single head over all pixels,
    channel width C, scale 1/sqrt(C), q/k/v/out linears with biases,
    residual;
  * build_decoder_graph (src/vae_graph.cpp:174-212): post_quant_conv (1x1),
    conv_in (3x3), mid block (resnet, attention, resnet), four up blocks of
    three resnets (nearest 2x upsample + 3x3 conv after blocks 0-2),
    conv_norm_out + SiLU, conv_out (3x3) -- raw values, no sigmoid.

The reference's ggml is not part of its tree, so this restatement is pinned
against the reference's own PyTorch decoder (tests/run_vae.py FluxDecoder +
preprocess_latent) through the committed fixtures tests/golden/vae_*.npz,
which tests/golden/make_vae_golden.py writes.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
GROUPS = 32
GN_EPS = 1e-6
BN_EPS = 1e-4


def lcg_latent(h: int, w: int, seed: int = 42) -> np.ndarray:
    """The reference's synthetic encoded latent (src/vae_decoder.cpp:394-400):
    seed = seed * 1664525 + 1013904223 (mod 2^32), value = (seed & 0xFFFF) /
    32768 - 1, in (128, h, w) order."""
    n = 128 * h * w
    out = np.empty(n, F32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = F32(s & 0xFFFF) / F32(32768.0) - F32(1.0)
    return out.reshape(128, h, w)


def preprocess(latent: np.ndarray, bn_mean: np.ndarray, bn_var: np.ndarray) -> np.ndarray:
    """(128, h, w) encoded latent -> (32, 2h, 2w) decoder input."""
    lat = np.asarray(latent, F32)
    _, h, w = lat.shape
    std = np.sqrt(np.asarray(bn_var, F32) + F32(BN_EPS)).astype(F32)
    v = (lat * std[:, None, None] + np.asarray(bn_mean, F32)[:, None, None]).astype(F32)
    return np.ascontiguousarray(
        v.reshape(32, 2, 2, h, w).transpose(0, 3, 1, 4, 2).reshape(32, 2 * h, 2 * w))


def conv2d(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Stride-1 convolution with 'same' zero padding (k // 2), as
    ggml_conv_2d_direct(w, x, 1, 1, p, p, 1, 1) + bias."""
    co, ci, kh, kw = w.shape
    c, hh, ww = x.shape
    assert c == ci, (c, ci)
    ph, pw = kh // 2, kw // 2
    xp = np.pad(x, ((0, 0), (ph, ph), (pw, pw)))
    cols = np.empty((ci, kh, kw, hh, ww), F32)
    for dy in range(kh):
        for dx in range(kw):
            cols[:, dy, dx] = xp[:, dy:dy + hh, dx:dx + ww]
    out = w.reshape(co, -1).astype(F32) @ cols.reshape(ci * kh * kw, hh * ww)
    return (out + b.astype(F32)[:, None]).reshape(co, hh, ww).astype(F32)


def group_norm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray) -> np.ndarray:
    c, hh, ww = x.shape
    xg = x.reshape(GROUPS, -1).astype(np.float64)
    mean = xg.mean(axis=1, keepdims=True)
    var = ((xg - mean) ** 2).mean(axis=1, keepdims=True)
    y = ((xg - mean) / np.sqrt(var + GN_EPS)).astype(F32).reshape(c, hh, ww)
    return (y * gamma.astype(F32)[:, None, None] + beta.astype(F32)[:, None, None]).astype(F32)


def silu(x: np.ndarray) -> np.ndarray:
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def resnet(x: np.ndarray, sd: dict, p: str) -> np.ndarray:
    h = silu(group_norm(x, sd[p + ".norm1.weight"], sd[p + ".norm1.bias"]))
    h = conv2d(h, sd[p + ".conv1.weight"], sd[p + ".conv1.bias"])
    h = silu(group_norm(h, sd[p + ".norm2.weight"], sd[p + ".norm2.bias"]))
    h = conv2d(h, sd[p + ".conv2.weight"], sd[p + ".conv2.bias"])
    if p + ".conv_shortcut.weight" in sd:
        x = conv2d(x, sd[p + ".conv_shortcut.weight"], sd[p + ".conv_shortcut.bias"])
    return (x + h).astype(F32)


def attention(x: np.ndarray, sd: dict, p: str) -> np.ndarray:
    c, hh, ww = x.shape
    g = group_norm(x, sd[p + ".group_norm.weight"], sd[p + ".group_norm.bias"])
    t = g.reshape(c, hh * ww).T  # [seq][C], pixel y*W + x

    def lin(name, v):
        return (v @ sd[f"{p}.{name}.weight"].T + sd[f"{p}.{name}.bias"]).astype(F32)

    q, k, v = lin("to_q", t), lin("to_k", t), lin("to_v", t)
    s = (q @ k.T).astype(F32) * F32(1.0 / np.sqrt(c))
    s = s - s.max(axis=1, keepdims=True)
    e = np.exp(s).astype(F32)
    pr = (e / e.sum(axis=1, keepdims=True)).astype(F32)
    o = lin("to_out.0", (pr @ v).astype(F32))
    return (x + o.T.reshape(c, hh, ww)).astype(F32)


def upsample2(x: np.ndarray) -> np.ndarray:
    return np.repeat(np.repeat(x, 2, axis=1), 2, axis=2)


def decoder(sd: dict, x: np.ndarray) -> np.ndarray:
    """(32, H, W) preprocessed latent -> (3, 8H, 8W) raw decoder output."""
    x = conv2d(x, sd["post_quant_conv.weight"], sd["post_quant_conv.bias"])
    x = conv2d(x, sd["decoder.conv_in.weight"], sd["decoder.conv_in.bias"])
    x = resnet(x, sd, "decoder.mid_block.resnets.0")
    x = attention(x, sd, "decoder.mid_block.attentions.0")
    x = resnet(x, sd, "decoder.mid_block.resnets.1")
    for i in range(4):
        for j in range(3):
            x = resnet(x, sd, f"decoder.up_blocks.{i}.resnets.{j}")
        if i < 3:
            p = f"decoder.up_blocks.{i}.upsamplers.0.conv"
            x = conv2d(upsample2(x), sd[p + ".weight"], sd[p + ".bias"])
    x = silu(group_norm(x, sd["decoder.conv_norm_out.weight"], sd["decoder.conv_norm_out.bias"]))
    return conv2d(x, sd["decoder.conv_out.weight"], sd["decoder.conv_out.bias"])


def decode(sd: dict, latent: np.ndarray) -> np.ndarray:
    """(128, h, w) encoded latent -> (3, 16h, 16w) raw image."""
    return decoder(sd, preprocess(latent, sd["bn.running_mean"], sd["bn.running_var"]))


def to_png(raw: np.ndarray) -> np.ndarray:
    """The reference's visualisation (tests/run_vae.py decode_to_png,
    src/vae_decoder.cpp:262-281): sigmoid, x255, clip, u8, HWC."""
    a = 1.0 / (1.0 + np.exp(-raw.astype(np.float64)))
    return np.clip(a * 255.0, 0, 255).astype(np.uint8).transpose(1, 2, 0)
