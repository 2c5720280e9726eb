"""The Flux VAE decoder oracle (oracle/vae_oracle.py) pinned to the
reference's own PyTorch decoder through the committed fixtures
tests/golden/vae_<h>x<w>.npz (written by tests/golden/make_vae_golden.py
from tests/run_vae.py FluxDecoder), plus the host-side pieces of the
decoder: the reference's synthetic latent and its checkpoint layout."""
from pathlib import Path

import numpy as np
import pytest

from oracle import vae_oracle as vo
from vae_weights import make_state_dict, vae_tensor_shapes

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def sd():
    return make_state_dict(7)


@pytest.mark.parametrize("hw", [(2, 2), (3, 5)])
def test_oracle_matches_reference_decoder(sd, hw):
    g = np.load(GOLDEN / f"vae_{hw[0]}x{hw[1]}.npz")
    assert int(g["seed"]) == 7
    lat = vo.lcg_latent(*hw)
    assert np.array_equal(lat, g["latent"])  # the reference's LCG latent, bit for bit
    out = vo.decode(sd, lat)
    ref = g["raw"]
    assert out.shape == ref.shape == (3, 16 * hw[0], 16 * hw[1])
    rms = np.sqrt((ref ** 2).mean())
    assert np.abs(out - ref).max() <= 1e-4 * rms
    # the reference test's own criterion (tests/test_vae.py: MSE < 5e-5 on
    # the sigmoid PNG); the f32 restatement reproduces the PNG exactly
    assert np.array_equal(vo.to_png(out), g["png"])


def test_preprocess_untiling():
    """Channel 4c + 2di + dj of latent pixel (i, j) lands at (2i+di, 2j+dj)
    of channel c, after x * sqrt(var + 1e-4) + mean (src/vae_decoder.cpp:402-421)."""
    rng = np.random.default_rng(0)
    lat = rng.standard_normal((128, 3, 4)).astype(np.float32)
    mean = rng.standard_normal(128).astype(np.float32)
    var = rng.uniform(0.1, 2, 128).astype(np.float32)
    post = vo.preprocess(lat, mean, var)
    std = np.sqrt(var + np.float32(1e-4)).astype(np.float32)
    for c, i, j, di, dj in [(0, 0, 0, 0, 0), (5, 2, 3, 1, 0), (31, 1, 2, 1, 1), (17, 2, 0, 0, 1)]:
        sc = 4 * c + 2 * di + dj
        assert post[c, 2 * i + di, 2 * j + dj] == lat[sc, i, j] * std[sc] + mean[sc]


def test_checkpoint_layout_matches_reference_loader():
    """Every tensor load_vae_weights reads, with the PyTorch shapes the
    reference's FluxDecoder state dict has (fixtures were made from it)."""
    names = dict(vae_tensor_shapes())
    assert len(names) == len(vae_tensor_shapes())
    assert names["decoder.conv_in.weight"] == (512, 32, 3, 3)
    assert names["decoder.mid_block.attentions.0.to_out.0.weight"] == (512, 512)
    assert names["decoder.up_blocks.2.resnets.0.conv_shortcut.weight"] == (256, 512, 1, 1)
    assert names["decoder.up_blocks.3.resnets.0.conv_shortcut.weight"] == (128, 256, 1, 1)
    assert "decoder.up_blocks.3.upsamplers.0.conv.weight" not in names
    assert "decoder.up_blocks.1.resnets.0.conv_shortcut.weight" not in names
    assert names["decoder.conv_out.weight"] == (3, 128, 3, 3)
    total = sum(int(np.prod(s)) for s in names.values())
    assert 49_000_000 < total < 50_000_000


def test_lcg_latent_prefix():
    """First values of the reference's generator (seed 42): s = s*1664525 +
    1013904223 mod 2^32, v = (s & 0xFFFF) / 32768 - 1."""
    lat = vo.lcg_latent(1, 1)
    s = 42
    for i in range(8):
        s = (s * 1664525 + 1013904223) % 2 ** 32
        assert lat.reshape(-1)[i] == np.float32((s & 0xFFFF) / 32768.0 - 1.0)
