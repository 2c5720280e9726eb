"""The Flux VAE decoder on the device (bonsai_vae_*, bonsai_conv2d_nhwc)
against the reference.

* bonsai_conv2d_nhwc (the tcgen05 implicit-GEMM kernel behind every conv and
  linear of the decoder) against torch's fp32 conv2d on the same 16-bit
  operands: 3x3 and 1x1, ragged images, narrow and wide channel counts, bias
  and residual -- in both forms of the kernel (CTA pair, the default, and
  single CTA; BONSAI_VAE_CONV selects).
* The whole decoder, loaded from a checkpoint in the reference's layout,
  against the reference's PyTorch decoder (golden fixtures) and against the
  f32 oracle at further sizes.  Tolerance: the reference's own bar for its
  C++ port (tests/test_vae.py: MSE of the sigmoid PNG < 5e-5), plus cosine
  >= 0.9999 and max |err| <= 5e-2 x RMS on the raw output (16-bit operands,
  f32 accumulation, ~35 chained convolutions).
* Full 1024^2 decode: deterministic and finite.
"""
from pathlib import Path

import numpy as np
import pytest

import bonsai_b200 as bb
from oracle import vae_oracle as vo
from st_writer import write_safetensors
from vae_weights import make_state_dict

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(params=["pair", "single"])
def conv_kernel(request, monkeypatch):
    monkeypatch.setenv("BONSAI_VAE_CONV", request.param)
    return request.param


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    sd = make_state_dict(7)
    p = tmp_path_factory.mktemp("vae") / "flux2-vae.safetensors"
    write_safetensors(p, sd)
    return sd, p


def _metrics(out, ref):
    rms = float(np.sqrt((ref.astype(np.float64) ** 2).mean()))
    err = float(np.abs(out - ref).max()) / rms
    cos = float((out.astype(np.float64) * ref).sum() /
                np.sqrt((out.astype(np.float64) ** 2).sum() * (ref.astype(np.float64) ** 2).sum()))
    png_mse = float((((vo.to_png(out).astype(np.float64) - vo.to_png(ref)) / 255.0) ** 2).mean())
    return err, cos, png_mse


@pytest.mark.parametrize("H,W,cin,cout,k,dtype,resid", [
    (8, 8, 64, 64, 3, "f16", False),
    (13, 29, 128, 256, 3, "f16", True),
    (32, 32, 512, 512, 3, "f16", True),
    (5, 7, 64, 16, 1, "bf16", False),
    (16, 200, 256, 128, 3, "bf16", False),
    (40, 24, 128, 3, 3, "f16", False),
    (3, 300, 512, 320, 1, "f16", True),
    (1, 1, 64, 32, 3, "f16", False),
    (24, 40, 64, 3, 3, "f16", True),
    (33, 65, 128, 128, 3, "bf16", True),
    # widths that are multiples of 128: one 128-pixel row per tile, the three
    # horizontal taps share one halo box
    (4, 256, 64, 128, 3, "f16", True),
    (3, 384, 128, 256, 3, "bf16", False),
    (2, 128, 512, 512, 3, "f16", True),
    (6, 128, 256, 3, 3, "f16", False),
    (9, 512, 128, 128, 3, "f16", True),
])
def test_conv2d_matches_torch(gpu, conv_kernel, H, W, cin, cout, k, dtype, resid):
    import torch
    g = torch.Generator(device="cuda").manual_seed(H * 1000 + W)
    td = torch.float16 if dtype == "f16" else torch.bfloat16
    x = torch.randn(H, W, cin, device="cuda", generator=g).to(td)
    w = (torch.randn(cout, cin, k, k, device="cuda", generator=g) / (cin * k * k) ** 0.5)
    b = torch.randn(cout, device="cuda", generator=g)
    r = torch.randn(H, W, cout, device="cuda", generator=g) if resid else None
    out = torch.empty(H, W, cout, device="cuda")
    bb.conv2d_nhwc(x, w, b, out, resid=r)
    torch.cuda.synchronize()
    ref = torch.nn.functional.conv2d(x.float().permute(2, 0, 1)[None], w.to(td).float(), b,
                                     padding=k // 2)[0].permute(1, 2, 0)
    if r is not None:
        ref = ref + r
    err = (out - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-3, err


@pytest.mark.parametrize("hw", [(2, 2), (3, 5)])
def test_decode_matches_reference_decoder(gpu, ckpt, conv_kernel, hw):
    import torch
    sd, path = ckpt
    g = np.load(GOLDEN / f"vae_{hw[0]}x{hw[1]}.npz")
    v = bb.Vae(*hw, seed=3)
    try:
        v.load_safetensors(path)
        lat = torch.from_numpy(g["latent"]).cuda()
        img = torch.empty(3, 16 * hw[0], 16 * hw[1], device="cuda")
        v.decode(lat, img)
        torch.cuda.synchronize()
        out = img.cpu().numpy()
    finally:
        v.close()
    err, cos, png_mse = _metrics(out, g["raw"])
    print(f"vae {hw} {conv_kernel}: max|err|/rms {err:.3e} cos {cos:.7f} png mse {png_mse:.2e}")
    assert png_mse < 5e-5
    assert cos >= 0.9999
    assert err <= 5e-2


@pytest.mark.parametrize("hw", [(1, 1), (4, 4), (1, 7), (8, 8), (16, 16)])
def test_decode_matches_oracle(gpu, ckpt, hw):
    sd, path = ckpt
    lat = np.random.default_rng(hw[0] * 10 + hw[1]).uniform(-1, 1, (128, *hw)).astype(np.float32)
    v = bb.Vae(*hw, seed=3)
    try:
        v.load_safetensors(path)
        out = v.decode_host(lat)
    finally:
        v.close()
    ref = vo.decode(sd, lat)
    err, cos, png_mse = _metrics(out, ref)
    print(f"vae {hw}: max|err|/rms {err:.3e} cos {cos:.7f} png mse {png_mse:.2e}")
    assert png_mse < 5e-5
    assert cos >= 0.9999
    assert err <= 5e-2


def test_rgb8_matches_reference_conversion(gpu):
    import torch
    x = torch.randn(3, 37, 53, device="cuda") * 4
    x[0, 0, :5] = torch.tensor([0.0, 100.0, -100.0, float("inf"), -float("inf")])
    rgb = torch.empty(37, 53, 3, dtype=torch.uint8, device="cuda")
    bb.vae_rgb8(x, rgb)
    torch.cuda.synchronize()
    ref = vo.to_png(x.cpu().numpy())
    got = rgb.cpu().numpy()
    assert np.abs(got.astype(int) - ref).max() <= 1
    assert (got != ref).mean() < 1e-3


def test_load_errors(gpu, ckpt, tmp_path):
    sd, _ = ckpt
    v = bb.Vae(1, 1, seed=3)
    try:
        bad = dict(sd)
        del bad["decoder.up_blocks.1.resnets.2.conv2.bias"]
        p = tmp_path / "missing.safetensors"
        write_safetensors(p, bad)
        with pytest.raises(bb.BonsaiError, match="conv2.bias' not found"):
            v.load_safetensors(p)
        bad = dict(sd)
        bad["decoder.conv_in.weight"] = bad["decoder.conv_in.weight"][:, :16]
        p = tmp_path / "shape.safetensors"
        write_safetensors(p, bad)
        with pytest.raises(bb.BonsaiError, match="conv_in.weight' must have shape"):
            v.load_safetensors(p)
        bad = dict(sd)
        bad["bn.running_var"] = bad["bn.running_var"].astype(np.float64)
        p = tmp_path / "dtype.safetensors"
        write_safetensors(p, bad)
        with pytest.raises(bb.BonsaiError, match="must be F32"):
            v.load_safetensors(p)
    finally:
        v.close()


def test_bf16_checkpoint_loads(gpu, ckpt, tmp_path):
    """A bf16 checkpoint gives the same device weights as its f32 upcast."""
    import torch
    sd, _ = ckpt
    lat = np.random.default_rng(5).uniform(-1, 1, (128, 2, 2)).astype(np.float32)
    bf = {k: torch.from_numpy(a).to(torch.bfloat16) for k, a in sd.items()}
    p16 = tmp_path / "bf16.safetensors"
    write_safetensors(p16, {k: t.view(torch.int16).numpy().view(np.uint16) for k, t in bf.items()},
                      dtypes={k: "BF16" for k in bf})
    p32 = tmp_path / "up.safetensors"
    write_safetensors(p32, {k: t.float().numpy() for k, t in bf.items()})
    outs = []
    for p in (p16, p32):
        v = bb.Vae(2, 2, seed=3)
        try:
            v.load_safetensors(p)
            outs.append(v.decode_host(lat))
        finally:
            v.close()
    assert np.array_equal(outs[0], outs[1])


def test_full_size_decode_deterministic(gpu):
    """1024^2 image (latent 64x64, attention over 16384 pixels) with seeded
    synthetic weights: two decodes are bit-identical and finite."""
    import torch
    v = bb.Vae(64, 64, seed=11)
    try:
        lat = torch.from_numpy(vo.lcg_latent(64, 64)).cuda()
        a = torch.empty(3, 1024, 1024, device="cuda")
        b = torch.empty_like(a)
        v.decode(lat, a)
        v.decode(lat, b)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
        assert torch.isfinite(a).all()
        assert a.std().item() > 1e-3
        assert bb.count_nonfinite(a) == 0
    finally:
        v.close()
