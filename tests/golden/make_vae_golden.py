"""Generate the Flux VAE decoder fixtures from the reference's own PyTorch
decoder.

Run where the reference checkout is readable; its directory is given by
--ref or the BONSAI_REF_DIR environment variable (one of them is required)
and torch:

    python tests/golden/make_vae_golden.py --ref <reference checkout>

For each latent size (h, w) it builds the reference's FluxDecoder
(tests/run_vae.py), loads the seeded synthetic checkpoint of
tests/vae_weights.py the way load_decoder_weights does (the 'decoder.'
prefix stripped, post_quant_conv kept), draws the reference's LCG latent
(generate_synthetic_latent, seed 42), preprocesses it with preprocess_latent
and decodes in f32 on the CPU.  vae_<h>x<w>.npz holds the latent, the raw
decoder output [3][16h][16w] and the reference's u8 PNG array
(decode_to_png); the weights are not stored -- tests rebuild them from the
seed.  The reference imports safetensors at module level only for its file
loader, which is not used here; a stub stands in when the package is absent.
"""
from __future__ import annotations

import argparse
import os
import importlib.util
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from vae_weights import make_state_dict  # noqa: E402

SIZES = [(2, 2), (3, 5)]
SEED = 7


def load_run_vae(ref: Path):
    try:
        import safetensors.torch  # noqa: F401
    except ImportError:
        stub = types.ModuleType("safetensors")
        stub_t = types.ModuleType("safetensors.torch")

        def _absent(*_a, **_k):
            raise RuntimeError("safetensors is not installed")

        stub_t.load_file = _absent
        stub.torch = stub_t
        sys.modules["safetensors"] = stub
        sys.modules["safetensors.torch"] = stub_t
    spec = importlib.util.spec_from_file_location("ref_run_vae", ref / "tests" / "run_vae.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BONSAI_REF_DIR"),
                    required="BONSAI_REF_DIR" not in os.environ,
                    help="the reference checkout (default: $BONSAI_REF_DIR)")
    args = ap.parse_args()
    import torch

    rv = load_run_vae(Path(args.ref))
    sd = make_state_dict(SEED)
    dec_sd = {}
    for k, v in sd.items():
        if k.startswith("decoder."):
            dec_sd[k[len("decoder."):]] = torch.from_numpy(v)
        elif k.startswith("post_quant_conv."):
            dec_sd[k] = torch.from_numpy(v)
    decoder = rv.FluxDecoder()
    decoder.load_state_dict(dec_sd)
    decoder.eval()
    mean = torch.from_numpy(sd["bn.running_mean"])
    var = torch.from_numpy(sd["bn.running_var"])
    torch.set_num_threads(max(1, torch.get_num_threads()))
    for h, w in SIZES:
        lat = rv.generate_synthetic_latent(h, w)
        x = rv.preprocess_latent(torch.from_numpy(lat), mean, var)
        with torch.no_grad():
            out = decoder(x)
        raw = out[0].numpy().astype(np.float32)
        png = rv.decode_to_png(out[0])
        np.savez(HERE / f"vae_{h}x{w}.npz", seed=np.int64(SEED), latent=lat.astype(np.float32),
                 raw=raw, png=png)
        print(f"vae_{h}x{w}.npz: raw {raw.shape} rms {np.sqrt((raw ** 2).mean()):.4f} "
              f"png mean {png.mean():.1f}")


if __name__ == "__main__":
    main()
