"""Record what the reference's own checkpoint converters write from the
seeded klein checkpoint of tests/klein_ckpt.py.

Run where the reference checkout is readable; its directory is given by
--ref or the BONSAI_REF_DIR environment variable (one of them is required):

    python tests/golden/make_checkpoint_golden.py --ref <reference checkout>

Steps: write the seeded f32 state dict as diffusion_pytorch_model.safetensors
in a scratch directory, run convert_to_b1_0_packed.py's and
convert_to_b1_0.py's main() there unmodified (imported from the reference
checkout; they read that file and write models/flux2_4b_1bit.safetensors and
models/flux2_4b_1bit.gguf), and store each output's size and SHA-256 in
tests/golden/klein_ckpt.json.  The files themselves (about 1 GB each) are not
committed: tests/klein_ckpt.py writes byte-identical ones, which the tests
check against these hashes before loading them.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib.util
import io
import json
import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

import klein_ckpt  # noqa: E402


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BONSAI_REF_DIR"),
                    required="BONSAI_REF_DIR" not in os.environ,
                    help="the reference checkout (default: $BONSAI_REF_DIR)")
    ap.add_argument("--seed", type=int, default=2024)
    args = ap.parse_args()
    ref = Path(args.ref)
    from safetensors.numpy import save_file
    sd = klein_ckpt.make_state_dict(args.seed)
    packed = _load(ref / "convert_to_b1_0_packed.py", "ref_convert_packed")
    gguf_conv = _load(ref / "convert_to_b1_0.py", "ref_convert_gguf")
    out = {"seed": args.seed, "generator": "tests/klein_ckpt.py make_state_dict",
           "made_by": "the reference's convert_to_b1_0_packed.py and convert_to_b1_0.py main()",
           "files": {}}
    cwd = os.getcwd()
    with tempfile.TemporaryDirectory() as d:
        save_file(sd, os.path.join(d, "diffusion_pytorch_model.safetensors"))
        del sd
        os.chdir(d)
        try:
            log = io.StringIO()
            with contextlib.redirect_stdout(log):
                packed.main()
                gguf_conv.main()
        finally:
            os.chdir(cwd)
        for kind, name in (("safetensors", "flux2_4b_1bit.safetensors"),
                           ("gguf", "flux2_4b_1bit.gguf")):
            p = Path(d) / "models" / name
            out["files"][kind] = {"name": name, "bytes": p.stat().st_size,
                                  "sha256": klein_ckpt.sha256(p)}
    (HERE / "klein_ckpt.json").write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
