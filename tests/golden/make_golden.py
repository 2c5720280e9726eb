"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run where the reference checkout is readable; its directory is given by
--ref or the BONSAI_REF_DIR environment variable (one of them is required)
and the reference's C kernels built into oracle/_ref (make -C oracle):

    python tests/golden/make_golden.py --ref <reference checkout>

Every output value comes from the reference itself:
  * b1_kat.npz       - the literal 64-weight row of the reference's B1_0
                       quantize/dequant known-answer test
                       (tests/ops/test_b1_linear.py:75-127), packed with the
                       reference packer quantize_b1_0
                       (convert_to_b1_0_packed.py:21-43).
  * b1_linear.npz    - seeded float weights packed by quantize_b1_0, seeded
                       activations, and the outputs of the reference kernel
                       b1_linear_f32_f32 (src/b1_0_kernel.h:37-288), both its
                       scalar and its AVX2 path, compiled from the reference
                       sources into oracle/_ref.
  * rope.npz         - RoPE frequency / cos / sin tables from the reference's
                       Python restatements _build_rope_freqs_table and
                       _build_rope_cos_sin (tests/ops/test_rope_2d.py:14-55)
                       for both axis presets, and rope_2d_fwd_f32
                       (src/b1_0_kernel.h:309-361) applied by oracle/_ref.
The fixtures are small (< 1 MB in total) and committed; tests read them
without needing the reference.
"""
from __future__ import annotations

import argparse
import os
import ast
import ctypes
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def kat_row(ref: Path) -> np.ndarray:
    """The literal weight row of test_quantification_b1_0_exact, read from the
    reference test file (not retyped)."""
    src = (ref / "tests/ops/test_b1_linear.py").read_text()
    tree = ast.parse(src)
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == "test_quantification_b1_0_exact":
            for sub in ast.walk(node):
                if (isinstance(sub, ast.Call) and getattr(sub.func, "attr", "") == "tensor"
                        and sub.args and isinstance(sub.args[0], ast.List)):
                    return np.array(ast.literal_eval(sub.args[0]), dtype=np.float32)
    raise RuntimeError("KAT row not found in the reference test")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BONSAI_REF_DIR"),
                    required="BONSAI_REF_DIR" not in os.environ,
                    help="the reference checkout (default: $BONSAI_REF_DIR)")
    args = ap.parse_args()
    ref = Path(args.ref)

    packer = load_module(ref / "convert_to_b1_0_packed.py", "ref_packer")
    quantize_b1_0 = packer.quantize_b1_0

    # ---------------------------------------------------------- B1_0 KAT
    w = kat_row(ref)                                  # [1][64]
    packed = quantize_b1_0(w)                         # [1][12]
    blocks = w.reshape(1, -1, 32)
    scales = np.abs(blocks).mean(-1)                  # the test's scale rule (mean |w|)
    deq = np.where(blocks >= 0, scales[..., None], -scales[..., None]).reshape(w.shape)
    np.savez(HERE / "b1_kat.npz", weight=w, packed=packed, scales=scales.astype(np.float32),
             dequant=deq.astype(np.float32))

    # ------------------------------------------------- B1_0 linear (reference C)
    lib_avx = ctypes.CDLL(str(REPO / "oracle/_ref/libbonsai_ref.so"))
    lib_sc = ctypes.CDLL(str(REPO / "oracle/_ref/libbonsai_ref_scalar.so"))
    assert lib_avx.ref_has_avx2() == 1 and lib_sc.ref_has_avx2() == 0
    for L in (lib_avx, lib_sc):
        L.ref_b1_linear.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                    ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        L.ref_rope_2d.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p,
                                                                             ctypes.c_int]
    shapes = [(1, 64, 32), (5, 96, 40), (17, 256, 130), (3, 3072, 24), (40, 512, 68)]
    out = {}
    rng = np.random.default_rng(20240601)
    for i, (T, K, N) in enumerate(shapes):
        wf = rng.standard_normal((N, K)).astype(np.float32) * 0.02
        pk = np.ascontiguousarray(quantize_b1_0(wf))
        act = rng.standard_normal((T, K)).astype(np.float32)
        o_avx = np.zeros((T, N), np.float32)
        o_sc = np.zeros((T, N), np.float32)
        lib_avx.ref_b1_linear(act.ctypes.data, T, K, pk.ctypes.data, N, o_avx.ctypes.data, 3)
        lib_sc.ref_b1_linear(act.ctypes.data, T, K, pk.ctypes.data, N, o_sc.ctypes.data, 3)
        out[f"packed_{i}"] = pk
        out[f"act_{i}"] = act
        out[f"out_avx2_{i}"] = o_avx
        out[f"out_scalar_{i}"] = o_sc
        out[f"shape_{i}"] = np.array([T, K, N], np.int32)
    out["n"] = np.array(len(shapes), np.int32)
    np.savez_compressed(HERE / "b1_linear.npz", **out)

    # ------------------------------------------------------------------ RoPE
    sys.path.insert(0, str(ref))
    rope_mod = load_module(ref / "tests/ops/test_rope_2d.py", "ref_rope_tests")
    res = {}
    presets = {"klein": ([32, 32, 32, 32], 2000.0, (0, 0, 1, 1)),
               "flux1": ([16, 56, 56], 10000.0, (0, 1, 1))}
    for name, (axes, theta, grid_axes) in presets.items():
        n_axes = len(axes)
        gh, gw, txt = 6, 5, 3
        seq = txt + gh * gw
        ids = np.zeros((n_axes, seq), np.float32)  # the reference helper's [n_axes][seq] layout
        for y in range(gh):
            for x in range(gw):
                ids[n_axes - 2, txt + y * gw + x] = y
                ids[n_axes - 1, txt + y * gw + x] = x
        freqs = rope_mod._build_rope_freqs_table(axes, theta)
        cos_t, sin_t = rope_mod._build_rope_cos_sin(ids, freqs, axes)  # [64][seq]
        half = cos_t.shape[0]
        heads, hd = 3, 2 * half
        x = rng.standard_normal((seq, heads, hd)).astype(np.float32)
        c_sd = np.ascontiguousarray(cos_t.T.astype(np.float32))  # [seq][64] (ggml ne = {64, seq})
        s_sd = np.ascontiguousarray(sin_t.T.astype(np.float32))
        y_ref = np.zeros_like(x)
        lib_sc.ref_rope_2d(x.ctypes.data, c_sd.ctypes.data, s_sd.ctypes.data, hd, heads, seq,
                           y_ref.ctypes.data, 2)
        res[f"{name}_axes"] = np.array(axes, np.int32)
        res[f"{name}_theta"] = np.array(theta, np.float32)
        res[f"{name}_ids"] = np.ascontiguousarray(ids.T)  # [seq][n_axes]
        res[f"{name}_freqs"] = freqs.astype(np.float32)
        res[f"{name}_cos"] = c_sd
        res[f"{name}_sin"] = s_sd
        res[f"{name}_x"] = x
        res[f"{name}_rot"] = y_ref
    np.savez_compressed(HERE / "rope.npz", **res)
    for f in ("b1_kat.npz", "b1_linear.npz", "rope.npz"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
