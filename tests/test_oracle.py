"""CPU oracle pinned against the reference (no GPU).

Golden fixtures come from tests/golden/make_golden.py, which ran the
reference's own packer (convert_to_b1_0_packed.py), its B1_0 / RoPE C
kernels (src/b1_0_kernel.h, compiled unmodified into oracle/_ref) and its
Python RoPE helpers (tests/ops/test_rope_2d.py).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import pyoracle as O
import bonsai_b200 as bb

GOLD = Path(__file__).resolve().parent / "golden"


def test_b1_kat_quantize_dequant():
    """Known-answer test of tests/ops/test_b1_linear.py:75-127 on the
    reference's literal 64-weight row, packed by the reference packer."""
    g = np.load(GOLD / "b1_kat.npz")
    w, packed = g["weight"], g["packed"]
    assert packed.shape == (1, 12)
    raw = packed.reshape(1, 2, 6)
    scales16 = raw[:, :, 0:2].copy().view(np.float16).reshape(1, 2)
    # scale = mean |w| per 32-block, stored as f16 (convert_to_b1_0_packed.py:34)
    np.testing.assert_array_equal(scales16, g["scales"].astype(np.float16))
    bits = np.unpackbits(raw[:, :, 2:6], axis=-1, bitorder="little").reshape(1, 64)
    np.testing.assert_array_equal(bits, (w >= 0).astype(np.uint8))
    deq = bb.dequant_b1(packed, 1, 64)
    np.testing.assert_allclose(deq, g["dequant"], rtol=1e-3, atol=1e-5)
    # the oracle's B1 linear of a one-hot activation reproduces each dequantised weight
    eye = np.eye(64, dtype=np.float32)
    cols = O.b1_linear(eye, packed, 1)[:, 0]
    np.testing.assert_array_equal(cols, deq[0])


def test_b1_linear_matches_reference_kernel():
    """orc_b1_linear is bit-exact with the reference's scalar kernel and within
    float rounding of its AVX2 kernel (different summation order)."""
    g = np.load(GOLD / "b1_linear.npz")
    for i in range(int(g["n"])):
        T, K, N = (int(v) for v in g[f"shape_{i}"])
        out = O.b1_linear(g[f"act_{i}"], g[f"packed_{i}"], N)
        np.testing.assert_array_equal(out, g[f"out_scalar_{i}"])
        ref = g[f"out_avx2_{i}"]
        rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
        assert np.max(np.abs(out - ref)) <= 1e-5 * rms + 1e-7


@pytest.mark.parametrize("preset", ["klein", "flux1"])
def test_rope_tables_and_rotation(preset):
    g = np.load(GOLD / "rope.npz")
    axes = g[f"{preset}_axes"]
    theta = float(g[f"{preset}_theta"])
    freqs = O.rope_freqs(axes, theta)
    np.testing.assert_allclose(freqs, g[f"{preset}_freqs"], rtol=1e-6)
    c, s = O.rope_cos_sin(g[f"{preset}_ids"], axes, theta)
    # the reference's RoPE tolerance (tests/ops/test_all_ops.py:339-340)
    np.testing.assert_allclose(c, g[f"{preset}_cos"], atol=1e-5)
    np.testing.assert_allclose(s, g[f"{preset}_sin"], atol=1e-5)
    np.testing.assert_allclose(c * c + s * s, 1.0, atol=1e-5)
    rot = O.rope_apply(g[f"{preset}_x"], g[f"{preset}_cos"], g[f"{preset}_sin"])
    assert np.max(np.abs(rot - g[f"{preset}_rot"])) < 1e-6


def test_rope_quarter_turn_kat():
    """cos = 0, sin = 1 maps (a, b) -> (-b, a) (tests/ops/test_rope_2d.py:103-127)."""
    x = np.ones((1, 1, 128), np.float32)
    x[0, 0, 1::2] = 2.0
    out = O.rope_apply(x, np.zeros((1, 64), np.float32), np.ones((1, 64), np.float32))
    np.testing.assert_array_equal(out[0, 0, 0::2], -x[0, 0, 1::2])
    np.testing.assert_array_equal(out[0, 0, 1::2], x[0, 0, 0::2])


def test_live_reference_matches_oracle():
    """When oracle/_ref is present, run the reference's kernels on fresh data."""
    if O.ref() is None or O.ref(scalar=True) is None:
        pytest.skip("oracle/_ref not built (needs the reference checkout)")
    rng = np.random.default_rng(9)
    T, K, N = 23, 768, 200
    packed = bb.random_b1_packed(N, K, rng)
    act = rng.standard_normal((T, K)).astype(np.float32)
    ours = O.b1_linear(act, packed, N)
    np.testing.assert_array_equal(ours, O.ref_b1_linear(act, packed, N, scalar=True))
    avx = O.ref_b1_linear(act, packed, N, nthreads=3)
    assert np.max(np.abs(ours - avx)) <= 1e-5 * np.sqrt(np.mean(avx.astype(np.float64) ** 2))


def test_pure_math_restatements():
    """LayerNorm / RMSNorm / SwiGLU / attention follow the reference's math
    restatements (tests/ops/test_all_ops.py:27-113)."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((7, 96)).astype(np.float32) * 3 + 1
    sh, sc = rng.standard_normal(96).astype(np.float32), rng.standard_normal(96).astype(np.float32)
    xd = x.astype(np.float64)
    ln = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-6)
    np.testing.assert_allclose(O.ln_modulate(x, sh, sc), ln * (1 + sc) + sh, rtol=1e-5, atol=1e-5)
    w = rng.standard_normal(96).astype(np.float32)
    rms = xd / np.sqrt((xd ** 2).mean(1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(O.rms_norm(x, w), rms, rtol=1e-5, atol=1e-5)
    g2 = rng.standard_normal((5, 64)).astype(np.float32)
    sw = g2[:, :32] / (1 + np.exp(-g2[:, :32].astype(np.float64))) * g2[:, 32:]
    np.testing.assert_allclose(O.swiglu(g2), sw, rtol=1e-5, atol=1e-6)
    q, k, v = (rng.standard_normal((19, 2, 16)).astype(np.float32) for _ in range(3))
    r16 = lambda a: a.astype(np.float16).astype(np.float64)
    s = np.einsum("qhd,khd->hqk", r16(q), r16(k)) * 0.25
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ref = np.einsum("hqk,khd->qhd", p, r16(v)).reshape(19, 32)
    np.testing.assert_allclose(O.attention(q, k, v, 0.25), ref, rtol=1e-4, atol=1e-5)


def test_timestep_embedding_sin_cos_order():
    """[sin, cos] after the half swap of src/diffuser_graph.cpp:288-292."""
    e = O.timestep_embedding(1000.0)
    j = np.arange(128)
    f = np.exp(-np.log(10000.0) * j / 128)
    np.testing.assert_allclose(e[:128], np.sin(1000.0 * f), atol=2e-3)
    np.testing.assert_allclose(e[128:], np.cos(1000.0 * f), atol=2e-3)
