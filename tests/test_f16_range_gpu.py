"""The range of the f16 operands.

The engine feeds the tensor cores f16 operands (the LayerNorm-modulated
activations, q / k / v, the MLP activation, the attention output) with f32
accumulation and an f32 residual stream; the reference computes in f32
throughout (src/b1_0_kernel.h:37-43).  f16 carries 3 more mantissa bits than
bf16 but stops at 65504.  A value beyond that rounds to +-inf where it is
written, and the inf turns every downstream value it reaches into inf / NaN,
so an overflow always ends as a non-finite prediction -- never as a finite,
silently wrong one -- and the engine reports it: bonsai_count_nonfinite on
the output, and the NaN / Inf counts of bonsai_dit_sample's per-step stats
(the reference instead aborts when its B1_0 kernel sees NaN / Inf:
src/b1_0_kernel.h:195-198, :230-233).  These tests push one block's linears
far past the range and check exactly that.  For the MLP activation the
reference path (f32, with its own f16 cast of K and V only:
src/diffuser_graph.cpp:409-410) stays finite on the same weights, so there
the difference is reported, not hidden; an overflowing V is non-finite in
the reference path too, because it casts V to f16 as well.
"""
import numpy as np
import pytest

import bonsai_b200 as bb
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def _inputs(m, seed):
    rng = np.random.default_rng(seed)
    img = rng.standard_normal((m.img, m.in_ch)).astype(np.float32)
    txt = rng.standard_normal((m.txt, m.ctx_dim)).astype(np.float32)
    pooled = rng.standard_normal(m.pooled).astype(np.float32)
    return img, txt, pooled


def _scale_b1(m, name, rows, in_dim, value):
    """Set every group scale of a B1_0 weight to `value` (signs unchanged)."""
    raw = m.weight(name).reshape(rows, in_dim // 32, 6).copy()
    raw[:, :, 0:2] = np.full((rows, in_dim // 32), value, np.float16).view(np.uint8).reshape(
        rows, in_dim // 32, 2)
    m.set_weight(name, raw)


@pytest.mark.parametrize("name,rows,ref_finite", [
    ("double.0.img_mlp_in", 12288, True),     # the GELU activation overflows
    ("double.0.img_qkv", 3 * 3072, False)])   # q / k / v overflow
def test_f16_overflow_ends_non_finite_and_is_reported(gpu, name, rows, ref_finite):
    import torch
    m = bb.Dit(bb.PRESET_FLUX1, 64, 32, 8, 8, depth=1, depth_single=1, seed=17)
    try:
        img, txt, pooled = _inputs(m, 3)
        dev = [torch.from_numpy(a).cuda() for a in (img, txt, pooled)]
        out = torch.empty(m.img, m.in_ch, device="cuda")
        m.forward(*dev, 1000.0, out)
        assert bb.count_nonfinite(out) == 0  # in range: finite
        # scales of 1000: outputs ~ 1000 * sqrt(3072) ~ 5.5e4 standard deviation
        _scale_b1(m, name, rows, 3072, 1000.0)
        m.forward(*dev, 1000.0, out)
        torch.cuda.synchronize()
        assert bb.count_nonfinite(out) > 0, "an f16 overflow produced a finite prediction"
        lat = dev[0].clone()
        stats = m.sample(lat, dev[1], dev[2], 1)
        assert stats[0, 0] + stats[0, 1] > 0, stats  # NaN + Inf counts of the step's prediction
        assert bb.device_error() == 0
        # the reference path on the same weights (f32, K and V cast to f16)
        ref = O.dit_forward(m, img, txt, pooled, 1000.0)
        assert bool(np.isfinite(ref).all()) == ref_finite
    finally:
        m.close()
