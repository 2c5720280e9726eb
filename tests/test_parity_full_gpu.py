"""Parity at the sizes the benchmark runs.

* the whole Flux.1 step at full depth (19 double + 38 single blocks), so the
  drift accumulated through every block is measured, against the oracle whose
  every B1_0 linear is the reference's own b1_linear_f32_f32 (AVX2 build in
  oracle/_ref; the reference runs all blocks in one graph:
  src/diffuser_graph.cpp:340-342, :475-477);
* one double and one single block at the 1024^2 step's sequence, L = 4608
  (512 text + 4096 image tokens), against the same oracle;
* the joint attention at L = 4608 and at the 2048^2 sequence L = 16896 against
  a torch fp32 softmax attention on the same f16 inputs, with key blocks
  planted so that a 64-key block's softmax row sum exceeds 2^15 against the
  running maximum: the attention kernel redoes such a block with its own max
  (the path random inputs almost never take).

Bar (the reference's GPU-vs-CPU acceptance, tests/c_ops/test_webgpu_diffuser_ops.cpp:310):
cos >= 0.9999 and max-abs <= 1e-2 * RMS.
"""
import os

import numpy as np
import pytest

import bonsai_b200 as bb
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu
H = 3072
THREADS = os.cpu_count() or 4


def _metrics(got, ref):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    cos = float(got @ ref / (np.linalg.norm(got) * np.linalg.norm(ref)))
    rel = float(np.max(np.abs(got - ref)) / np.sqrt(np.mean(ref ** 2)))
    return cos, rel


def _check(got, ref, what, cos_min=0.9999, rel_max=1e-2):
    cos, rel = _metrics(got, ref)
    print(f"{what}: cos={cos:.7f} maxabs/rms={rel:.2e}")
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    assert cos >= cos_min and rel <= rel_max, f"{what}: cos={cos:.7f} maxabs/rms={rel:.3e}"


def test_forward_full_depth_flux1(gpu):
    """19 + 38 blocks, 32 text + 8x8 image tokens, vs the reference-kernel oracle."""
    import torch
    m = bb.Dit(bb.PRESET_FLUX1, 64, 32, 8, 8, seed=31)
    assert (m.depth, m.depth_single) == (19, 38)
    rng = np.random.default_rng(8)
    img = rng.standard_normal((m.img, m.in_ch)).astype(np.float32)
    txt = rng.standard_normal((m.txt, m.ctx_dim)).astype(np.float32)
    pooled = rng.standard_normal(m.pooled).astype(np.float32)
    out = torch.empty(m.img, m.in_ch, device="cuda")
    m.forward(torch.from_numpy(img).cuda(), torch.from_numpy(txt).cuda(),
              torch.from_numpy(pooled).cuda(), 750.0, out)
    got = out.cpu().numpy()
    assert bb.device_error() == 0
    used = O.use_reference_b1(True, nthreads=THREADS)
    try:
        ref = O.dit_forward(m, img, txt, pooled, 750.0)
    finally:
        O.use_reference_b1(False)
    m.close()
    _check(got, ref, f"full-depth flux1 forward (reference b1 kernel={used})")


@pytest.mark.parametrize("kind", ["double", "single"])
def test_flux1_block_at_step_sequence(gpu, kind):
    """One block at L = 4608 (the 1024^2 step), every B1_0 linear through the
    reference's own kernel in the oracle."""
    import torch
    m = bb.Dit(bb.PRESET_FLUX1, 4096, 512, 64, 64, depth=1, depth_single=1, seed=41)
    rng = np.random.default_rng(42)
    hidden = rng.standard_normal((m.L, H)).astype(np.float32)
    vec = rng.standard_normal(H).astype(np.float32)
    hd, vd = torch.from_numpy(hidden).cuda(), torch.from_numpy(vec).cuda()
    m.set_state(hd, vd)
    (m.double_block if kind == "double" else m.single_block)(0)
    out = torch.empty_like(hd)
    m.get_state(out)
    got = out.cpu().numpy()
    assert bb.device_error() == 0
    mods, _ = O.modulations(m, vec)
    c, s = O.rope_cos_sin(m.rope_ids(), m.axes, m.theta)
    used = O.use_reference_b1(True, nthreads=THREADS)
    try:
        if kind == "double":
            ref = O.double_block(m, 0, hidden, mods["double"][0][0], mods["double"][0][1], c, s)
        else:
            ref = O.single_block(m, 0, hidden, mods["single"][0], c, s)
    finally:
        O.use_reference_b1(False)
    m.close()
    _check(got, ref, f"flux1 {kind} block at L=4608 (reference b1 kernel={used})")


@pytest.fixture(params=["pair", "single", "v2"])
def attn_form(request, monkeypatch):
    monkeypatch.setenv("BONSAI_ATTN", request.param)
    return request.param


@pytest.mark.parametrize("L", [4608, 16896])
def test_attention_long_sequence_with_redo(gpu, attn_form, L):
    """24 heads x 128 at the step's sequences.  Head 5 gets two planted key
    blocks whose logits exceed the running maximum by ~16 and ~32 (natural
    units) for half of the queries and by up to ~10 / ~20 for the others:
    those blocks' softmax row sums exceed 2^15 and are redone."""
    import torch
    nh, hd = 24, 128
    g = torch.Generator(device="cuda").manual_seed(L)
    q, k, v = (torch.randn(nh, L, hd, device="cuda", generator=g) for _ in range(3))
    hp = 5
    q[hp, : L // 2, 0] += 6.0
    b1, b2 = (L // 2 // 64) * 64, (3 * L // 4 // 64) * 64
    k[hp, b1:b1 + 64, 0] = 30.0
    k[hp, b2:b2 + 64, 0] = 60.0
    q, k, v = q.half(), k.half(), v.half()
    out = torch.empty(L, nh * hd, device="cuda", dtype=torch.float16)
    scale = hd ** -0.5
    bb.check(bb.lib().bonsai_joint_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), nh, L, hd,
                                             scale, out.data_ptr(), out.stride(0), bb.stream_ptr()),
             "attention")
    torch.cuda.synchronize()
    assert bb.device_error() == 0
    for h in (0, hp, 17, 23):
        s = (q[h].float() @ k[h].float().t()) * scale
        ref = torch.softmax(s, -1) @ v[h].float()
        del s
        got = out[:, h * hd:(h + 1) * hd].float()
        _check(got.cpu().numpy(), ref.cpu().numpy(), f"attention L={L} head {h} ({attn_form})")


@pytest.mark.parametrize("L,nh,split", [(1000, 2, 2), (1000, 2, 3), (4608, 3, 2), (16896, 3, 2),
                                        (333, 1, 4)])
def test_attention_key_split(gpu, attn_form, monkeypatch, L, nh, split):
    """The key-range split (BONSAI_ATTN_SPLIT forces it; the launcher picks
    it for the 2048^2 head split on 8 GPUs): each range's normalised partial
    and log2 exponential sum, merged, against torch fp32 -- ragged last
    ranges and ragged last key blocks included."""
    import torch
    monkeypatch.setenv("BONSAI_ATTN_SPLIT", str(split))
    hd = 128
    g = torch.Generator(device="cuda").manual_seed(L + split)
    q, k, v = (torch.randn(nh, L, hd, device="cuda", generator=g) for _ in range(3))
    q[0, : L // 2, 0] += 6.0          # a planted block (redo path) inside one range
    b1 = (L // 3 // 64) * 64
    k[0, b1:b1 + 64, 0] = 30.0
    q, k, v = q.half(), k.half(), v.half()
    out = torch.full((L, nh * hd), float("nan"), device="cuda", dtype=torch.float16)
    scale = hd ** -0.5
    bb.check(bb.lib().bonsai_joint_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), nh, L, hd,
                                             scale, out.data_ptr(), out.stride(0), bb.stream_ptr()),
             "attention")
    torch.cuda.synchronize()
    assert bb.device_error() == 0
    for h in range(nh):
        s = (q[h].float() @ k[h].float().t()) * scale
        ref = torch.softmax(s, -1) @ v[h].float()
        del s
        got = out[:, h * hd:(h + 1) * hd].float()
        _check(got.cpu().numpy(), ref.cpu().numpy(), f"attention split={split} L={L} head {h} ({attn_form})")
