"""The head/token split of one image, every rank emulated on ONE GPU.

`world` partitioned models (bonsai_dit_set_partition(rank, world)) run the
phases of each block in lock step; the two exchanges that NCCL performs on a
real multi-GPU run (all-gather of token rows, all-to-all of attention-head
columns; bonsai_b200.headsplit) are done here with device copies between the
models' buffers -- or, fused, by the kernels themselves: each model is given
the other models' xm / cat as its peers (bonsai_dit_set_peers), so phase 0
stores its rows into every model's xm and phase 1's attention stores every
row into its owner's cat, the path a multi-GPU run takes over peer-mapped
memory; in the QKV scatter form each model is also given the other models'
q/k/v buffers, and phase 0's Q/K/V GEMM over its own rows stores every head
into its owner's buffer.  Every rank's prediction must equal the
unpartitioned forward.  World 3 and 8 give 8 and 3 heads per rank, so the
Q/K/V weight-tile selections have even and odd tile counts; each GEMM kernel
is forced in turn.
"""
import numpy as np
import pytest

import bonsai_b200 as bb

pytestmark = pytest.mark.gpu

IMG_H, IMG_W, TXT = 16, 16, 32   # L = 288 tokens: divisible by 2, 3, 4 and 8
H = 3072


def _inputs(m, seed=3):
    import torch
    rng = np.random.default_rng(seed)
    img = torch.from_numpy(rng.standard_normal((m.img, m.in_ch)).astype(np.float32)).cuda()
    txt = torch.from_numpy(rng.standard_normal((m.txt, m.ctx_dim)).astype(np.float32)).cuda()
    pooled = torch.from_numpy(rng.standard_normal(m.pooled).astype(np.float32)).cuda()
    return img, txt, pooled


def _emulated_forward(preset, world, img, txt, pooled, t, fused=False, scatter=False):
    import torch
    ms = [bb.Dit(preset, IMG_H * IMG_W, TXT, IMG_H, IMG_W, depth=1, depth_single=1, seed=5)
          for _ in range(world)]
    try:
        for r, m in enumerate(ms):
            m.set_partition(r, world)
        L = ms[0].L
        C = H + ms[0].mlp
        rows, hc = L // world, H // world
        xm = [m.buffer("xm", torch.float16, (L, H)) for m in ms]
        cat = [m.buffer("cat", torch.float16, (L, C)) for m in ms]
        hidden = [m.buffer("hidden", torch.float32, (L, H)) for m in ms]
        if fused:
            for m in ms:
                m.set_peers([b.data_ptr() for b in xm], [b.data_ptr() for b in cat])
        if scatter:  # phase 0's Q/K/V GEMM stores each head into its owner's qkv
            qkv = [m.buffer("qkv", torch.float16, (3 * 24 * L * 128,)) for m in ms]
            for m in ms:
                m.set_qkv_peers([b.data_ptr() for b in qkv])

        def gather_rows(bufs):
            for r in range(world):
                for d in range(world):
                    if d != r:
                        bufs[d][r * rows:(r + 1) * rows].copy_(bufs[r][r * rows:(r + 1) * rows])

        def heads_to_rows():
            mine = [cat[s][:, s * hc:(s + 1) * hc].clone() for s in range(world)]
            for d in range(world):
                for s in range(world):
                    cat[d][d * rows:(d + 1) * rows, s * hc:(s + 1) * hc].copy_(
                        mine[s][d * rows:(d + 1) * rows])

        for m in ms:
            m.begin(img, txt, pooled, t)
        for kind, n in ((0, ms[0].depth), (1, ms[0].depth_single)):
            for i in range(n):
                for m in ms:
                    m.phase(kind, i, 0)
                if not fused:
                    gather_rows(xm)
                for m in ms:
                    m.phase(kind, i, 1)
                if not fused:
                    heads_to_rows()
                for m in ms:
                    m.phase(kind, i, 2)
        gather_rows(hidden)
        outs = []
        for m in ms:
            o = torch.empty(m.img, m.in_ch, device="cuda")
            m.end(o)
            outs.append(o)
        torch.cuda.synchronize()
        return outs
    finally:
        for m in ms:
            m.close()


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("kernel", ["single", "pair"])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_headsplit_emulated_matches_forward(gpu, monkeypatch, world, kernel, fused):
    import torch
    monkeypatch.setenv("BONSAI_B1_KERNEL", kernel)
    preset = bb.PRESET_FLUX1
    ref_m = bb.Dit(preset, IMG_H * IMG_W, TXT, IMG_H, IMG_W, depth=1, depth_single=1, seed=5)
    try:
        img, txt, pooled = _inputs(ref_m)
        ref = torch.empty(ref_m.img, ref_m.in_ch, device="cuda")
        ref_m.forward(img, txt, pooled, 600.0, ref)
        torch.cuda.synchronize()
    finally:
        ref_m.close()
    outs = _emulated_forward(preset, world, img, txt, pooled, 600.0, fused=fused)
    r = ref.double().flatten()
    for rank, o in enumerate(outs):
        g = o.double().flatten()
        cos = float(g @ r / (g.norm() * r.norm()))
        rel = float((g - r).abs().max() / r.pow(2).mean().sqrt())
        assert cos >= 0.99999 and rel <= 1e-3, (world, kernel, fused, rank, cos, rel)
    assert bb.device_error() == 0


@pytest.mark.parametrize("fused", [False, True])
def test_headsplit_emulated_with_key_split(gpu, monkeypatch, fused):
    """World 8 (3 heads per rank, the layout whose attention the launcher
    splits by key range at 2048^2) with the key split forced on at this small
    size: the merged partial outputs reach every rank's cat, directly or
    routed to the row owners (fused).  The split changes the attention's
    rounding (each range's P is rounded against its own maximum), so the bar
    is the attention's parity bar, not the bit-level agreement of the
    unsplit partition."""
    import torch
    preset = bb.PRESET_FLUX1
    ref_m = bb.Dit(preset, IMG_H * IMG_W, TXT, IMG_H, IMG_W, depth=1, depth_single=1, seed=5)
    try:
        img, txt, pooled = _inputs(ref_m)
        ref = torch.empty(ref_m.img, ref_m.in_ch, device="cuda")
        ref_m.forward(img, txt, pooled, 600.0, ref)
        torch.cuda.synchronize()
    finally:
        ref_m.close()
    monkeypatch.setenv("BONSAI_ATTN_SPLIT", "3")  # 5 key blocks -> ranges of 2, 2 and 1
    outs = _emulated_forward(preset, 8, img, txt, pooled, 600.0, fused=fused)
    r = ref.double().flatten()
    for rank, o in enumerate(outs):
        g = o.double().flatten()
        cos = float(g @ r / (g.norm() * r.norm()))
        rel = float((g - r).abs().max() / r.pow(2).mean().sqrt())
        assert cos >= 0.9999 and rel <= 1e-2, (fused, rank, cos, rel)
    assert bb.device_error() == 0


@pytest.mark.parametrize("kernel", ["single", "pair"])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_headsplit_emulated_qkv_scatter(gpu, monkeypatch, world, kernel):
    """The QKV scatter form of the fused exchanges (bonsai_dit_set_qkv_peers)
    equals the unpartitioned forward."""
    import torch
    monkeypatch.setenv("BONSAI_B1_KERNEL", kernel)
    preset = bb.PRESET_FLUX1
    ref_m = bb.Dit(preset, IMG_H * IMG_W, TXT, IMG_H, IMG_W, depth=1, depth_single=1, seed=5)
    try:
        img, txt, pooled = _inputs(ref_m)
        ref = torch.empty(ref_m.img, ref_m.in_ch, device="cuda")
        ref_m.forward(img, txt, pooled, 600.0, ref)
        torch.cuda.synchronize()
    finally:
        ref_m.close()
    outs = _emulated_forward(preset, world, img, txt, pooled, 600.0, fused=True, scatter=True)
    r = ref.double().flatten()
    for rank, o in enumerate(outs):
        g = o.double().flatten()
        cos = float(g @ r / (g.norm() * r.norm()))
        rel = float((g - r).abs().max() / r.pow(2).mean().sqrt())
        assert cos >= 0.99999 and rel <= 1e-3, (world, kernel, rank, cos, rel)
    assert bb.device_error() == 0


def test_qkv_scatter_needs_fused_peers(gpu):
    m = bb.Dit(bb.PRESET_FLUX1, IMG_H * IMG_W, TXT, IMG_H, IMG_W, depth=1, depth_single=1, seed=5)
    try:
        m.set_partition(0, 2)
        with pytest.raises(bb.BonsaiError, match="set the xm / cat peers first"):
            m.set_qkv_peers([1 << 20, 2 << 20])
    finally:
        m.close()
