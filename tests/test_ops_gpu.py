"""Attention and pointwise kernels on the GPU vs the CPU oracle / golden data."""
from pathlib import Path

import numpy as np
import pytest

import bonsai_b200 as bb
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
U16 = None


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def _assert_block_tol(got, ref, what):
    """Acceptance bar of the reference's GPU-vs-CPU tests: cos >= 0.9999 and
    max-abs <= 1e-2 * RMS(ref) (tests/c_ops/test_webgpu_diffuser_ops.cpp:310)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref ** 2))
    c = _cos(got, ref)
    err = np.max(np.abs(got - ref))
    assert c >= 0.9999 and err <= 1e-2 * rms, f"{what}: cos={c:.6f} maxabs={err:.3e} rms={rms:.3e}"


@pytest.fixture(params=["pair", "single", "v2"])
def attn_form(request, monkeypatch):
    """Every form of the attention kernel: CTA pair (the default), one CTA
    (BONSAI_ATTN=single), and the CTA pair with 128-key blocks and two
    key-half softmaxes (BONSAI_ATTN=v2)."""
    monkeypatch.setenv("BONSAI_ATTN", request.param)
    return request.param


def _attn_gpu(q, k, v, scale):
    """q, k, v f32 [seq][H][128] numpy -> GPU output f32 [seq][H*128]."""
    import torch
    seq, H, hd = q.shape
    to_heads = lambda a: torch.from_numpy(np.ascontiguousarray(a.transpose(1, 0, 2))).cuda().half().contiguous()
    qd, kd, vd = to_heads(q), to_heads(k), to_heads(v)
    out = torch.zeros(seq, H * hd, device="cuda", dtype=torch.float16)
    bb.check(bb.lib().bonsai_joint_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), H, seq,
                                             hd, scale, out.data_ptr(), out.stride(0),
                                             bb.stream_ptr()), "attention")
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("seq,H", [(128, 1), (200, 2), (333, 3), (1280, 2), (77, 1), (64, 1), (65, 2),
                                   (1, 1), (191, 1), (513, 2), (1100, 1)])
def test_attention_vs_oracle(gpu, attn_form, seq, H):
    rng = np.random.default_rng(seq * 10 + H)
    q, k, v = (rng.standard_normal((seq, H, 128)).astype(np.float32) for _ in range(3))
    scale = 1.0 / np.sqrt(128.0)
    got = _attn_gpu(q, k, v, scale)
    ref = O.attention(q, k, v, scale)
    _assert_block_tol(got, ref, f"attention seq={seq} H={H}")


def test_attention_default_is_the_pair_form(gpu, monkeypatch):
    """On a B200 the default launch is the CTA-pair kernel: its results differ
    in the last bits from the one-CTA form's (4/16 vs 2/16 of the
    exponentials on the polynomial) while both meet the tolerance."""
    rng = np.random.default_rng(11)
    seq, H = 700, 2
    q, k, v = (rng.standard_normal((seq, H, 128)).astype(np.float32) for _ in range(3))
    scale = 1.0 / np.sqrt(128.0)
    monkeypatch.delenv("BONSAI_ATTN", raising=False)
    pair = _attn_gpu(q, k, v, scale)
    monkeypatch.setenv("BONSAI_ATTN", "single")
    single = _attn_gpu(q, k, v, scale)
    ref = O.attention(q, k, v, scale)
    _assert_block_tol(pair, ref, "attention default form")
    _assert_block_tol(single, ref, "attention single form")
    assert not np.array_equal(pair, single)


def test_attention_large_logits_rescale(gpu, attn_form):
    """Rows whose max grows across key tiles exercise the lazy O rescale."""
    rng = np.random.default_rng(5)
    seq, H = 640, 2
    q = rng.standard_normal((seq, H, 128)).astype(np.float32) * 3
    k = rng.standard_normal((seq, H, 128)).astype(np.float32) * 3
    k[seq // 2:] *= 2.5  # later key tiles carry much larger scores
    v = rng.standard_normal((seq, H, 128)).astype(np.float32)
    scale = 1.0 / np.sqrt(128.0)
    _assert_block_tol(_attn_gpu(q, k, v, scale), O.attention(q, k, v, scale), "attention rescale")


def test_attention_config2_full_size(gpu, attn_form):
    """BASELINE config 2 shape (H=24, D=128, L=4352 = 256 text + 4096 image),
    against a torch fp32 softmax attention on the same f16 inputs."""
    import torch
    H, L = 24, 4352
    g = torch.Generator(device="cuda").manual_seed(2)
    q, k, v = (torch.randn(H, L, 128, device="cuda", generator=g).half() for _ in range(3))
    out = torch.empty(L, H * 128, device="cuda", dtype=torch.float16)
    scale = 1.0 / 128 ** 0.5
    bb.check(bb.lib().bonsai_joint_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), H, L, 128,
                                             scale, out.data_ptr(), out.stride(0), bb.stream_ptr()))
    worst_cos, worst_err = 1.0, 0.0
    for h in range(0, H, 6):
        s = (q[h].float() @ k[h].float().t()) * scale
        ref = torch.softmax(s, -1) @ v[h].float()
        got = out[:, h * 128:(h + 1) * 128].float()
        rms = ref.pow(2).mean().sqrt().item()
        worst_err = max(worst_err, (got - ref).abs().max().item() / rms)
        worst_cos = min(worst_cos, torch.nn.functional.cosine_similarity(
            got.flatten().double(), ref.flatten().double(), dim=0).item())
    assert worst_cos >= 0.9999 and worst_err <= 1e-2, (worst_cos, worst_err)


def test_qk_norm_rope_vs_oracle(gpu):
    import torch
    rng = np.random.default_rng(11)
    H, seq, split = 3, 150, 40
    x = rng.standard_normal((H, seq, 128)).astype(np.float32) * 2
    w_lo = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    w_hi = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    ids = np.zeros((seq, 3), np.float32)
    ids[split:, 1] = np.arange(seq - split) // 10
    ids[split:, 2] = np.arange(seq - split) % 10
    c, s = O.rope_cos_sin(ids, [16, 56, 56], 10000.0)
    x16 = x.astype(np.float16)
    ref = O.qk_norm_rope_heads(x16.astype(np.float32), w_lo, w_hi, split, c, s)
    xd = torch.from_numpy(x16).cuda()
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    wl, wh, cd, sd = T(w_lo), T(w_hi), T(c), T(s)
    bb.check(bb.lib().bonsai_qk_norm_rope(xd.data_ptr(), H, seq, 128, wl.data_ptr(), wh.data_ptr(),
                                          split, 1e-6, cd.data_ptr(), sd.data_ptr(), bb.stream_ptr()))
    torch.cuda.synchronize()
    got = xd.float().cpu().numpy()
    assert np.max(np.abs(got - ref)) <= 4e-3 * np.max(np.abs(ref))
    _assert_block_tol(got, ref, "qk_norm_rope")


def test_ln_modulate_vs_oracle(gpu):
    import torch
    rng = np.random.default_rng(12)
    for rows, dim in [(37, 3072), (5, 100), (9, 6144)]:
        x = (rng.standard_normal((rows, dim)) * 4 + 2).astype(np.float32)
        sh = rng.standard_normal(dim).astype(np.float32)
        sc = rng.standard_normal(dim).astype(np.float32)
        ref = O.ln_modulate(x, sh, sc)
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        xd, shd, scd = T(x), T(sh), T(sc)
        y16 = torch.empty(rows, dim, device="cuda", dtype=torch.float16)
        bb.check(bb.lib().bonsai_ln_modulate(xd.data_ptr(), rows, dim, shd.data_ptr(), scd.data_ptr(),
                                             1e-6, y16.data_ptr(), dim, bb.stream_ptr()))
        y32 = torch.empty(rows, dim, device="cuda")
        bb.check(bb.lib().bonsai_ln_modulate_f32(xd.data_ptr(), rows, dim, shd.data_ptr(),
                                                 scd.data_ptr(), 1e-6, y32.data_ptr(), bb.stream_ptr()))
        torch.cuda.synchronize()
        np.testing.assert_allclose(y32.cpu().numpy(), ref, rtol=1e-4, atol=2e-4)
        np.testing.assert_allclose(y16.float().cpu().numpy(), ref, rtol=2e-3, atol=4e-3)


def test_rope_2d_and_tables_vs_golden(gpu):
    """rope_2d_f32 drop-in and the device RoPE tables against the reference's
    own outputs (golden rope.npz, generated by the reference code)."""
    import torch
    g = np.load(GOLD / "rope.npz")
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    for preset in ("klein", "flux1"):
        x = g[f"{preset}_x"]
        seq, H, hd = x.shape
        out = torch.empty(seq, H, hd, device="cuda")
        xd, cd, sd = T(x), T(g[f"{preset}_cos"]), T(g[f"{preset}_sin"])
        bb.check(bb.lib().bonsai_rope_2d_f32(xd.data_ptr(), cd.data_ptr(), sd.data_ptr(), hd, H,
                                             seq, out.data_ptr(), bb.stream_ptr()))
        axes = g[f"{preset}_axes"].astype(np.int32)
        ids = T(g[f"{preset}_ids"])
        cc = torch.empty(seq, hd // 2, device="cuda")
        ss = torch.empty(seq, hd // 2, device="cuda")
        bb.check(bb.lib().bonsai_rope_tables(ids.data_ptr(), seq, len(axes), axes.ctypes.data,
                                             float(g[f"{preset}_theta"]), cc.data_ptr(), ss.data_ptr(),
                                             bb.stream_ptr()))
        torch.cuda.synchronize()
        assert np.max(np.abs(out.cpu().numpy() - g[f"{preset}_rot"])) < 1e-5
        np.testing.assert_allclose(cc.cpu().numpy(), g[f"{preset}_cos"], atol=1e-5)
        np.testing.assert_allclose(ss.cpu().numpy(), g[f"{preset}_sin"], atol=1e-5)


def test_rms_norm_vs_oracle(gpu):
    import torch
    rng = np.random.default_rng(13)
    x = rng.standard_normal((300, 128)).astype(np.float32) * 3
    w = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    xd, wd = T(x), T(w)
    y = torch.empty_like(xd)
    bb.check(bb.lib().bonsai_rms_norm_f32(xd.data_ptr(), wd.data_ptr(), 300, 128, 1e-6, y.data_ptr(),
                                          bb.stream_ptr()))
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), O.rms_norm(x, w), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("T,K,N", [
    (512, 4096, 3072),   # context_embedder at 1024^2: split-K over 4 slices
    (4096, 3072, 64),    # proj_out (flux1): narrow output, split-K over 8 slices
    (4096, 64, 3072),    # x_embedder (flux1): K = 64, no split
    (7, 40, 33),         # ragged, K % 8 != 0
    (300, 1000, 130),    # ragged split-K slices
    (1, 3072, 1000),     # one token (GEMV path)
])
def test_linear_f32_edges(gpu, T, K, N):
    """The f32 edge projections (ggml_mul_mat f32, src/diffuser_graph.cpp:283-286,
    :544-556) against float64 numpy, including every split-K slice."""
    import torch
    rng = np.random.default_rng(T * 7 + K + N)
    x = rng.standard_normal((T, K)).astype(np.float32)
    W = (0.05 * rng.standard_normal((N, K))).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    out = torch.empty(T, N, device="cuda")
    bb.linear_f32(torch.from_numpy(x).cuda(), torch.from_numpy(W).cuda(), torch.from_numpy(b).cuda(), out)
    ref = x.astype(np.float64) @ W.astype(np.float64).T + b
    got = out.cpu().numpy()
    err = np.max(np.abs(got - ref)) / (np.sqrt(np.mean(ref ** 2)) + 1e-30)
    assert err <= 2e-6 * np.sqrt(K), (T, K, N, err)
