"""B1_0 GEMM on the GPU vs exact references.

Reference semantics: b1_linear_f32_f32 (src/b1_0_kernel.h:37-288),
out[t][r] = sum_blk scale[r][blk] * sum_i (bit ? +x : -x).
The kernel rounds activations to f16 and accumulates in f32, so it is
compared (1) against an f64 dequantised product of the SAME f16-rounded
activations (tight: only summation order differs) and (2) against the f32
reference semantics with the acceptance bar of the reference's GPU-vs-CPU
tests (cos >= 0.9999, max-abs <= 1e-2 * RMS; tests/c_ops/test_webgpu_ops.cpp:129).
"""
import numpy as np
import pytest

import bonsai_b200 as bb

pytestmark = pytest.mark.gpu

SWEEP_M = [1280, 4352, 8704]
SWEEP_KN = [(3072, 9216), (3072, 3072), (3072, 12288), (12288, 3072), (3072, 21504), (15360, 3072)]


@pytest.fixture(params=["single", "pair"])
def kernel(request, monkeypatch):
    """Run the test with each GEMM kernel forced (the launcher otherwise
    picks by estimated time): 'single' = one CTA per 128x128 tile with the
    weights in TMEM, 'pair' = a two-SM cluster per 256x256 tile."""
    monkeypatch.setenv("BONSAI_B1_KERNEL", request.param)
    return request.param


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def _case(M, K, N, seed):
    rng = np.random.default_rng(seed)
    packed = bb.random_b1_packed(N, K, rng)
    x = rng.standard_normal((M, K)).astype(np.float32)
    return packed, x


@pytest.mark.parametrize("M,K,N", [
    (1, 64, 32),        # the reference's own unit-test shape (tests/c_ops/test_b1_linear.py:43-45)
    (7, 96, 40),        # ragged: K % 64 == 32, N % 128 != 0, M < 32
    (128, 128, 128),
    (300, 3072, 200),
    (129, 256, 384),
    (256, 512, 1000),
])
def test_b1_linear_f32_small(gpu, kernel, M, K, N):
    import torch
    packed, x = _case(M, K, N, 1000 + M + K + N)
    w = bb.B1Weight(packed, N, K)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    bb.b1_linear_f32(xd, w, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    wd = bb.dequant_b1(packed, N, K).astype(np.float64)
    ref32 = x.astype(np.float64) @ wd.T
    if M == 1:  # one token: the f32 matrix-vector kernel (no f16 rounding of x)
        assert np.max(np.abs(got - ref32)) <= 1e-5 * np.sqrt(np.mean(ref32 ** 2)) + 1e-7
    else:
        x16 = x.astype(np.float16).astype(np.float64)
        exact16 = x16 @ wd.T
        rms = np.sqrt(np.mean(exact16 ** 2)) + 1e-30
        assert np.max(np.abs(got - exact16)) <= 1e-4 * rms + 1e-6
    assert _cos(got, ref32) >= 0.9999
    assert np.max(np.abs(got - ref32)) <= 1e-2 * np.sqrt(np.mean(ref32 ** 2))


@pytest.mark.parametrize("K,N", [(32, 1), (96, 200), (3072, 3072), (3072, 9000), (8192, 300),
                                 (8224, 130)])
def test_b1_linear_f32_one_token(gpu, K, N):
    """A single token takes the B1_0 matrix-vector kernel (f32 activations,
    sign-sum tables; in_dim <= 8192) -- the engine's stacked per-block
    modulation linear is this shape with N = 1,050,624 -- and beyond 8192
    inputs the tensor-core GEMM (f16 activations)."""
    import torch
    packed, x = _case(1, K, N, 77 + K + N)
    w = bb.B1Weight(packed, N, K)
    xd = torch.from_numpy(x).cuda()
    out = torch.full((1, N), float("nan"), device="cuda", dtype=torch.float32)
    bb.b1_linear_f32(xd, w, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    wd = bb.dequant_b1(packed, N, K).astype(np.float64)
    xr = x.astype(np.float64) if K <= 8192 else x.astype(np.float16).astype(np.float64)
    ref = xr @ wd.T
    tol = 1e-5 if K <= 8192 else 1e-4
    assert np.max(np.abs(got - ref)) <= tol * np.sqrt(np.mean(ref ** 2)) + 1e-7
    w.free()


def test_b1_zero_tokens_is_noop(gpu, kernel):
    import torch
    packed, _ = _case(1, 64, 32, 5)
    w = bb.B1Weight(packed, 32, 64)
    x = torch.zeros(0, 64, device="cuda")
    out = torch.zeros(0, 32, device="cuda")
    bb.b1_linear_f32(x, w, out)
    torch.cuda.synchronize()


@pytest.mark.parametrize("K,N", SWEEP_KN)
def test_b1_gemm_sweep_shapes(gpu, kernel, K, N):
    """Every (K,N) of the BASELINE GEMM sweep at every M, vs a torch fp32
    product of the dequantised weights and the same f16 activations."""
    import torch
    rng = np.random.default_rng(K * 7 + N)
    packed = bb.random_b1_packed(N, K, rng)
    w = bb.B1Weight(packed, N, K)
    wd = torch.from_numpy(bb.dequant_b1(packed, N, K)).cuda()
    for M in SWEEP_M:
        g = torch.Generator(device="cuda").manual_seed(M)
        x16 = torch.randn(M, K, device="cuda", generator=g).half()
        out = torch.empty(M, N, device="cuda", dtype=torch.float32)
        bb.b1_gemm(x16, w, bb.BONSAI_EPI_F32, out)
        ref = x16.float() @ wd.t()
        torch.cuda.synchronize()
        rms = ref.pow(2).mean().sqrt().item()
        err = (out - ref).abs().max().item()
        cos = torch.nn.functional.cosine_similarity(out.flatten().double(), ref.flatten().double(), dim=0).item()
        assert cos >= 0.99999, (M, K, N, cos)
        assert err <= 1e-3 * rms, (M, K, N, err, rms)


def test_b1_gemm_epilogues(gpu, kernel):
    import torch
    M, K, N = 300, 1024, 512
    rng = np.random.default_rng(77)
    packed = bb.random_b1_packed(N, K, rng)
    w = bb.B1Weight(packed, N, K)
    wd = torch.from_numpy(bb.dequant_b1(packed, N, K)).cuda()
    x16 = torch.randn(M, K, device="cuda").half()
    ref = x16.float() @ wd.t()
    # f16 store
    o16 = torch.empty(M, N, device="cuda", dtype=torch.float16)
    bb.b1_gemm(x16, w, bb.BONSAI_EPI_F16, o16)
    torch.testing.assert_close(o16.float(), ref.half().float(), rtol=2e-3, atol=2e-3)
    # GELU-tanh
    og = torch.empty(M, N, device="cuda", dtype=torch.float16)
    bb.b1_gemm(x16, w, bb.BONSAI_EPI_GELU, og)
    torch.testing.assert_close(og.float(), torch.nn.functional.gelu(ref, approximate="tanh"),
                               rtol=4e-3, atol=4e-3)
    # gate-residual: h += g * acc
    h0 = torch.randn(M, N, device="cuda")
    gate = torch.randn(N, device="cuda")
    h = h0.clone()
    bb.b1_gemm(x16, w, bb.BONSAI_EPI_RESID, h, gate=gate)
    torch.testing.assert_close(h, h0 + gate[None, :] * ref, rtol=1e-4, atol=1e-4)
    # SwiGLU on [gate; value] halves (ggml_swiglu: silu(first half) * second half)
    ws = bb.B1Weight(packed, N, K, swiglu_from=0)
    osw = torch.empty(M, N // 2, device="cuda", dtype=torch.float16)
    bb.b1_gemm(x16, ws, bb.BONSAI_EPI_SWIGLU, osw)
    g_, v_ = ref[:, : N // 2], ref[:, N // 2:]
    torch.testing.assert_close(osw.float(), torch.nn.functional.silu(g_) * v_, rtol=4e-3, atol=4e-3)
    torch.cuda.synchronize()


@pytest.mark.parametrize("M,K,N,split", [(300, 1024, 512, 2), (2112, 3072, 3072, 2),
                                         (77, 96 * 32, 384, 3), (513, 9 * 64, 256, 4)])
def test_b1_gemm_resid_k_split(gpu, monkeypatch, M, K, N, split):
    """The two-SM kernel with K split into parts whose gate-residual
    epilogues add atomically (the partitioned step's residual GEMMs at 8
    GPUs: M = 2112, K = 3072, N = 3072); forced by BONSAI_B1_SPLITK, ragged
    token counts and k-block counts that do not divide by the split."""
    import torch
    monkeypatch.setenv("BONSAI_B1_KERNEL", "pair")
    rng = np.random.default_rng(M + K + N)
    packed = bb.random_b1_packed(N, K, rng)
    w = bb.B1Weight(packed, N, K)
    wd = torch.from_numpy(bb.dequant_b1(packed, N, K)).cuda()
    x16 = torch.randn(M, K, device="cuda").half()
    ref = x16.float() @ wd.t()
    h0 = torch.randn(M, N, device="cuda")
    gate = torch.randn(N, device="cuda")
    h_whole = h0.clone()
    bb.b1_gemm(x16, w, bb.BONSAI_EPI_RESID, h_whole, gate=gate)
    monkeypatch.setenv("BONSAI_B1_SPLITK", str(split))
    h_split = h0.clone()
    bb.b1_gemm(x16, w, bb.BONSAI_EPI_RESID, h_split, gate=gate)
    torch.cuda.synchronize()
    assert bb.device_error() == 0
    expect = h0 + gate[None, :] * ref
    torch.testing.assert_close(h_split, expect, rtol=1e-4, atol=1e-4)
    # the two parts' f32 partial sums are rounded separately: equal to the
    # unsplit launch up to f32 accumulation order
    torch.testing.assert_close(h_split, h_whole, rtol=1e-4, atol=1e-4)
    w.free()


def test_b1_linear_f32_two_streams_interleaved(gpu):
    """The drop-in linear's f16 scratch is per (thread, device, stream): calls
    of growing size issued alternately on two streams from one host thread,
    with nothing synchronised between them, give the results of the same
    calls run one after another on one stream (same kernels, same bits)."""
    import torch
    rng = np.random.default_rng(77)
    K, N = 3072, 1024
    w = bb.B1Weight(bb.random_b1_packed(N, K, rng), N, K)
    sizes = [96, 640, 1500, 2900, 4100, 6200]  # every call grows its stream's scratch
    acts = [torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32)).cuda() for T in sizes]
    outs = [torch.full((T, N), float("nan"), device="cuda") for T in sizes]
    refs = [torch.empty(T, N, device="cuda") for T in sizes]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for i, (a, o) in enumerate(zip(acts, outs)):
        bb.b1_linear_f32(a, w, o, stream=streams[i % 2])
    torch.cuda.synchronize()
    for a, r in zip(acts, refs):
        bb.b1_linear_f32(a, w, r)
    torch.cuda.synchronize()
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
    w.free()
