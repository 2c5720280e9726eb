"""The bounded device waits that replace the reference's abort()
(src/b1_0_kernel.h:193-198): a wait that runs out records an error code the
host reads with bonsai_device_error(), the kernel returns, and the context
stays usable.

The wait is made to run out without faulting anything: the test hook
bonsai_debug_stall_next_gemm makes the next B1_0 GEMM launch run with its load
warp idle, so the barriers the other roles wait on are never completed; no
copy is issued and no MMA starts, so nothing is in flight when they give up
after the 2 s limit.
"""
import numpy as np
import pytest

import bonsai_b200 as bb

pytestmark = pytest.mark.gpu

DEV_ERR_TIMEOUTS = (1, 2, 3, 4)  # TMA, MMA, producer (expansion), epilogue


def _ref(x16, packed, N, K):
    w = bb.dequant_b1(packed, N, K).astype(np.float64)
    return x16.astype(np.float64) @ w.T


def test_gemm_wait_timeout_is_reported_and_the_context_recovers(gpu):
    import torch
    L = bb.lib()
    assert bb.device_error() == 0
    rng = np.random.default_rng(9)
    T, K, N = 200, 512, 256
    packed = bb.random_b1_packed(N, K, rng)
    w = bb.B1Weight(packed, N, K)
    x = rng.standard_normal((T, K)).astype(np.float16)
    x16 = torch.from_numpy(x).cuda()
    out = torch.full((T, N), float("nan"), device="cuda")
    try:
        bb.check(L.bonsai_debug_stall_next_gemm(), "bonsai_debug_stall_next_gemm")
        bb.b1_gemm(x16, w, bb.BONSAI_EPI_F32, out)  # the launch itself succeeds
        code = bb.device_error()                     # synchronises; reads and clears
        assert code in DEV_ERR_TIMEOUTS, code
        assert bb.device_error() == 0                # the word was cleared
        assert torch.isnan(out).all()                # the stalled launch wrote nothing
        # the context is intact: the next launch of the same kernel is correct
        bb.b1_gemm(x16, w, bb.BONSAI_EPI_F32, out)
        torch.cuda.synchronize()
        assert bb.device_error() == 0
        got = out.cpu().numpy().astype(np.float64)
        ref = _ref(x, packed, N, K)
        err = np.abs(got - ref).max() / np.sqrt(np.mean(ref ** 2))
        assert err < 1e-4, err
    finally:
        w.free()
