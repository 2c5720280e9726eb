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


def test_peer_barrier_timeout_is_reported_and_the_context_recovers(gpu):
    """The peer flag barrier of the split step (bonsai_dit_barrier) waits for
    every rank's store into this GPU's flags.  Here the model is partitioned
    as rank 0 of 2 and "rank 1's flags" is a plain device buffer: rank 1 never
    runs, nothing sets its arrival word, and the wait gives up after its 2 s
    limit with DEV_ERR_TIMEOUT_BARRIER (6).  The barrier's own store into the
    stand-in buffer is checked, and the context stays usable."""
    import ctypes
    import torch
    L = bb.lib()
    assert bb.device_error() == 0
    m = bb.Dit(bb.PRESET_FLUX1, 64, 32, 8, 8, depth=1, depth_single=1, seed=5)
    try:
        m.set_partition(0, 2)
        own = m.buffer("flags", torch.int32, (64,))
        fake_peer = torch.zeros(64, dtype=torch.int32, device="cuda")
        ptrs = (ctypes.c_void_p * 2)(own.data_ptr(), fake_peer.data_ptr())
        bb.check(L.bonsai_dit_set_flag_peers(m.handle, ptrs, 2), "set_flag_peers")
        m.barrier()
        code = bb.device_error()          # synchronises; reads and clears
        assert code == 6, code
        assert bb.device_error() == 0
        assert fake_peer[0].item() == 1   # this rank's arrival at barrier 1 reached the "peer"
        assert own[0].item() == 1 and own[32].item() == 1  # own arrival word and barrier count
        # the context is intact: a GPU op after the timed-out wait is correct
        x = torch.arange(1024, device="cuda", dtype=torch.float32)
        assert float((x * 2).sum().item()) == 2.0 * 1023 * 1024 / 2
        # and the barrier is refused until peers are set again
        bb.check(L.bonsai_dit_set_flag_peers(m.handle, None, 0), "set_flag_peers off")
        assert L.bonsai_dit_barrier(m.handle, bb.stream_ptr()) != 0
    finally:
        m.close()
