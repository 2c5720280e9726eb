"""bonsai_b1_linear_f32_noalloc: the B1_0 linear for callers that cannot let
the library allocate (their allocator owns all device memory, or an
allocation's stall is not allowed).

It must give the same result as the allocating drop-in bonsai_b1_linear_f32,
call after call (its fixed scratch array keeps the previous call's contents),
and refuse inputs larger than its 8 MiB scratch with an error, not a fault.
This file is collected last so a failure here cannot hide other results.
"""
import ctypes

import numpy as np
import pytest

import bonsai_b200 as bb

pytestmark = pytest.mark.gpu


def test_noalloc_matches_allocating_linear_twice(gpu):
    import torch
    L = bb.lib()
    # second call smaller: stale scratch must not leak; third: one token, the
    # matrix-vector kernel both forms share
    shapes = [(300, 3072, 512), (17, 1024, 200), (1, 3072, 512)]
    for i, (T, K, N) in enumerate(shapes):
        rng = np.random.default_rng(40 + i)
        w = bb.B1Weight(bb.random_b1_packed(N, K, rng), N, K)
        act = torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32)).cuda()
        ref = torch.empty(T, N, device="cuda")
        got = torch.full((T, N), float("nan"), device="cuda")
        bb.b1_linear_f32(act, w, ref)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        bb.check(L.bonsai_b1_linear_f32_noalloc(act.data_ptr(), T, w.handle, got.data_ptr(),
                                                bb.stream_ptr()), "b1_linear_f32_noalloc")
        torch.cuda.synchronize()
        if i > 0:  # after the first call has loaded the library's kernels on this device
            assert torch.cuda.mem_get_info()[0] == free_before, "the no-allocation call allocated"
        # same kernels on the same (f16-rounded, or for one token f32) activations:
        # identical up to f32 summation order
        torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)
        w.free()


def test_noalloc_rejects_oversized_input(gpu):
    import torch
    L = bb.lib()
    K, N = 3072, 64
    w = bb.B1Weight(bb.random_b1_packed(N, K, np.random.default_rng(1)), N, K)
    T = (4 << 20) // K + 1  # one token past the fixed scratch
    act = torch.zeros(T, K, device="cuda")
    out = torch.zeros(T, N, device="cuda")
    rc = L.bonsai_b1_linear_f32_noalloc(act.data_ptr(), T, w.handle, out.data_ptr(), bb.stream_ptr())
    assert rc == -2 and b"exceeds the fixed scratch" in L.bonsai_last_error()
    torch.cuda.synchronize()
    w.free()
