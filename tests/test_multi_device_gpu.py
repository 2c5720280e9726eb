"""One process driving two GPUs through the C ABI: the kernels' launch set-up
(shared-memory attributes, cluster occupancy) is cached per device, so the
second device's first launches must work and give the same bits as the
first's.  Needs >= 2 GPUs (skipped otherwise)."""
import numpy as np
import pytest

import bonsai_b200 as bb

pytestmark = pytest.mark.gpu


def _run_on(device, packed, N, K, x_np, qkv_np):
    import torch
    torch.cuda.set_device(device)
    bb.init(device)
    w = bb.B1Weight(packed, N, K)
    try:
        x16 = torch.from_numpy(x_np).cuda().half()
        out = torch.empty(x16.shape[0], N, device="cuda")
        bb.b1_gemm(x16, w, bb.BONSAI_EPI_F32, out)
        q, k, v = (torch.from_numpy(a).cuda().half() for a in qkv_np)
        att = torch.empty(q.shape[1], q.shape[0] * 128, device="cuda", dtype=torch.float16)
        bb.joint_attention(q, k, v, att)
        torch.cuda.synchronize()
        assert bb.device_error() == 0
        return out.cpu().numpy(), att.float().cpu().numpy()
    finally:
        w.free()


def test_two_devices_one_process(gpu):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    rng = np.random.default_rng(21)
    N, K, T = 3072, 3072, 700
    packed = bb.random_b1_packed(N, K, rng)
    x = rng.standard_normal((T, K)).astype(np.float32)
    qkv = [rng.standard_normal((4, 1000, 128)).astype(np.float32) for _ in range(3)]
    try:
        g0, a0 = _run_on(0, packed, N, K, x, qkv)
        g1, a1 = _run_on(1, packed, N, K, x, qkv)
    finally:
        torch.cuda.set_device(0)
        bb.init(0)
    assert np.array_equal(g0, g1)
    assert np.array_equal(a0, a1)


def test_weight_on_another_device_is_rejected(gpu):
    """A B1_0 weight uploaded on device 0 and used while device 1 is current
    is an argument error for the drop-in linears, not a launch against memory
    of another GPU."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    L = bb.lib()
    rng = np.random.default_rng(5)
    K, N, T = 256, 128, 16
    torch.cuda.set_device(0)
    bb.init(0)
    w = bb.B1Weight(bb.random_b1_packed(N, K, rng), N, K)
    try:
        torch.cuda.set_device(1)
        bb.init(1)
        act = torch.zeros(T, K, device="cuda")
        out = torch.zeros(T, N, device="cuda")
        for fn in (L.bonsai_b1_linear_f32, L.bonsai_b1_linear_f32_noalloc):
            rc = fn(act.data_ptr(), T, w.handle, out.data_ptr(), bb.stream_ptr())
            assert rc == -1 and b"lives on device 0" in L.bonsai_last_error()
        torch.cuda.synchronize()
    finally:
        torch.cuda.set_device(0)
        bb.init(0)
        w.free()
