"""Head/token-split forward on 2 GPUs equals the one-GPU forward.

Spawns two NCCL ranks (one per GPU); each builds the same seeded model, runs
bonsai_b200.headsplit.forward, and rank 0 compares the prediction with the
unpartitioned bonsai_dit_forward of an identical model.  Both exchange forms
run: NCCL collectives between the phases, the fused form in which the
kernels store into the other GPU's buffers through CUDA IPC mappings
(headsplit.enable_fused), and its QKV scatter variant (phase 0's Q/K/V GEMM
stores every head into its owner's buffer); the fused forms order the ranks
with the engine's peer flag barrier, and once with a NCCL all-reduce.  Needs >= 2 GPUs (skipped otherwise).
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SMALL = dict(img=256, txt=64, grid=16, depth=2, single=2)
# BASELINE config 5(b) at full size: 2048^2 (128 x 128 latent tokens) + 512
# text tokens, all 19 + 38 blocks.
FULL = dict(img=16384, txt=512, grid=128, depth=19, single=38)


def _worker(rank, world, port, q, shape, fused, scatter=False, flags=True):
    import datetime
    import sys
    from pathlib import Path
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "bonsai.cpp_b200"))
    import torch
    import torch.distributed as dist
    import bonsai_b200 as bb
    from bonsai_b200 import headsplit
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        bb.init(rank)
        c = shape
        m = bb.Dit(bb.PRESET_FLUX1, c["img"], c["txt"], c["grid"], c["grid"], depth=c["depth"],
                   depth_single=c["single"], seed=11)
        m.set_partition(rank, world)
        if fused:
            headsplit.enable_fused(m, scatter_qkv=scatter, flag_barrier=flags)
        rng = np.random.default_rng(3)
        img = torch.from_numpy(rng.standard_normal((m.img, m.in_ch)).astype(np.float32)).cuda()
        txt = torch.from_numpy(rng.standard_normal((m.txt, m.ctx_dim)).astype(np.float32)).cuda()
        pooled = torch.from_numpy(rng.standard_normal(m.pooled).astype(np.float32)).cuda()
        out = torch.empty(m.img, m.in_ch, device="cuda")
        headsplit.forward(m, img, txt, pooled, 600.0, out)
        torch.cuda.synchronize()
        res = None
        if rank == 0:
            ref_m = bb.Dit(bb.PRESET_FLUX1, c["img"], c["txt"], c["grid"], c["grid"],
                           depth=c["depth"], depth_single=c["single"], seed=11)
            ref = torch.empty_like(out)
            ref_m.forward(img, txt, pooled, 600.0, ref)
            torch.cuda.synchronize()
            g, r = out.double().flatten(), ref.double().flatten()
            cos = float(g @ r / (g.norm() * r.norm()))
            rel = float((g - r).abs().max() / r.pow(2).mean().sqrt())
            res = (cos, rel)
            ref_m.close()
        dist.barrier()
        m.close()
        q.put((rank, res, bb.device_error()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused,scatter,flags",
                         [(False, False, False), (True, False, True), (True, True, True),
                          (True, True, False)],
                         ids=["nccl", "fused", "fused_qkv_scatter", "fused_qkv_scatter_nccl_order"])
@pytest.mark.parametrize("shape", [SMALL, FULL], ids=["small", "2048sq_full_depth"])
def test_headsplit_two_gpus_matches_single(shape, fused, scatter, flags):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, shape, fused, scatter, flags))
             for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (res, err)) for r, res, err in (q.get(timeout=600) for _ in range(2)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cos, rel = results[0][0]
    assert results[0][1] == 0 and results[1][1] == 0
    assert cos >= 0.9999 and rel <= 1e-2, (cos, rel)
