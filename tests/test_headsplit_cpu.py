"""Host logic of the multi-GPU head/token split, on CPU with gloo (world 2).

The engine computes each rank's heads for every row and each rank's rows
for every head; bonsai_b200.headsplit moves the data between those two
layouts.  These tests run that data movement on CPU ranks and check every
element lands where a single-process run would have it.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "bonsai.cpp_b200"))
    from bonsai_b200 import headsplit
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L, width, C = 12, 8, 11  # rows, attention columns, cat width
        rows, hc = L // world, width // world
        # reference: element (t, c) = 1000*t + c
        full = (torch.arange(L)[:, None] * 1000 + torch.arange(C)[None, :]).float()
        # after phase 1: this rank knows its head columns for every row
        cat = torch.full((L, C), -1.0)
        cat[:, rank * hc:(rank + 1) * hc] = full[:, rank * hc:(rank + 1) * hc]
        headsplit.heads_to_rows(cat, width, rank, world)
        mine = slice(rank * rows, (rank + 1) * rows)
        ok1 = torch.equal(cat[mine, :width], full[mine, :width])
        # row all-gather in place
        buf = torch.full((L, 3), -1.0)
        buf[mine] = full[mine, :3]
        headsplit.gather_rows_inplace(buf, rank, world)
        ok2 = torch.equal(buf, full[:, :3])
        q.put((rank, bool(ok1), bool(ok2)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_row_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok1 and ok2 for _, ok1, ok2 in results), results
