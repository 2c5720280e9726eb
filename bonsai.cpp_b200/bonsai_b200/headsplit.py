"""One long image across GPUs: token rows and attention heads split by rank.

BASELINE config 5(b): a 2048^2 image (16384 image + 512 text tokens) on
2/4/8 GPUs, one process per GPU.  Every rank holds a full model (weights are
1.6-2.2 GB) and calls bonsai_dit_set_partition(rank, world); the engine then
computes, per block,
  phase 0  LN-modulate of its L/world token rows,
  phase 1  Q/K/V for its 24/world heads over ALL rows (the QKV weight is
           split by head, so no FLOP is repeated), Q/K norm + RoPE and the
           attention of those heads,
  phase 2  out-projection, MLP and gate-residuals of its own rows,
and the data moves between the phases in one of two ways:
  * fused (enable_fused, the default on GPUs): every rank maps the others'
    `xm` and `cat` buffers (CUDA IPC over NVLink) and the producing kernels
    store there directly -- phase 0's LayerNorm-modulate kernel writes its
    rows into every rank's xm, phase 1's attention kernel writes each output
    row into its owner's cat -- so the only collective left per phase is a
    one-element all-reduce that orders the ranks (no rank reads a buffer
    before every rank has finished writing into it);
  * caller-side (torch.distributed, NCCL or gloo): an in-place all-gather of
    the rows of `xm` (phase 0 -> 1) and an all-to-all of the attention output
    in `cat` (every rank holds its heads' columns for every row and needs
    every head's columns for its own rows).
The reference has no multi-device path (SURVEY: single process).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

H = 3072


def gather_rows_inplace(buf: torch.Tensor, rank: int, world: int, group=None) -> None:
    """buf [L][...]: rank r's rows [r*L/world, (r+1)*L/world) are valid on rank
    r; afterwards every rank holds all rows (NCCL in-place all-gather)."""
    rows = buf.shape[0] // world
    dist.all_gather_into_tensor(buf, buf[rank * rows:(rank + 1) * rows], group=group)


def heads_to_rows(cat: torch.Tensor, width: int, rank: int, world: int, group=None) -> None:
    """cat [L][>= width]: on entry rank r holds columns [r*width/world,
    (r+1)*width/world) (its heads) for every row; on exit it holds all `width`
    columns for its own rows [r*L/world, (r+1)*L/world)."""
    L = cat.shape[0]
    rows, hc = L // world, width // world
    send = cat[:, rank * hc:(rank + 1) * hc].reshape(world, rows, hc).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    mine = cat[rank * rows:(rank + 1) * rows, :width].view(rows, world, hc)
    mine.copy_(recv.permute(1, 0, 2))


def enable_fused(model, group=None) -> None:
    """Exchange CUDA IPC handles of every rank's xm / cat and give them to
    the engine (bonsai_dit_open_peers).  Collective: every rank calls it."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    mine = torch.frombuffer(bytearray(model.ipc_handles()), dtype=torch.uint8).cuda()
    every = torch.empty(world * mine.numel(), dtype=torch.uint8, device="cuda")
    dist.all_gather_into_tensor(every, mine, group=group)
    model.open_peers(bytes(every.cpu().numpy()), world)
    model.fused_exchange = True


def _order(token: torch.Tensor, group) -> None:
    """Stream-ordered barrier: the next kernels on this rank start after every
    rank has finished the kernels it issued before (they wrote into this
    rank's buffers)."""
    dist.all_reduce(token, group=group)


def forward(model, img, txt, pooled, t: float, out, group=None) -> None:
    """One denoise-step forward of a partitioned bonsai_b200.Dit.  img/txt/
    pooled are the full inputs (device tensors) on every rank; out
    [img_tokens][in_ch] receives the full prediction on every rank."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        model.forward(img, txt, pooled, t, out)  # one rank: the plain (graph-replayed) step
        return
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    L = model.L
    C = H + model.mlp
    xm = model.buffer("xm", torch.float16, (L, H))
    cat = model.buffer("cat", torch.float16, (L, C))
    hidden = model.buffer("hidden", torch.float32, (L, H))
    fused = getattr(model, "fused_exchange", False)
    token = torch.zeros(1, dtype=torch.int32, device="cuda") if fused else None
    model.begin(img, txt, pooled, t)
    for kind, n in ((0, model.depth), (1, model.depth_single)):
        for i in range(n):
            model.phase(kind, i, 0)
            if fused:
                _order(token, group)
            else:
                gather_rows_inplace(xm, rank, world, group)
            model.phase(kind, i, 1)
            if fused:
                _order(token, group)
            else:
                heads_to_rows(cat, H, rank, world, group)
            model.phase(kind, i, 2)
    gather_rows_inplace(hidden, rank, world, group)
    model.end(out)
