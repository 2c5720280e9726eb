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
The reference has no multi-device path: it runs in one process on one device.
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


def _all_gather_bytes(data: bytes, world: int, group) -> bytes:
    mine = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    every = torch.empty(world * mine.numel(), dtype=torch.uint8, device="cuda")
    dist.all_gather_into_tensor(every, mine, group=group)
    return bytes(every.cpu().numpy())


def enable_fused(model, group=None, scatter_qkv: bool = False, flag_barrier: bool = True) -> None:
    """Exchange CUDA IPC handles of every rank's xm / cat and give them to
    the engine (bonsai_dit_open_peers).  scatter_qkv: also every rank's qkv
    (bonsai_dit_open_qkv_peers), so that phase 0's Q/K/V GEMM stores each
    head into its owner's buffer instead of phase 0 broadcasting xm rows.
    flag_barrier: order the ranks between the phases with the engine's peer
    flag barrier (bonsai_dit_barrier: one small kernel, stores of a counter
    into every rank's flags over NVLink) instead of a one-element NCCL
    all-reduce.  Collective: every rank calls it (one process per GPU)."""
    world = dist.get_world_size(group)
    model.open_peers(_all_gather_bytes(model.ipc_handles(), world, group), world)
    if scatter_qkv:
        model.open_qkv_peers(_all_gather_bytes(model.ipc_handle("qkv"), world, group), world)
    model.flag_barrier = False
    if flag_barrier:
        model.open_flag_peers(_all_gather_bytes(model.ipc_handle("flags"), world, group), world)
        dist.barrier(group=group)  # every rank's flags are zeroed before the first barrier
        model.flag_barrier = True
    model.fused_exchange = True


def _order(model, token: torch.Tensor, group) -> None:
    """Stream-ordered barrier: the next kernels on this rank start after every
    rank has finished the kernels it issued before (they wrote into this
    rank's buffers).  The engine's peer flag barrier where enable_fused set
    it up, else a one-element NCCL all-reduce."""
    if getattr(model, "flag_barrier", False):
        model.barrier()
    else:
        dist.all_reduce(token, group=group)


class _Span:
    """Records a (name, start, end) pair of CUDA events on the current stream
    into `timers` around a block of issued work (no-op when timers is None)."""

    def __init__(self, timers, name):
        self.timers, self.name = timers, name

    def __enter__(self):
        if self.timers is not None:
            self.e0 = torch.cuda.Event(enable_timing=True)
            self.e0.record()
        return self

    def __exit__(self, *exc):
        if self.timers is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            self.timers.append((self.name, self.e0, e1))


def phase_times(timers) -> dict:
    """Sum the event pairs recorded by forward(timers=...) per name (ms);
    call after the stream has been synchronised."""
    out = {}
    for name, e0, e1 in timers:
        out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
    return out


def forward(model, img, txt, pooled, t: float, out, group=None, timers=None,
            phased: bool = False) -> None:
    """One denoise-step forward of a partitioned bonsai_b200.Dit.  img/txt/
    pooled are the full inputs (device tensors) on every rank; out
    [img_tokens][in_ch] receives the full prediction on every rank.

    timers: optional list; a (name, start event, end event) triple is
    appended for every stage -- "edges" (begin + end), "phase0", "phase1",
    "phase2", and the exchanges ("order" for the fused form's ordering
    all-reduce, "xm_gather" / "cat_exchange" for the NCCL form, "hidden_gather")
    -- for a per-phase breakdown (phase_times).  phased: on one rank, run the
    phase entry points instead of the replayed step graph (same result; used
    for the one-GPU breakdown)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1 and not phased and timers is None:
        model.forward(img, txt, pooled, t, out)  # one rank: the plain (graph-replayed) step
        return
    rank = dist.get_rank(group) if world > 1 else 0
    L = model.L
    C = H + model.mlp
    xm = model.buffer("xm", torch.float16, (L, H))
    cat = model.buffer("cat", torch.float16, (L, C))
    hidden = model.buffer("hidden", torch.float32, (L, H))
    fused = world > 1 and getattr(model, "fused_exchange", False)
    token = torch.zeros(1, dtype=torch.int32, device="cuda") if fused else None
    with _Span(timers, "edges"):
        model.begin(img, txt, pooled, t)
    for kind, n in ((0, model.depth), (1, model.depth_single)):
        for i in range(n):
            with _Span(timers, "phase0"):
                model.phase(kind, i, 0)
            if fused:
                with _Span(timers, "order"):
                    _order(model, token, group)
            elif world > 1:
                with _Span(timers, "xm_gather"):
                    gather_rows_inplace(xm, rank, world, group)
            with _Span(timers, "phase1"):
                model.phase(kind, i, 1)
            if fused:
                with _Span(timers, "order"):
                    _order(model, token, group)
            elif world > 1:
                with _Span(timers, "cat_exchange"):
                    heads_to_rows(cat, H, rank, world, group)
            with _Span(timers, "phase2"):
                model.phase(kind, i, 2)
    if world > 1:
        with _Span(timers, "hidden_gather"):
            gather_rows_inplace(hidden, rank, world, group)
    with _Span(timers, "edges"):
        model.end(out)
