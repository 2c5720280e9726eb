#!/usr/bin/env python
"""Benchmark: ms per 1024^2 Flux.1-schnell denoise step on B200.

Workload (one image per GPU): 19 double + 38 single
blocks, hidden 3072, 24 x 128 heads, GELU MLP 12288, 4096 image tokens
(16-ch 128x128 latent, 2x2-packed) + 512 text tokens, pooled [768]; every
block linear (QKV, out-proj, MLP, per-block modulation) is B1_0 with
random-init weights (signs Bernoulli(0.5), scales |N(0,0.02)| as f16);
synthetic N(0,1) inputs.  A "step" is one transformer forward
(bonsai_dit_forward) at timestep t = 1000 * (1 - i/steps).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl bonsai|reference]

N > 1 runs under torch.distributed.run, one rank per GPU, each rank its own
image (data parallel, no collective on the data path; weak scaling).
--impl reference times the reference's own CPU path (its b1_linear_f32_f32
AVX2 kernel compiled into oracle/_ref, plus the CPU restatement of the
ggml built-ins) on a bounded sample and extrapolates to ms per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "bonsai.cpp_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np

H, HEADS, HD = 3072, 24, 128
MLP = 12288
IMG, TXT, GRID, POOLED, IN_CH, CTX = 4096, 512, 64, 768, 64, 4096
DEPTH, SINGLE = 19, 38
L = IMG + TXT
METRIC = "ms/denoise step @1024² Flux-DiT (1–8 B200); B1_0 GEMM & attn % of bf16 peak"
WORKLOAD = ("flux1-schnell DiT denoise step @1024^2: 19 double + 38 single blocks, "
            "L = 512 text + 4096 image tokens, all block linears B1_0 (1-bit)")
WORKLOAD_2048 = ("flux1-schnell DiT denoise step @2048^2: 19 double + 38 single blocks, "
                 "L = 512 text + 16384 image tokens, one image split across the GPUs")


# DRAM traffic of the B1_0 GEMM (dram__bytes_read.sum + dram__bytes_write.sum)
# per launch of the flux1 1024^2 step: one ncu capture of one launch of each
# of the step's ten GEMM shapes (kernel_bench, L2 flushed before the launch),
# weighted by the shapes' launch counts (profiles/b1_gemm_dram_flux1_1024.md).
# It applies to the default workload only.
GEMM_DRAM_BYTES_PER_LAUNCH = 115.82e6


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"],
                "bf16_sustained": d["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def step_flops(L=None, IMG=None):
    """Algorithmic FLOPs of one step (GEMM 2*M*N*K, attention 4*L^2*D*H)."""
    L = L or globals()["L"]
    IMG = IMG or globals()["IMG"]
    attn = 4.0 * L * L * HD * HEADS
    dbl = 2.0 * L * H * (3 * H + H + MLP) + 2.0 * L * MLP * H + attn
    sgl = 2.0 * L * H * (3 * H + MLP) + 2.0 * L * (H + MLP) * H + attn
    mods = 2.0 * H * (DEPTH * 12 * H + SINGLE * 3 * H)
    edges = 2.0 * (TXT * CTX * H + IMG * IN_CH * H + IMG * H * IN_CH + 256 * H + 2 * H * H
                   + POOLED * H + 2 * H * H)
    return DEPTH * dbl + SINGLE * sgl + mods + edges


# ------------------------------------------------------------ CPU reference
_JSON_FD = None  # the process's original stdout, kept for the JSON lines only


def emit_json(obj) -> None:
    """Write one JSON line to the original stdout.  Everything else that
    reaches fd 1 (library banners such as NCCL's version line, stray prints)
    goes to stderr, so stdout carries the JSON line(s) only."""
    sys.stdout.flush()
    data = (json.dumps(obj) + "\n").encode()
    fd = _JSON_FD if _JSON_FD is not None else 1
    while data:
        data = data[os.write(fd, data):]


class stdout_to_stderr:
    """Send fd 1 to fd 2 for the duration (the reference's kernel prints a
    banner with fprintf(stdout) on first use; bench.py's stdout must carry the
    JSON line only)."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


class CpuSample:
    """Bounded sample of the reference CPU path at the bench workload.

    One double block and one single block at the full token count
    (L = 4608), with the reference's own b1_linear_f32_f32 (AVX2 build in
    oracle/_ref, all host threads) on every output row of each linear,
    attention for `heads` of the 24 heads, and the remaining ops
    (LayerNorm-modulate, Q/K RMSNorm + RoPE, GELU) in full through the CPU
    restatement of the ggml built-ins.  Each part's time is scaled by the
    work it skipped, then ms/step = 19 * double + 38 * single + edges.
    Both the bench line's cpu_baseline and the --impl reference arm use
    every output row and 4 heads (about 5-10 s of CPU work per sample on a
    16-core host); the reference kernel runs on a persistent worker pool
    (oracle/ref_bridge.cpp), as ggml's CPU backend does.
    """

    def __init__(self, threads: int, heads: int = 4):
        self.ROW_FRAC = 1
        self.heads = heads
        import ctypes
        from oracle import pyoracle as O
        self.O = O
        self.threads = threads
        self.fast = ctypes.CDLL(str(ROOT / "oracle/_build/libbonsai_oracle_fast.so"))
        vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        self.fast.orc_attention.argtypes = [vp, vp, vp, i, i, i, f, vp]
        self.fast.orc_ln_modulate.argtypes = [vp, i, i, vp, vp, f, vp]
        self.fast.orc_gelu.argtypes = [vp, i, i, vp, i]
        self.fast.orc_qk_norm_rope_heads.argtypes = [vp, i, i, i, vp, vp, i, f, vp, vp]
        self.fast.orc_linear_f32.argtypes = [vp, i, i, vp, vp, i, vp]
        self.fast.orc_set_threads.argtypes = [i]
        self.fast.orc_set_threads(threads)
        R = O.ref()
        self.kind = "reference" if R is not None else "port"
        rng = np.random.default_rng(77)
        self.rng = rng
        self.x = rng.standard_normal((L, MLP + H)).astype(np.float32)  # activations (any row/col slice)
        self.h = rng.standard_normal((L, H)).astype(np.float32)
        self.y = np.zeros((L, MLP + H), np.float32)
        self.shift = rng.standard_normal(H).astype(np.float32)
        self.scale = rng.standard_normal(H).astype(np.float32)
        self.qkh = rng.standard_normal((1, L, HD)).astype(np.float32)
        self.nw = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
        ids = np.zeros((L, 3), np.float32)
        for y in range(GRID):
            for x in range(GRID):
                ids[TXT + y * GRID + x, 1:] = (y, x)
        self.cos, self.sin = O.rope_cos_sin(ids, [16, 56, 56], 10000.0)
        self.q1 = rng.standard_normal((L, 1, HD)).astype(np.float32)
        self.att = np.zeros((L, HD), np.float32)
        self.w = {}

    def _packed(self, rows, K):
        key = (rows, K)
        if key not in self.w:
            nb = K // 32
            raw = np.zeros((rows, nb, 6), np.uint8)
            raw[:, :, 0:2] = (np.abs(self.rng.standard_normal((rows, nb))) * 0.02).astype(
                np.float16).view(np.uint8).reshape(rows, nb, 2)
            raw[:, :, 2:6] = self.rng.integers(0, 256, size=(rows, nb, 4), dtype=np.uint8)
            self.w[key] = raw.reshape(rows, nb * 6)
        return self.w[key]

    def _lin(self, tokens, K, N, row_frac=None):
        """Time the reference B1 kernel on N/row_frac rows (all rows unless given);
        return the full-N estimate (s)."""
        O = self.O
        n = max(1, N // (row_frac or self.ROW_FRAC))
        w = self._packed(n, K)
        act = np.ascontiguousarray(self.x[:tokens, :K])
        out = np.zeros((tokens, n), np.float32)
        t0 = time.perf_counter()
        if self.kind == "reference":
            O.ref().ref_b1_linear(act.ctypes.data, tokens, K, w.ctypes.data, n, out.ctypes.data,
                                  self.threads)
        else:
            O.lib().orc_b1_linear(act.ctypes.data, tokens, K, w.ctypes.data, n, out.ctypes.data)
        return (time.perf_counter() - t0) * N / n

    def _timed(self, fn):
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    def _ln(self, rows):
        return self._timed(lambda: self.fast.orc_ln_modulate(
            self.h.ctypes.data, rows, H, self.shift.ctypes.data, self.scale.ctypes.data, 1e-6,
            self.y.ctypes.data))

    def _qk(self):  # q and k of all 24 heads: time one head's rows x 48
        return 2 * HEADS * self._timed(lambda: self.fast.orc_qk_norm_rope_heads(
            self.qkh.ctypes.data, 1, L, HD, self.nw.ctypes.data, self.nw.ctypes.data, TXT, 1e-6,
            self.cos.ctypes.data, self.sin.ctypes.data))

    def _attn(self):  # `heads` of 24 heads, one at a time, scaled
        t = sum(self._timed(lambda: self.fast.orc_attention(
            self.q1.ctypes.data, self.q1.ctypes.data, self.q1.ctypes.data, L, 1, HD,
            float(HD ** -0.5), self.att.ctypes.data)) for _ in range(self.heads))
        return HEADS / self.heads * t

    def _gelu(self, rows):
        return self._timed(lambda: self.fast.orc_gelu(self.x.ctypes.data, rows, MLP,
                                                      self.y.ctypes.data, MLP))

    def run(self):
        """One sampled step; returns (extrapolated ms per denoise step, sample seconds)."""
        t_start = time.perf_counter()
        dbl = 2 * self._ln(L) + self._qk() + self._attn() + self._gelu(L)
        for tok in (TXT, IMG):
            dbl += (self._lin(tok, H, 3 * H) + self._lin(tok, H, H) + self._lin(tok, H, MLP)
                    + self._lin(tok, MLP, H))
        sgl = self._ln(L) + self._qk() + self._attn() + self._gelu(L)
        sgl += self._lin(L, H, 3 * H + MLP) + self._lin(L, H + MLP, H)
        # one token x 1.05 M modulation rows: sampled at 1/16 of the rows (a
        # full-size packed copy would be 0.6 GB of host memory; a GEMV of one
        # token is a small share of the step either way)
        mods = self._lin(1, H, DEPTH * 12 * H + SINGLE * 3 * H, row_frac=16)
        edges = self._lin(TXT, CTX, H)  # text embedder (dominant edge op), B1-rate proxy
        ms = 1000.0 * (DEPTH * dbl + SINGLE * sgl + mods + edges)
        return ms, time.perf_counter() - t_start

    def describe(self):
        rows = "all" if self.ROW_FRAC == 1 else f"1/{self.ROW_FRAC}"
        return (f"1 double + 1 single block at L=4608 per sample: reference b1_linear_f32_f32 "
                f"(AVX2, oracle/_ref) on {rows} of each linear's output rows, attention "
                f"on {self.heads} of 24 heads, LayerNorm/RMSNorm/RoPE/GELU in full (CPU restatement "
                f"of the ggml built-ins); scaled to 19 double + 38 single blocks + modulation + edges")


ORDER_DESC = {"flags": "a peer flag barrier per phase for ordering",
              "nccl": "one-element NCCL all-reduce per phase for ordering"}


def step_config(world: int, split: bool = False, exchange: str = "scatter",
                order: str = "flags") -> dict:
    """The bench line's `config`, identical in both arms for the same N."""
    if split:
        par = {"fused": f"head/row split over {world} GPUs, exchanges fused into the producing "
                        "kernels over peer memory (CUDA IPC), " + ORDER_DESC[order],
               "scatter": f"head/row split over {world} GPUs, Q/K/V of own rows stored into the "
                          "heads' owners by the GEMM epilogue and attention rows into the rows' "
                          "owners, over peer memory (CUDA IPC), " + ORDER_DESC[order],
               "nccl": f"head/row split over {world} GPUs (NCCL all-gather + all-to-all per "
                       "block)"}[exchange]
    else:
        par = f"dp{world} (one image per GPU, no collective)"
    return {"workload": WORKLOAD_2048 if split else WORKLOAD,
            "global_batch": 1 if split else world, "img_tokens": IMG, "txt_tokens": TXT,
            "parallelism": par,
            "l2": "inputs larger than L2: every step streams all 2.2 GB of B1_0 weights"}


def run_reference(args):
    """--impl reference: the reference's CPU path on this host's cores, one
    bounded sample per step -- the same sample as the GPU arm's cpu_baseline
    leg (one double + one single block at L = 4608, every output row of every
    B1_0 linear through the reference's own kernel, 4 of 24 attention heads),
    scaled to the 57 blocks + modulation + edges.  Only rank 0 works."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    with stdout_to_stderr():
        cs = CpuSample(threads)
        for _ in range(args.warmup):
            cs.run()
        vals = []
        for _ in range(args.steps):
            ms, _ = cs.run()
            vals.append(ms)
    v = statistics.mean(vals)
    line = {
        "metric": METRIC, "value": round(v, 1), "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v, 1),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": step_config(args.gpus),
        "cpu_baseline": {"value": round(v, 1), "unit": "ms", "cores": threads, "kind": cs.kind,
                         "sample": f"mean of {args.steps} samples; each " + cs.describe(),
                         "spread_ms": [round(min(vals), 1), round(max(vals), 1)]},
        "e2e": {"value": round(v, 1), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit_json(line)
    return 0


# ------------------------------------------------------------------ GPU arm
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int, log: str | None = None):
        self.log = log
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.gpu = vis.split(",")[local_rank] if vis else str(local_rank)
        self.proc = None

    def start(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", self.gpu], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.seek(0)
        raw = self.f.read()
        if self.log:
            Path(self.log).write_text(raw)
        rows = [r.split(",") for r in raw.strip().splitlines() if r.count(",") >= 8]
        self.f.close()
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if r[5 + j].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def measure_split_2048(args, rank: int, world: int, dist) -> dict:
    """BASELINE config 5(b) beside the headline: one 2048^2 image (16384 image +
    512 text tokens, all 57 blocks) split by heads and token rows over the
    `world` GPUs of this run (one GPU: the plain step), outside the headline's
    timed region.  Every rank calls it (it takes collective steps).

    ms_per_step: device time of `split_steps` steps (CUDA events on the
    launching stream, barrier + synchronize on both sides, max over ranks).
    e2e_ms: the same with the step's inputs copied in from pinned host memory
    and the prediction copied back, inside the timed region.  phase_ms: one
    more step with a CUDA-event pair around every phase and exchange, summed
    per stage (max over ranks); on one GPU the phases run unsplit, without
    exchanges.  parity_vs_unsplit (N > 1): rank 0 runs the unpartitioned
    forward of the same model on the same inputs and compares (cos, max-abs /
    RMS)."""
    import torch
    import bonsai_b200 as bb
    from bonsai_b200 import headsplit
    img_n, grid = 16384, 128
    m = bb.Dit(bb.PRESET_FLUX1, img_n, TXT, grid, grid, seed=1234)
    if world > 1:
        m.set_partition(rank, world)
        if args.exchange in ("fused", "scatter"):
            headsplit.enable_fused(m, scatter_qkv=args.exchange == "scatter",
                                   flag_barrier=args.order == "flags")
    rng = np.random.default_rng(2048)  # one shared image on every rank
    img_h = torch.from_numpy(rng.standard_normal((img_n, IN_CH)).astype(np.float32)).pin_memory()
    txt_h = torch.from_numpy(rng.standard_normal((TXT, CTX)).astype(np.float32)).pin_memory()
    pooled_h = torch.from_numpy(rng.standard_normal(POOLED).astype(np.float32)).pin_memory()
    out_h = torch.empty(img_n, IN_CH).pin_memory()
    img_d, txt_d, pooled_d = img_h.cuda(), txt_h.cuda(), pooled_h.cuda()
    out_d = torch.empty(img_n, IN_CH, device="cuda")
    K, W = args.split_steps, max(3, args.split_warmup)
    ts = [1000.0 * (1.0 - (i % 4) / 4.0) for i in range(max(K, W))]
    stream = torch.cuda.current_stream()

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def step(t, timers=None):
        headsplit.forward(m, img_d, txt_d, pooled_d, t, out_d, timers=timers,
                          phased=timers is not None)

    def timed(fn):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(K):
            fn(ts[i])
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / K)

    for i in range(W):
        step(ts[i])
    torch.cuda.synchronize()
    assert bb.device_error() == 0
    ms = timed(step)

    def step_host(t):  # pinned host inputs in, prediction out, inside the timed region
        img_d.copy_(img_h, non_blocking=True)
        txt_d.copy_(txt_h, non_blocking=True)
        pooled_d.copy_(pooled_h, non_blocking=True)
        step(t)
        out_h.copy_(out_d, non_blocking=True)
        stream.synchronize()
    ms_e2e = timed(step_host)

    timers = []
    barrier()
    torch.cuda.synchronize()
    step(ts[0], timers)
    torch.cuda.synchronize()
    pt = headsplit.phase_times(timers)
    # every rank ran the same stages, so the key set (and the order of the
    # reductions below) is the same on all ranks
    phase_ms = {k: round(max_over_ranks(pt[k]), 3) for k in sorted(pt)}
    phase_ms_min = {k: round(-max_over_ranks(-pt[k]), 3) for k in sorted(pt)}
    keys = sorted(pt)
    if dist:  # every rank's own phase times (same key order on all ranks)
        mine = torch.tensor([pt[k] for k in keys], device="cuda", dtype=torch.float64)
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        by_rank = [{k: round(float(v), 3) for k, v in zip(keys, e.tolist())} for e in every]
    else:
        by_rank = [{k: round(pt[k], 3) for k in keys}]
    assert bb.device_error() == 0

    res = {"n_gpus": world, "ms_per_step": round(ms, 3), "e2e_ms": round(ms_e2e, 3),
           "steps": K, "warmup": W, "img_tokens": img_n, "txt_tokens": TXT,
           "exchange": (args.exchange if world > 1 else "none (one GPU: the plain step)"),
           "order": (ORDER_DESC[args.order] if world > 1 and args.exchange != "nccl" else None),
           "images_per_s": round(1000.0 / ms, 3),
           "step_tflops": round(step_flops(img_n + TXT, img_n) / (ms / 1e3) / 1e12, 1),
           "phase_ms": phase_ms, "phase_ms_min_rank": phase_ms_min, "phase_ms_by_rank": by_rank,
           "phase_ms_note": "one extra step, a CUDA-event pair around every phase and exchange "
                            "call, summed per stage; phase_ms = max over ranks, "
                            "phase_ms_min_rank = min over ranks (the spread is load imbalance)"}
    step(ts[0])
    torch.cuda.synchronize()
    split_out = out_d.clone()
    if world > 1:
        parity = None
        if rank == 0:  # the unpartitioned forward of the same weights on the same inputs
            m.set_partition(0, 1)
            ref = torch.empty_like(out_d)
            m.forward(img_d, txt_d, pooled_d, ts[0], ref)
            torch.cuda.synchronize()
            g, r = split_out.double().flatten(), ref.double().flatten()
            parity = {"cos": round(float(g @ r / (g.norm() * r.norm())), 8),
                      "maxabs_rms": float((g - r).abs().max() / r.pow(2).mean().sqrt()),
                      "vs": "unpartitioned bonsai_dit_forward of the same model on rank 0"}
        barrier()
        res["parity_vs_unsplit"] = parity
    else:
        res["parity_vs_unsplit"] = {"note": "one GPU: the split is the unpartitioned step"}
    res["output_finite"] = bool(torch.isfinite(split_out).all().item())
    assert bb.device_error() == 0
    m.close()
    return res


def run_bonsai(args):
    import torch
    import bonsai_b200 as bb

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    bb.init(local)
    split = args.workload == "2048"
    global IMG, GRID, L
    if split:  # BASELINE config 5(b): 128 x 128 latent tokens + 512 text tokens
        IMG, GRID = 16384, 128
        L = IMG + TXT
    model = bb.Dit(bb.PRESET_FLUX1, IMG, TXT, GRID, GRID, seed=1234)
    if split:
        from bonsai_b200 import headsplit
        if world > 1:
            model.set_partition(rank, world)
            if args.exchange in ("fused", "scatter"):
                headsplit.enable_fused(model, scatter_qkv=args.exchange == "scatter",
                                       flag_barrier=args.order == "flags")

    rng = np.random.default_rng(1000 + (0 if split else rank))  # split: one shared image
    img_h = torch.from_numpy(rng.standard_normal((IMG, IN_CH)).astype(np.float32)).pin_memory()
    txt_h = torch.from_numpy(rng.standard_normal((TXT, CTX)).astype(np.float32)).pin_memory()
    pooled_h = torch.from_numpy(rng.standard_normal(POOLED).astype(np.float32)).pin_memory()
    out_h = torch.empty(IMG, IN_CH).pin_memory()
    img_d, txt_d, pooled_d = img_h.cuda(), txt_h.cuda(), pooled_h.cuda()
    out_d = torch.empty(IMG, IN_CH, device="cuda")
    K, W = args.steps, args.warmup
    ts = [1000.0 * (1.0 - (i % 4) / 4.0) for i in range(max(K, W))]  # schnell's 4-step schedule

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream()

    def step(t):
        if split:
            headsplit.forward(model, img_d, txt_d, pooled_d, t, out_d)
        else:
            model.forward(img_d, txt_d, pooled_d, t, out_d)

    for i in range(W):
        step(ts[i])
    torch.cuda.synchronize()
    assert bb.device_error() == 0

    # ---- timed region: device-resident inputs
    clocks = ClockSampler(local, os.environ.get("BONSAI_CLOCK_LOG"))
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    bb.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        step(ts[i])
    e1.record(stream)
    torch.cuda.synchronize()
    launches = bb.launch_count()
    clk = clocks.stop()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / K)
    assert bb.device_error() == 0

    # ---- the same K steps again with every launch bracketed by CUDA events on
    # its stream (per-kernel durations for the roofline); kept out of the
    # headline timing because ~940 event records per step add ~1 ms.
    bb.profile_start()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for i in range(K):
        step(ts[i])
    p1.record(stream)
    torch.cuda.synchronize()
    prof = bb.profile_stop()
    ms_profiled = p0.elapsed_time(p1) / K

    # ---- end to end through the host-buffer C-ABI entry point
    out_np = out_h.numpy()
    img_np, txt_np, pooled_np = img_h.numpy(), txt_h.numpy(), pooled_h.numpy()
    def step_host(t):
        if split:  # copies in, partitioned step, prediction out
            img_d.copy_(img_h, non_blocking=True)
            txt_d.copy_(txt_h, non_blocking=True)
            pooled_d.copy_(pooled_h, non_blocking=True)
            headsplit.forward(model, img_d, txt_d, pooled_d, t, out_d)
            out_h.copy_(out_d, non_blocking=True)
            torch.cuda.current_stream().synchronize()
        else:
            model.forward_host(img_np, txt_np, pooled_np, t, out_np)

    for i in range(2):
        step_host(ts[i])
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for i in range(K):
        step_host(ts[i])
    f1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(f0.elapsed_time(f1) / K)
    finite = bool(np.isfinite(out_np).all())

    pk = peaks()
    g = prof.get("b1_gemm", {})
    a = prof.get("attention", {})
    gemm_tf = g["flop"] / (g["ms"] / 1e3) / 1e12 if g else None
    attn_tf = a["flop"] / (a["ms"] / 1e3) / 1e12 if a else None
    per_step = {k: {"launches": v["launches"] / K, "ms": round(v["ms"] / K, 4),
                    "share": round(v["ms"] / sum(x["ms"] for x in prof.values()), 4)}
                for k, v in prof.items()}
    line = {
        "metric": METRIC, "value": round(ms, 3), "unit": "ms", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(ms, 3), "higher_is_better": False,
        "scaling": "strong" if split else "weak",
        "vs_baseline": None, "dtype": "f16 operands, f32 accumulate and residual",
        "data": "synthetic",
        "config": step_config(world, split, args.exchange, args.order),
        "images_per_s": round((1 if split else world) * 1000.0 / ms, 3),
        "step_tflops": round(step_flops() / (ms / 1e3) / 1e12 * (1 if split else world), 1),
        "roofline": {"bound": "tensor", "kernel": "b1_gemm", "achieved": round(gemm_tf, 1),
                     "peak": pk["bf16_sustained"], "unit": "TFLOP/s",
                     "frac": round(gemm_tf / pk["bf16_sustained"], 4),
                     "peak_kind": f"{pk['source']} sustained bf16 (dense GEMM under the power cap)",
                     "frac_of_burst": round(gemm_tf / pk["bf16"], 4),
                     "traffic": None if split else GEMM_DRAM_BYTES_PER_LAUNCH,
                     "traffic_unit": "bytes per launch (ncu, one launch per GEMM shape of the step, "
                                     "weighted by launch count)",
                     "algorithmic_bytes": round(g["bytes"] / g["launches"]) if g else None,
                     "measured": "sum of 2*M*N*K over every b1_gemm launch / sum of their "
                                 "CUDA-event durations, over a second pass of the K steps"},
        "attention_roofline": {"bound": "tensor", "kernel": "attention",
                               "achieved": round(attn_tf, 1), "peak": pk["bf16_sustained"],
                               "unit": "TFLOP/s", "frac": round(attn_tf / pk["bf16_sustained"], 4),
                               "frac_of_burst": round(attn_tf / pk["bf16"], 4)},
        "kernels_per_step": per_step,
        "profiled_pass_ms_per_step": round(ms_profiled, 3),
        "gpu_launches": launches,
        "clocks": clk,
        "e2e": {"value": round(ms_e2e, 3), "unit": "ms",
                "h2d_bytes_per_step": (IMG * IN_CH + TXT * CTX + POOLED + 256) * 4,
                "d2h_bytes_per_step": IMG * IN_CH * 4, "output_finite": finite},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not split:
        threads = os.cpu_count() or 1
        with stdout_to_stderr():
            cs = CpuSample(threads)
            runs = [cs.run() for _ in range(2)]  # two samples, ~10-20 s of CPU work in total
            cpu_ms = statistics.mean(r[0] for r in runs)
            sample_s = sum(r[1] for r in runs)
        line["cpu_baseline"] = {"value": round(cpu_ms, 1), "unit": "ms", "cores": threads,
                                "kind": cs.kind, "sample": "mean of 2 samples; each " + cs.describe(),
                                "sample_seconds": round(sample_s, 2)}
    model.close()
    if not split and not args.no_split:
        line["split_2048"] = measure_split_2048(args, rank, world, dist)
    if world == 1 and not split and not args.no_side:
        # BASELINE configs 1-3 (GPU and reference CPU path) and the next
        # pipeline stage, the VAE decode, outside the headline's timed region
        with stdout_to_stderr():
            line["configs_1_3"] = measure_configs(args)
            vae = measure_vae(10, 3, not args.no_cpu_baseline)
        line["vae_1024"] = {k: vae[k] for k in ("metric", "value", "unit", "steps", "warmup",
                                                "roofline", "e2e", "clocks", "cpu_baseline",
                                                "gn_apply_gbs", "gpu_launches") if k in vae}
    if rank == 0:
        emit_json(line)
    if dist:
        dist.destroy_process_group()
    return 0


def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_configs(args):
    """--configs: BASELINE configs 1-3 as JSON lines (see measure_configs)."""
    for d in measure_configs(args):
        emit_json(d)
    return 0


def measure_configs(args) -> list:
    """BASELINE configs 1-3 timed on the GPU and with the reference CPU path
    on all host cores; one dict per config.

    C1 one Flux double block, 256 text + 1024 image tokens (32x32 grid);
    C2 joint attention only, 24 heads x 128, L = 4352;
    C3 the 18-shape B1_0 GEMM sweep (M in 1280/4352/8704 x six (K, N)).
    CPU: the reference's own b1_linear_f32_f32 (AVX2, oracle/_ref) for
    every B1_0 linear, the vectorised CPU restatement of the ggml built-ins
    for the rest (flash attention with f16 K/V, norms, RoPE).  GPU: the C ABI
    (CUDA events, mean of `steps` calls after `warmup`).  Speedups are
    GPU vs CPU on the same seeded inputs; not a parity check (the tests are).
    """
    import ctypes
    import torch
    import bonsai_b200 as bb
    from oracle import pyoracle as O
    torch.cuda.init()
    bb.init(0)
    threads = os.cpu_count() or 1
    info = {"cpu_threads": threads, "cpu_model": _cpu_model(), "device": torch.cuda.get_device_name(0)}
    R = O.ref()
    if R is None:
        return [{"configs": "unavailable", "why": "oracle/_ref (the reference's b1 kernel) is not built"}]
    fast = ctypes.CDLL(str(ROOT / "oracle/_build/libbonsai_oracle_fast.so"))
    vp, ci, cf = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fast.orc_set_threads.argtypes = [ci]
    fast.orc_set_threads(threads)
    fast.orc_use_reference_b1.argtypes = [vp, ci]
    fast.orc_set_attention_f16.argtypes = [ci]
    fast.orc_attention.argtypes = [vp, vp, vp, ci, ci, ci, cf, vp]
    fast.orc_double_block.argtypes = [ctypes.POINTER(O.Dims), ci, ci, vp] + [vp] * 16
    K_steps, W = args.steps, args.warmup

    def gpu_time(fn):
        for _ in range(W):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(K_steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / K_steps

    results = []

    def emit(name, flop, gms, cms, extra=None):
        d = {"config": name, "gpu_ms": round(gms, 4), "cpu_ms": round(cms, 1),
             "speedup": round(cms / gms, 1), "gpu_tflops": round(flop / gms / 1e9, 1),
             "cpu_gflops": round(flop / cms / 1e6, 1), **info}
        if extra:
            d.update(extra)
        results.append(d)

    rng = np.random.default_rng(1234)
    # ---- C1: one double block
    m = bb.Dit(bb.PRESET_FLUX1, 1024, 256, 32, 32, depth=1, depth_single=1, seed=1234)
    hidden = rng.standard_normal((m.L, H)).astype(np.float32)
    vec = rng.standard_normal(H).astype(np.float32)
    hd, vd = torch.from_numpy(hidden).cuda(), torch.from_numpy(vec).cuda()
    m.set_state(hd, vd)
    gms = gpu_time(lambda: m.double_block(0))
    mods, _ = O.modulations(m, vec)
    cos_t, sin_t = O.rope_cos_sin(m.rope_ids(), m.axes, m.theta)
    p = "double.0."
    w = {n: m.weight(p + n) for n in ("img_qkv", "txt_qkv", "img_out", "txt_out", "img_mlp_in",
                                      "img_mlp_out", "txt_mlp_in", "txt_mlp_out")}
    nrm = {n: m.weight_f32(p + n) for n in ("img_norm_q", "img_norm_k", "txt_norm_q", "txt_norm_k")}
    D = O.dims(m.swiglu, m.mlp)
    fast.orc_use_reference_b1(ctypes.cast(R.ref_b1_linear, vp), threads)
    fast.orc_set_attention_f16(1)
    h = hidden.copy()
    f = lambda a: np.ascontiguousarray(a, np.float32)
    mi, mt, ct, st = f(mods["double"][0][0]), f(mods["double"][0][1]), f(cos_t), f(sin_t)
    with stdout_to_stderr():
        t0 = time.perf_counter()
        fast.orc_double_block(ctypes.byref(D), m.txt, m.img, O.P(h), O.P(mi), O.P(mt),
                              O.P(w["img_qkv"]), O.P(w["txt_qkv"]), O.P(w["img_out"]), O.P(w["txt_out"]),
                              O.P(w["img_mlp_in"]), O.P(w["img_mlp_out"]), O.P(w["txt_mlp_in"]),
                              O.P(w["txt_mlp_out"]), O.P(nrm["img_norm_q"]), O.P(nrm["img_norm_k"]),
                              O.P(nrm["txt_norm_q"]), O.P(nrm["txt_norm_k"]), O.P(ct), O.P(st))
        cms = 1000 * (time.perf_counter() - t0)
    fast.orc_use_reference_b1(None, 1)
    L1 = m.L
    flop = 2.0 * L1 * H * (3 * H + H + MLP + MLP) + 4.0 * L1 * L1 * HD * HEADS
    emit("C1 double block, 256 txt + 1024 img tokens (flux1 dims)", flop, gms, cms)
    m.close()

    # ---- C2: attention, L = 4352
    L2 = 4352
    q, k, v = (torch.randn(HEADS, L2, HD, device="cuda").half() for _ in range(3))
    out = torch.empty(L2, HEADS * HD, device="cuda", dtype=torch.float16)
    gms = gpu_time(lambda: bb.joint_attention(q, k, v, out))
    qc, kc, vc = (np.ascontiguousarray(t.float().permute(1, 0, 2).cpu().numpy()) for t in (q, k, v))
    oc = np.zeros((L2, HEADS, HD), np.float32)
    with stdout_to_stderr():
        t0 = time.perf_counter()
        fast.orc_attention(qc.ctypes.data, kc.ctypes.data, vc.ctypes.data, L2, HEADS, HD,
                           float(HD ** -0.5), oc.ctypes.data)
        cms = 1000 * (time.perf_counter() - t0)
    emit("C2 joint attention, 24 heads x 128, L = 4352", 4.0 * L2 * L2 * HD * HEADS, gms, cms)

    # ---- C3: GEMM sweep
    for (Kd, N) in [(3072, 9216), (3072, 3072), (3072, 12288), (12288, 3072), (3072, 21504), (15360, 3072)]:
        packed = bb.random_b1_packed(N, Kd, rng)
        wgt = bb.B1Weight(packed, N, Kd)
        for M in (1280, 4352, 8704):
            x = torch.randn(M, Kd, device="cuda")
            x16 = x.half()
            o16 = torch.empty(M, N, device="cuda", dtype=torch.float16)
            gms = gpu_time(lambda: bb.b1_gemm(x16, wgt, bb.BONSAI_EPI_F16, o16))
            xc = np.ascontiguousarray(x.cpu().numpy())
            oc = np.zeros((M, N), np.float32)
            with stdout_to_stderr():
                t0 = time.perf_counter()
                R.ref_b1_linear(xc.ctypes.data, M, Kd, packed.ctypes.data, N, oc.ctypes.data, threads)
                cms = 1000 * (time.perf_counter() - t0)
            emit(f"C3 GEMM M={M} K={Kd} N={N}", 2.0 * M * N * Kd, gms, cms)
        wgt.free()
    return results


def vae_flops(lh: int, lw: int, folded: bool) -> float:
    """FLOPs of one decode of a lh x lw encoded latent: convolutions 2*P*Cin*Cout*k^2
    (folded = the upsampling convs as four 2x2 phase convolutions, as executed;
    else 3x3 over the upsampled image, as the reference computes them), the
    attention projections and products (4*S^2*C)."""
    H0, W0 = 2 * lh, 2 * lw
    P = H0 * W0
    f = 2.0 * P * 32 * 32 + 2.0 * P * 32 * 512 * 9            # post_quant, conv_in
    res = lambda p, ci, co: 2.0 * p * (ci * co * 9 + co * co * 9 + (ci * co if ci != co else 0))
    f += 2 * res(P, 512, 512) + 4 * 2.0 * P * 512 * 512 + 4.0 * P * P * 512  # mid block
    ins, outs = [512, 512, 512, 256], [512, 512, 256, 128]
    for i in range(4):
        f += res(P, ins[i], outs[i]) + 2 * res(P, outs[i], outs[i])
        if i < 3:
            f += 2.0 * P * outs[i] * outs[i] * (16 if folded else 36)
            P *= 4
    return f + 2.0 * P * 128 * 3 * 9


def run_vae(args):
    """--vae: the VAE decode as the bench line (see measure_vae)."""
    emit_json(measure_vae(args.steps, args.warmup, not args.no_cpu_baseline,
                          os.environ.get("BONSAI_CLOCK_LOG")))
    return 0


def measure_vae(steps: int, warmup: int, cpu_baseline: bool, clock_log=None) -> dict:
    """The Flux VAE decoder (the stage after the denoise loop in the
    reference's pipeline, src/vae_decoder.cpp + src/vae_graph.cpp) decoding a
    64 x 64 x 128 encoded latent to a 1024^2 image on one GPU, synthetic
    seeded weights.  value = device-timed ms per decode (latent resident);
    e2e = bonsai_vae_decode_host (latent copied in, image copied out);
    cpu_baseline = the f32 NumPy restatement of the reference's decoder
    (oracle/vae_oracle.py; the reference's own ggml path is not in its tree)
    on an 8 x 8 latent (128^2 image), scaled to the 1024^2 decode by FLOPs."""
    import torch
    import bonsai_b200 as bb
    torch.cuda.init()
    bb.init(0)
    lh = lw = 64
    K, W = steps, max(3, warmup)
    v = bb.Vae(lh, lw, seed=1234)
    rng = np.random.default_rng(7)
    lat_h = torch.from_numpy(rng.uniform(-1, 1, (128, lh, lw)).astype(np.float32)).pin_memory()
    lat = lat_h.cuda()
    img = torch.empty(3, 16 * lh, 16 * lw, device="cuda")
    for _ in range(W):
        v.decode(lat, img)
    torch.cuda.synchronize()
    assert bb.device_error() == 0
    stream = torch.cuda.current_stream()
    clocks = ClockSampler(0, clock_log)
    clocks.start()
    bb.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        v.decode(lat, img)
    e1.record(stream)
    torch.cuda.synchronize()
    launches = bb.launch_count()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / K
    assert bb.device_error() == 0
    bb.profile_start()
    for _ in range(K):
        v.decode(lat, img)
    prof = bb.profile_stop()
    finite = bb.count_nonfinite(img) == 0
    lat_np = lat_h.numpy()
    v.decode_host(lat_np)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(K):
        out_np = v.decode_host(lat_np)
    f1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1) / K
    pk = peaks()
    convs = {k: e for k, e in prof.items() if k.startswith(("vae_conv", "vae_attn_gemm"))}
    c_flop = sum(e["flop"] for e in convs.values())
    c_ms = sum(e["ms"] for e in convs.values())
    conv_tf = c_flop / (c_ms / 1e3) / 1e12
    gn = prof.get("vae_gn_apply", {})
    total = sum(e["ms"] for e in prof.values())
    line = {
        "metric": "ms/VAE decode @1024² (Flux VAE decoder, latent 128x64x64 -> 3x1024x1024)",
        "value": round(ms, 3), "unit": "ms", "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16/bf16 operands, f32 accumulate and residual",
        "data": "synthetic (seeded weights, U(-1,1) latent)",
        "config": {"workload": "Flux VAE decoder, 1024^2 image (src/vae_graph.cpp:174-212)",
                   "latent": [128, lh, lw], "image": [3, 16 * lh, 16 * lw],
                   "decode_tflop_reference_form": round(vae_flops(lh, lw, False) / 1e12, 3),
                   "decode_tflop_executed": round(vae_flops(lh, lw, True) / 1e12, 3),
                   "l2": "activations of 0.5-1 GB per tensor stream through HBM"},
        "roofline": {"bound": "tensor", "kernel": "vae conv (implicit-GEMM tcgen05)",
                     "achieved": round(conv_tf, 1), "peak": pk["bf16_sustained"], "unit": "TFLOP/s",
                     "frac": round(conv_tf / pk["bf16_sustained"], 4),
                     "peak_kind": f"{pk['source']} sustained bf16", "traffic": None,
                     "measured": "sum of executed conv/GEMM FLOPs / sum of their CUDA-event durations"},
        "gn_apply_gbs": round(gn["bytes"] / (gn["ms"] / 1e3) / 1e9, 1) if gn else None,
        "kernels_per_decode": {k: {"launches": e["launches"] / K, "ms": round(e["ms"] / K, 4),
                                   "share": round(e["ms"] / total, 4)} for k, e in prof.items()},
        "gpu_launches": launches, "clocks": clk,
        "e2e": {"value": round(ms_e2e, 3), "unit": "ms", "h2d_bytes_per_step": 128 * lh * lw * 4,
                "d2h_bytes_per_step": 3 * 256 * lh * lw * 4,
                "output_finite": bool(finite and np.isfinite(out_np).all())},
    }
    v.close()
    if cpu_baseline:
        from oracle import vae_oracle as vo
        sys.path.insert(0, str(ROOT / "tests"))
        from vae_weights import make_state_dict
        sd = make_state_dict(1234)
        s_lat = rng.uniform(-1, 1, (128, 8, 8)).astype(np.float32)
        t0 = time.perf_counter()
        vo.decode(sd, s_lat)
        s_sec = time.perf_counter() - t0
        scale = vae_flops(lh, lw, False) / vae_flops(8, 8, False)
        line["cpu_baseline"] = {"value": round(s_sec * 1e3 * scale, 1), "unit": "ms",
                                "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"NumPy f32 restatement, 8x8 latent (128^2 image) in "
                                          f"{s_sec:.2f} s, scaled x{scale:.1f} by FLOPs"}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["bonsai", "reference"], default="bonsai")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["1024", "2048"], default="1024",
                    help="1024: config 4, one image per GPU (data parallel, default); "
                         "2048: config 5(b), one 2048^2 image split by heads/rows across the GPUs")
    ap.add_argument("--exchange", choices=["fused", "scatter", "nccl"], default="scatter",
                    help="the 2048^2 split on N > 1 GPUs: exchanges fused into the kernels over "
                         "peer memory (fused: the LN-modulate kernel broadcasts xm rows; scatter: "
                         "the Q/K/V GEMM stores every head into its owner's buffer) or NCCL "
                         "collectives between the phases")
    ap.add_argument("--order", choices=["flags", "nccl"], default="flags",
                    help="the fused exchanges' ordering of the ranks after phases 0 and 1: the "
                         "engine's peer flag barrier (bonsai_dit_barrier) or a one-element NCCL "
                         "all-reduce")
    ap.add_argument("--no-side", action="store_true",
                    help="skip the 1-GPU side measurements (BASELINE configs 1-3 and the VAE "
                         "decode) that a default 1-GPU run adds to its line")
    ap.add_argument("--no-split", action="store_true",
                    help="skip the 2048^2 head/row-split measurement (split_2048) that every "
                         "default run adds beside the headline")
    ap.add_argument("--split-steps", type=int, default=10,
                    help="timed steps of the split_2048 measurement")
    ap.add_argument("--split-warmup", type=int, default=3)
    ap.add_argument("--configs", action="store_true",
                    help="instead of the step: BASELINE configs 1-3, GPU vs the reference CPU "
                         "path, one JSON line per config")
    ap.add_argument("--vae", action="store_true",
                    help="instead of the step: the Flux VAE decoder at 1024^2 (the next "
                         "pipeline stage), one JSON line")
    args = ap.parse_args()
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    if args.warmup < 3:
        args.warmup = 3
    if args.vae:
        if args.impl == "reference":
            emit_json({"impl": "reference", "unavailable":
                       "the reference's VAE decoder runs on ggml, which its tree does not "
                       "contain (empty llama.cpp submodule); see cpu_baseline of the --vae line"})
            return 0
        return run_vae(args)
    if args.configs:
        return run_configs(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_bonsai(args)


if __name__ == "__main__":
    sys.exit(main())
