"""Time one kernel of the step in isolation (and give ncu a small, fixed case).

    python -m bonsai_b200.kernel_bench gemm M K N [--kernel auto|pair|single]
                                       [--epi f16|f32|gelu|resid] [--flush] [--reps R]
    python -m bonsai_b200.kernel_bench attention L [--heads H] [--reps R]
    python -m bonsai_b200.kernel_bench conv H W CIN COUT [--k 3] [--bf16] [--reps R]
    python -m bonsai_b200.kernel_bench vae LATENT_H LATENT_W [--reps R]
    python -m bonsai_b200.kernel_bench ln_modulate ROWS [--reps R]
    python -m bonsai_b200.kernel_bench qk_norm_rope L [--heads H] [--reps R]
    python -m bonsai_b200.kernel_bench gemv N K [--reps R]

gemm: B1_0 GEMM of M tokens x K inputs -> N outputs (f16 store epilogue) on
seeded random weights/activations; attention: joint attention over L tokens,
H heads of 128; conv: one VAE decoder convolution (NHWC f16/bf16 in, f32
out, bias) on the implicit-GEMM kernel; vae: one whole decode of a
latent_h x latent_w latent (synthetic weights) with the per-kernel time
split; ln_modulate: LayerNorm + modulate of f32 [ROWS][3072] into f16
(bytes ROWS*3072*6); qk_norm_rope: Q/K RMSNorm + RoPE in place on f16
[H][L][128] (bytes H*L*128*4); gemv: the B1_0 matrix-vector kernel on one f32
row (the step's stacked modulation linear is N = 1050624, K = 3072; bytes
N*K*6/32 + 4K + 4N).  Prints one line: mean time per call over R
calls after 3 warm-up calls (CUDA events on the current stream) and the
TFLOP/s (GB/s for the two HBM-bound kernels).
"""
from __future__ import annotations

import argparse
import os
import sys


def _time(fn, reps: int) -> float:
    import torch
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="op", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("M", type=int)
    g.add_argument("K", type=int)
    g.add_argument("N", type=int)
    g.add_argument("--kernel", choices=["auto", "pair", "single"], default="auto")
    g.add_argument("--epi", choices=["f16", "f32", "gelu", "resid"], default="f16",
                   help="epilogue: f16 / f32 store, GELU-tanh -> f16, or the gate-residual "
                        "f32 read-modify-write of the out-projection / MLP-out linears")
    g.add_argument("--flush", action="store_true",
                   help="write a 256 MB buffer before every call, so the weights and "
                        "activations come from DRAM as in the step (which streams 2.2 GB "
                        "of weights) instead of from the 126 MB L2")
    g.add_argument("--reps", type=int, default=10)
    a = sub.add_parser("attention")
    a.add_argument("L", type=int)
    a.add_argument("--heads", type=int, default=24)
    a.add_argument("--reps", type=int, default=10)
    c = sub.add_parser("conv")
    c.add_argument("H", type=int)
    c.add_argument("W", type=int)
    c.add_argument("cin", type=int)
    c.add_argument("cout", type=int)
    c.add_argument("--k", type=int, default=3)
    c.add_argument("--bf16", action="store_true")
    c.add_argument("--reps", type=int, default=10)
    vae = sub.add_parser("vae")
    vae.add_argument("lh", type=int)
    vae.add_argument("lw", type=int)
    vae.add_argument("--reps", type=int, default=5)
    ln = sub.add_parser("ln_modulate")
    ln.add_argument("rows", type=int)
    ln.add_argument("--reps", type=int, default=20)
    qk = sub.add_parser("qk_norm_rope")
    qk.add_argument("L", type=int)
    qk.add_argument("--heads", type=int, default=48)
    qk.add_argument("--reps", type=int, default=20)
    gv = sub.add_parser("gemv")
    gv.add_argument("N", type=int)
    gv.add_argument("K", type=int)
    gv.add_argument("--reps", type=int, default=20)
    args = ap.parse_args(argv)
    nbytes = 0.0

    import numpy as np
    import torch
    import bonsai_b200 as bb
    torch.cuda.init()
    bb.init(0)
    if args.op == "gemm":
        if args.kernel != "auto":
            os.environ["BONSAI_B1_KERNEL"] = args.kernel
        w = bb.B1Weight(bb.random_b1_packed(args.N, args.K, np.random.default_rng(1)), args.N, args.K)
        x = torch.randn(args.M, args.K, device="cuda").half()
        mode, odt = {"f16": (bb.BONSAI_EPI_F16, torch.float16), "f32": (bb.BONSAI_EPI_F32, torch.float32),
                     "gelu": (bb.BONSAI_EPI_GELU, torch.float16),
                     "resid": (bb.BONSAI_EPI_RESID, torch.float32)}[args.epi]
        out = torch.zeros(args.M, args.N, device="cuda", dtype=odt)
        gate = torch.full((args.N,), 1e-3, device="cuda") if args.epi == "resid" else None
        flush = torch.empty(64 << 20, device="cuda") if args.flush else None

        def call():
            if flush is not None:
                flush.zero_()
            bb.b1_gemm(x, w, mode, out, gate=gate)
        if flush is None:
            ms = _time(call, args.reps)
        else:  # the GEMM alone, timed by the library's per-launch events
            _time(call, 1)
            bb.profile_start()
            for _ in range(args.reps):
                call()
            e = bb.profile_stop()["b1_gemm"]
            ms = e["ms"] / e["launches"]
        flop = 2.0 * args.M * args.N * args.K
        desc = (f"gemm M={args.M} K={args.K} N={args.N} kernel={args.kernel} epi={args.epi}"
                + (" flushed" if flush is not None else ""))
    elif args.op == "conv":
        td = torch.bfloat16 if args.bf16 else torch.float16
        x = torch.randn(args.H, args.W, args.cin, device="cuda").to(td)
        w = torch.randn(args.cout, args.cin, args.k, args.k, device="cuda") * 0.02
        b = torch.randn(args.cout, device="cuda")
        out = torch.empty(args.H, args.W, args.cout, device="cuda")
        # bonsai_conv2d_nhwc converts the f32 weights every call; time the
        # convolution kernel alone with the library's per-launch events.
        _time(lambda: bb.conv2d_nhwc(x, w, b, out), 1)
        bb.profile_start()
        for _ in range(args.reps):
            bb.conv2d_nhwc(x, w, b, out)
        prof = bb.profile_stop()
        e = next(v for k, v in prof.items() if k.startswith("vae_conv"))
        ms = e["ms"] / e["launches"]
        flop = 2.0 * args.H * args.W * args.cin * args.cout * args.k * args.k
        desc = f"conv {args.H}x{args.W} {args.cin}->{args.cout} k={args.k} {'bf16' if args.bf16 else 'f16'}"
    elif args.op == "ln_modulate":
        R = args.rows
        x = torch.randn(R, 3072, device="cuda")
        sh = torch.randn(3072, device="cuda")
        sc = torch.randn(3072, device="cuda")
        y = torch.empty(R, 3072, device="cuda", dtype=torch.float16)
        ms = _time(lambda: bb.check(bb.lib().bonsai_ln_modulate(
            x.data_ptr(), R, 3072, sh.data_ptr(), sc.data_ptr(), 1e-6, y.data_ptr(), 3072,
            bb.stream_ptr()), "bonsai_ln_modulate"), args.reps)
        flop, nbytes = 0.0, R * 3072 * 6.0
        desc = f"ln_modulate rows={R} dim=3072"
    elif args.op == "qk_norm_rope":
        H, L = args.heads, args.L
        qkt = torch.randn(H, L, 128, device="cuda").half()
        w = torch.ones(128, device="cuda")
        cs = torch.rand(L, 64, device="cuda")
        sn = torch.rand(L, 64, device="cuda")
        ms = _time(lambda: bb.check(bb.lib().bonsai_qk_norm_rope(
            qkt.data_ptr(), H, L, 128, w.data_ptr(), w.data_ptr(), 0, 1e-6, cs.data_ptr(),
            sn.data_ptr(), bb.stream_ptr()), "bonsai_qk_norm_rope"), args.reps)
        flop, nbytes = 0.0, H * L * 128 * 4.0
        desc = f"qk_norm_rope heads={H} L={L}"
    elif args.op == "gemv":
        import numpy as np
        N, K = args.N, args.K
        nb = K // 32
        g = torch.Generator().manual_seed(1)
        raw = torch.randint(0, 256, (N, nb, 6), dtype=torch.uint8, generator=g)
        scales = (torch.randn(N, nb, generator=g).abs() * 0.02).half()
        raw[:, :, 0:2] = scales.view(torch.uint8).view(N, nb, 2)
        w = bb.B1Weight(raw.reshape(N, nb * 6).numpy(), N, K)
        del raw, scales
        x = torch.randn(1, K, device="cuda")
        y = torch.empty(1, N, device="cuda")
        ms = _time(lambda: bb.b1_linear_f32(x, w, y), args.reps)
        flop, nbytes = 2.0 * N * K, N * K * 6.0 / 32 + 4.0 * (K + N)
        desc = f"gemv N={N} K={K}"
    elif args.op == "vae":
        import json
        v = bb.Vae(args.lh, args.lw, seed=1)
        lat = torch.rand(128, args.lh, args.lw, device="cuda") * 2 - 1
        img = torch.empty(3, 16 * args.lh, 16 * args.lw, device="cuda")
        ms = _time(lambda: v.decode(lat, img), args.reps)
        bb.profile_start()
        v.decode(lat, img)
        prof = bb.profile_stop()
        v.close()
        tot = sum(e["ms"] for e in prof.values())
        for name, e in sorted(prof.items(), key=lambda kv: -kv[1]["ms"]):
            tf = e["flop"] / (e["ms"] / 1e3) / 1e12 if e["ms"] > 0 else 0.0
            gbs = e["bytes"] / (e["ms"] / 1e3) / 1e9 if e["ms"] > 0 else 0.0
            print(json.dumps({"kernel": name, "launches": e["launches"], "ms": round(e["ms"], 3),
                              "share": round(e["ms"] / tot, 3), "tflops": round(tf, 1),
                              "gbs": round(gbs, 1)}))
        flop = sum(e["flop"] for e in prof.values())
        desc = f"vae decode latent {args.lh}x{args.lw} -> {16 * args.lh}x{16 * args.lw}"
    else:
        H, L = args.heads, args.L
        q, k, v = (torch.randn(H, L, 128, device="cuda").half() for _ in range(3))
        out = torch.empty(L, H * 128, device="cuda", dtype=torch.float16)
        ms = _time(lambda: bb.joint_attention(q, k, v, out), args.reps)
        flop = 4.0 * L * L * 128 * H
        desc = f"attention L={L} heads={H}"
    err = bb.device_error()
    rate = (f"{nbytes / (ms / 1e3) / 1e9:.0f} GB/s" if nbytes else
            f"{flop / (ms / 1e3) / 1e12:.1f} TFLOP/s")
    print(f"{desc}: {ms * 1e3:.1f} us/call, {rate}, device_error={err}")
    return 0 if err == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
