"""Benchmarks of the single-GPU configurations other than the MoE layer
(`python bench.py --workload gemm|mlp|fp8`). Each prints one JSON line in
bench.py's format.

  gemm  bf16 matmul A[1024,1024] x B[1024,1024] (kernel.matmul layout), fp32
        accumulate, bf16 out. Inputs (6 MB) fit in L2, so L2 is flushed (a
        256 MB write) before every timed launch and only the launch is timed.
  mlp   gated MLP block: x[4096,4096] -> RMSNorm (eps 1e-5, gamma 1) ->
        SiLU(x Wg) * (x Wu) with Wg, Wu [4096,14336] -> . Wd [14336,4096].
        352 MB of weights per step (> L2).
  fp8   W8A8 block-scaled GEMM [M,8192] x [8192,28672] e4m3 with 128x128 fp32
        scales, bf16 out, M in {16, 128, 1024}; 235 MB of weights (> L2).
Data: seeded torch.randn on the device, weights N(0, 0.02) (fp8: N(0,1)
quantised per block to amax 448).
"""
from __future__ import annotations

import json
import statistics
import time

import torch

from . import ops


def _time(fn, steps, warmup, flush=None):
    """Mean ms per launch (CUDA events on the current stream)."""
    for _ in range(warmup):
        if flush is not None:
            flush()
        fn()
    torch.cuda.synchronize()
    if flush is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps
    ts = []
    for _ in range(steps):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        ts.append((a, b))
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(b) for a, b in ts)


def _line(args, clocks, t0, t1, **kw):
    base = {"n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "data": "synthetic (seeded torch.randn, random-init weights)",
            "clocks": clocks.summary(t0, t1)}
    base.update(kw)
    print(json.dumps(base), flush=True)


def run(args, peaks, ClockSampler) -> int:
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    steps, warmup = args.steps, max(args.warmup, 3)
    if args.workload == "gemm":
        a = torch.randn((1024, 1024), generator=g, device=dev).to(torch.bfloat16)
        b = torch.randn((1024, 1024), generator=g, device=dev).to(torch.bfloat16)
        d = torch.empty((1024, 1024), dtype=torch.bfloat16, device=dev)
        scratch = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        with ClockSampler(0) as ck:
            t0 = time.time()
            ms = _time(lambda: ops.matmul(a, b, out=d), steps, warmup,
                       flush=lambda: scratch.fill_(1))
            t1 = time.time()
        flop = 2.0 * 1024 ** 3
        tf = flop / (ms / 1e3) / 1e12
        _line(args, ck, t0, t1, metric="GEMM TFLOP/s", value=tf, unit="TFLOP/s",
              ms_per_step=ms, dtype="bf16",
              config={"workload": "bf16_matmul_1024x1024x1024", "l2": "flushed before each launch"},
              roofline={"bound": "tensor", "achieved": tf, "peak": peaks["bf16"],
                        "unit": "TFLOP/s", "frac": tf / peaks["bf16"], "traffic": None},
              gpu_launches=steps)
        return 0
    if args.workload == "mlp":
        T, H, F = 4096, 4096, 14336
        x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
        wg = (torch.randn((F, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wu = (torch.randn((F, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wd = (torch.randn((H, F), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w13 = ops.pack_gate_up(wg, wu, layout="nk")
        del wg, wu
        xn = torch.empty_like(x)
        h = torch.empty((T, F), dtype=torch.bfloat16, device=dev)
        y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)

        def step():
            ops.rmsnorm(x, None, 1e-5, out=xn)
            ops.silu_gate_matmul(xn, w13, out=h)
            ops.matmul(h, wd, b_layout="nk", out=y)
        with ClockSampler(0) as ck:
            t0 = time.time()
            ms = _time(step, steps, warmup)
            t1 = time.time()
        t_gu = _time(lambda: ops.silu_gate_matmul(xn, w13, out=h), steps, warmup)
        flop = 2.0 * T * H * F * 3
        tf = flop / (ms / 1e3) / 1e12
        gu_tf = 2.0 * T * H * 2 * F / (t_gu / 1e3) / 1e12
        _line(args, ck, t0, t1, metric="gated MLP block TFLOP/s", value=tf, unit="TFLOP/s",
              ms_per_step=ms, dtype="bf16",
              config={"workload": "gated_mlp_T4096_H4096_F14336", "l2": "weights 352 MB > L2"},
              roofline={"bound": "tensor", "achieved": gu_tf, "peak": peaks["bf16_sustained"],
                        "unit": "TFLOP/s", "frac": gu_tf / peaks["bf16_sustained"],
                        "traffic": None, "kernel": "gate/up GEMM + fused SiLU-gate",
                        "ms": t_gu},
              gpu_launches=3 * steps)
        return 0
    # fp8
    K, N = 8192, 28672
    w = torch.randn((K, N), generator=g, device=dev)          # graph layout [K, N]
    wq_kn, sw_kn = ops.quantize_e4m3(w)
    del w
    wq, sw = ops.transpose_u8(wq_kn), ops.transpose_f32(sw_kn)  # one-time re-layout
    del wq_kn
    res = {}
    with ClockSampler(0) as ck:
        t0 = time.time()
        for M in (16, 128, 1024):
            a = torch.randn((M, K), generator=g, device=dev)
            aq, sa = ops.quantize_e4m3(a)
            d = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            ms = _time(lambda: ops.matmul_fp8(aq, sa, wq, sw, out=d), steps, warmup)
            flop = 2.0 * M * N * K
            byt = M * K + K * N + 4 * (sa.numel() + sw.numel()) + 2 * M * N
            res[M] = {"ms": ms, "tflops": flop / (ms / 1e3) / 1e12,
                      "gbs": byt / (ms / 1e3) / 1e9, "bytes": byt, "flop": flop}
        t1 = time.time()
    fp8_peak = 2 * peaks["bf16"]   # dense fp8 rate is twice bf16 on this part
    rows = {str(M): dict(r, frac_hbm=r["gbs"] / peaks["hbm"],
                         frac_fp8=r["tflops"] / fp8_peak) for M, r in res.items()}
    r16 = res[16]
    _line(args, ck, t0, t1, metric="FP8 W8A8 GEMM GB/s (M=16, HBM-bound)",
          value=r16["gbs"], unit="GB/s", ms_per_step=r16["ms"], dtype="e4m3",
          config={"workload": "fp8_w8a8_blockscaled_K8192_N28672", "per_m": rows,
                  "fp8_peak_tflops": f"{fp8_peak:.0f} (2 x measured bf16)"},
          roofline={"bound": "hbm", "achieved": r16["gbs"], "peak": peaks["hbm"],
                    "unit": "GB/s", "frac": r16["gbs"] / peaks["hbm"], "traffic": None},
          gpu_launches=3 * steps)
    return 0
