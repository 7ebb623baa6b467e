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
  attn  the decoder layer's causal GQA attention alone: q [4*2048, 64*128],
        k/v [4*2048, 8*128] bf16 (168 MB > L2), one fused launch.
  decode  one decode step of 64 sequences over a paged KV cache: 4096 cached
        tokens each, 64 query / 8 kv heads of 128 (the decoder layer's heads),
        16-token pages scattered over the pool (page_first); a step writes
        the new token's K/V (kvcache.write) and runs attn.decode over the
        4097 keys. 1.07 GB of K/V read per step (> L2).
Data: seeded torch.randn on the device, weights N(0, 0.02) (fp8: N(0,1)
quantised per block to amax 448).
"""
from __future__ import annotations

import json
import statistics
import time

import torch

from . import ops

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# each line's dominant kernel, from the ncu capture summarised in the named
# file under profiles/ (which gives the command), scaled where that capture
# ran a smaller case.
TRAFFIC = {
    "attn_fwd_B4_L2048_HQ64": (265392384.0, "ncu capture at the bench's own size"),
    "paged_decode_S16_ctx4096": (1105584128.0, "ncu capture of 16 sequences x4 to the "
                                               "bench's 64 (each sequence's keys once)"),
    "fused_elementwise_silu_8192x14336": (677293568.0, "ncu capture at the bench's own size"),
    "gemm_bf16_1024x1024x1024": (4226304.0, "ncu capture at the bench's own size"),
    "gated_mlp_T4096_H4096_F14336": (399734272.0, "ncu capture at the bench's own size"),
    "fp8_gemm_K8192_N28672": (244381440.0, "ncu capture at the bench's own size"),
}


def _bf16_peak(peaks, ms_per_step, steps):
    """(peak, source) for a timed region of steps x ms_per_step: the burst
    bf16 figure under 2 s, the sustained (power-capped) one from 2 s on."""
    if ms_per_step * steps / 1e3 >= 2.0:
        return peaks["bf16_sustained"], f"{peaks['src']} (sustained bf16)"
    return peaks["bf16"], f"{peaks['src']} (burst bf16)"


def _traffic(profile: str):
    """DRAM bytes per launch of a line's dominant kernel (TRAFFIC), or None."""
    t = TRAFFIC.get(profile)
    return t[0] if t else None


def _traffic_src(profile: str):
    t = TRAFFIC.get(profile)
    return f"{t[1]}: profiles/{profile}.md" if t else None


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


# Set by bench.py: runs a CPU-baseline job (the oracle on the host cores) and
# returns its cpu_baseline dict. This package never touches the oracle itself.
CPU_LEG = None


def _cpu_job(name, args, units, unit, sample, max_reps=20, **kw):
    """The CPU baseline of a line: job `name` on `args` processes `units` of the
    metric's unit per call; None when no CPU leg is wired in."""
    if CPU_LEG is None:
        return None
    return CPU_LEG(name, args, kw, units, unit, sample, max_reps)


def _bits(t):
    import numpy as np
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _l2_flusher(dev):
    """Evict L2 (126 MB) by reading 256 MB: the lines left behind are clean,
    so the timed kernel's misses do not also pay for write-backs of a flush."""
    buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    return lambda: torch.amax(buf)


def _line(args, clocks, t0, t1, **kw):
    base = {"n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "data": "synthetic (seeded torch.randn, random-init weights)",
            "clocks": clocks.summary(t0, t1)}
    base.update(kw)
    print(json.dumps(base), flush=True)


def run_tp(args, peaks, ClockSampler) -> int:
    """Tensor-parallel decoder layer: hidden 8192, 64 query / 8 kv heads of 128,
    batch 4 x seq 2048, FFN 28672; P ranks (torchrun), strong scaling."""
    import os
    import torch.distributed as dist
    from datetime import timedelta
    from .tp import TPDecoderLayer
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    B, L, H, HQ, HKV, FF = 4, 2048, 8192, 64, 8, 28672
    hq, hkv, fr = HQ // world, HKV // world, FF // world
    g = torch.Generator(device=dev)
    g.manual_seed(100 + rank)

    def rnd(*shape, std=0.02):
        return (torch.randn(shape, generator=g, device=dev) * std).to(torch.bfloat16)
    wqkv = rnd((hq + 2 * hkv) * 128, H)
    wo = rnd(H, hq * 128)
    w13 = torch.empty((2 * fr, H), dtype=torch.bfloat16, device=dev)
    for i in range(0, 2 * fr, 4096):
        w13[i:i + 4096] = rnd(min(4096, 2 * fr - i), H)
    w2 = rnd(H, fr)
    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    g.manual_seed(7)
    x = torch.randn((B * L, H), generator=g, device=dev).to(torch.bfloat16)
    layer = TPDecoderLayer(wqkv, wo, w13, w2, ones, ones, batch=B, seq_len=L, heads_q=HQ,
                           heads_kv=HKV, rank=rank, world=world)
    steps, warmup = args.steps, max(args.warmup, 3)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for _ in range(warmup):
        layer(x)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as ck:
        t0 = time.time()
        e0.record()
        for i in range(steps):
            layer(x, probe=ev[i])
        e1.record()
        torch.cuda.synchronize()
        t1 = time.time()
    ms = e0.elapsed_time(e1) / steps
    att_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    ar_ms = None
    if world > 1:
        buf = torch.randn((B * L, H), device=dev).to(torch.bfloat16)
        for _ in range(3):
            dist.all_reduce(buf)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            dist.all_reduce(buf)
        b.record()
        torch.cuda.synchronize()
        ar_ms = a.elapsed_time(b) / 10
        t = torch.tensor([ms, att_ms, ar_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, att_ms, ar_ms = (float(v) for v in t)
    T = B * L
    flop_lin = 2.0 * T * H * ((HQ + 2 * HKV) * 128 + HQ * 128 + 3 * FF)
    flop_att = 2.0 * 2.0 * B * HQ * L * L * 128 / 2
    tf = (flop_lin + flop_att) / (ms / 1e3) / 1e12
    att_tf = flop_att / world / (att_ms / 1e3) / 1e12
    if rank == 0:
        ar = None
        if ar_ms:
            nbytes = T * H * 2
            ar = {"ms": ar_ms, "algbw_gbs": nbytes / (ar_ms / 1e3) / 1e9,
                  "busbw_gbs": nbytes * 2 * (world - 1) / world / (ar_ms / 1e3) / 1e9}
        _line(args, ck, t0, t1, metric="TP decoder layer tokens/s", value=T / (ms / 1e3),
              unit="tokens/s", ms_per_step=ms, n_gpus=world, scaling="strong", dtype="bf16",
              config={"workload": "tp_decoder_H8192_HQ64_HKV8_B4_L2048_F28672",
                      "parallelism": f"tp{world}", "tflops_total": tf,
                      "tflops_per_gpu": tf / world, "attention_ms": att_ms,
                      "attention_tflops_per_gpu": att_tf, "allreduce_8192x8192_bf16": ar},
              roofline={"bound": "tensor", "achieved": tf / world,
                        "peak": _bf16_peak(peaks, ms, steps)[0], "unit": "TFLOP/s",
                        "frac": tf / world / _bf16_peak(peaks, ms, steps)[0],
                        "peak_src": _bf16_peak(peaks, ms, steps)[1], "traffic": None,
                        "kernel": "whole layer (GEMMs dominate)"},
              gpu_launches=layer.launches() * steps)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def run_attn(args, peaks, ClockSampler, dev, g) -> int:
    B, L, HQ, HKV = 4, 2048, 64, 8
    q = torch.randn((B * L, HQ * 128), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((B * L, HKV * 128), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((B * L, HKV * 128), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    steps, warmup = args.steps, max(args.warmup, 3)
    fn = lambda: ops.attention_prefill(q, k, v, batch=B, heads_q=HQ, heads_kv=HKV, out=out)
    with ClockSampler(0) as ck:
        t0 = time.time()
        ms = _time(fn, steps, warmup)
        t1 = time.time()
    # causal: keys 0..pos for each query -> 2 * (L (L + 1) / 2) * 128 * 2 per head
    flop = 4.0 * B * HQ * 128 * (L * (L + 1) / 2)
    tf = flop / (ms / 1e3) / 1e12
    grp = HQ // HKV
    cpu = _cpu_job("attention", (_bits(q[:, :grp * 128]), _bits(k[:, :128]), _bits(v[:, :128]),
                                 B, grp, 1),
                   flop * grp / HQ / 1e12, "TFLOP/s",
                   f"the {grp} query heads of kv head 0 (of {HQ}), all {B} x {L} rows",
                   max_reps=3)
    _line(args, ck, t0, t1, metric="causal attention TFLOP/s", value=tf, unit="TFLOP/s",
          ms_per_step=ms, dtype="bf16", cpu_baseline=cpu,
          config={"workload": f"causal_gqa_attention_B{B}_L{L}_HQ{HQ}_HKV{HKV}_hd128",
                  "l2": "168 MB of q/k/v > L2"},
          roofline={"bound": "tensor", "achieved": tf, "peak": peaks["bf16"],
                    "unit": "TFLOP/s", "frac": tf / peaks["bf16"],
                    "traffic": _traffic("attn_fwd_B4_L2048_HQ64"),
                    "traffic_src": _traffic_src("attn_fwd_B4_L2048_HQ64"),
                    "kernel": "attn_fwd_kernel"},
          gpu_launches=steps)
    return 0


def run_decode(args, peaks, ClockSampler, dev, g) -> int:
    from .kvcache import PagedKVCache
    S, ctx, HQ, HKV, bs = args.seqs, 4096, 64, 8, 16
    keys = ctx + 1
    per_seq = (keys + bs - 1) // bs
    pages = S * per_seq
    cache = PagedKVCache(pages=pages, layers=1, block_size=bs, heads_kv=HKV,
                         layout="page_first", device=dev)
    cache.pool.copy_(torch.randn(cache.pool.shape, generator=g, device=dev))
    perm = torch.randperm(pages, generator=g, device=dev).to(torch.int32)
    bt_off = (torch.arange(S + 1, device=dev, dtype=torch.int32) * per_seq)
    q_off = torch.arange(S + 1, device=dev, dtype=torch.int32)
    q_pos = torch.full((S,), ctx, device=dev, dtype=torch.int32)
    q = torch.randn((S, HQ * 128), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((S, HKV * 128), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((S, HKV * 128), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty((S, HQ * 128), dtype=torch.bfloat16, device=dev)
    from ._lib import lib
    ws = torch.empty(int(lib().kvm_sm100_attention_decode_workspace(S, HQ, HKV, 1, keys)),
                     dtype=torch.uint8, device=dev)
    steps, warmup = args.steps, max(args.warmup, 3)

    def step():
        cache.write(0, k, v, q_off, q_pos, perm, bt_off)
        cache.decode(0, q, q_off, q_pos, perm, bt_off, heads_q=HQ, max_q_rows=1,
                     max_keys=keys, out=out, workspace=ws)
    with ClockSampler(0) as ck:
        t0 = time.time()
        ms = _time(step, steps, warmup)
        t1 = time.time()
    kv_bytes = S * HKV * keys * 128 * 2 * 2
    byt = kv_bytes + 2 * S * HQ * 128 * 2 + 2 * S * HKV * 128 * 2
    gbs = byt / (ms / 1e3) / 1e9
    flop = 4.0 * S * HQ * keys * 128
    n_cpu = min(S, 8)
    cpu = _cpu_job("attention_decode",
                   (_bits(q[:n_cpu]), _bits(cache.pool), cache.strides, bs, 0,
                    q_off[:n_cpu + 1].cpu().numpy(), q_pos[:n_cpu].cpu().numpy(),
                    perm.cpu().numpy(), bt_off[:n_cpu + 1].cpu().numpy(), HQ, HKV),
                   byt * n_cpu / S / 1e9, "GB/s",
                   f"decode attention of {n_cpu} of the {S} sequences (K/V already written)",
                   max_reps=5)
    _line(args, ck, t0, t1, metric="paged decode attention GB/s", value=gbs, unit="GB/s",
          ms_per_step=ms, dtype="bf16", cpu_baseline=cpu,
          config={"workload": f"paged_decode_S{S}_ctx4096_HQ64_HKV8_hd128_bs16",
                  "kv_bytes_per_step": kv_bytes, "tflops": flop / (ms / 1e3) / 1e12,
                  "l2": f"{kv_bytes / 1e9:.2f} GB of K/V per step > L2"},
          roofline={"bound": "hbm", "achieved": gbs, "peak": peaks["hbm"], "unit": "GB/s",
                    "frac": gbs / peaks["hbm"],
                    "traffic": _traffic("paged_decode_S16_ctx4096") if S == 64 else None,
                    "traffic_src": _traffic_src("paged_decode_S16_ctx4096") if S == 64 else None,
                    "kernel": "decode_attn_kernel + combine + kvcache.write"},
          gpu_launches=3 * steps)
    return 0


SILU_PROGRAM = [("load", 0, 0, 0), ("load", 1, 0, 1), ("neg", 0, 0, 2), ("exp", 2, 0, 3),
                ("load", 2, 0, 4), ("add", 3, 4, 5), ("div", 0, 5, 6), ("mul", 6, 1, 7)]
NORM_PROGRAM = [("load", 0, 0, 0), ("load", 1, 0, 1), ("mul", 0, 1, 2), ("load", 2, 0, 3),
                ("mul", 2, 3, 4)]


def run_ew(args, peaks, ClockSampler, dev, g) -> int:
    """Generic fused elementwise programs (kernels generated per program):
    SiLU(g) * u over [8192, 14336] bf16 (the MoE/MLP gate shape) and the
    RMSNorm scaling x * r[T, 1] * gamma[H] over [8192, 4096]; the interpreter
    kernel (KVM_SM100_EW_JIT=0) timed beside it."""
    import os
    T, F, H = 8192, 14336, 4096
    gt = torch.randn((T, F), generator=g, device=dev).to(torch.bfloat16)
    ut = torch.randn((T, F), generator=g, device=dev).to(torch.bfloat16)
    one = torch.ones((), dtype=torch.float32, device=dev)
    ht = torch.empty((T, F), dtype=torch.bfloat16, device=dev)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    r = torch.rand((T, 1), generator=g, device=dev)
    gamma = torch.randn((H,), generator=g, device=dev).to(torch.bfloat16)
    y = torch.empty_like(x)
    steps, warmup = args.steps, max(args.warmup, 3)
    flush = _l2_flusher(dev)
    silu = lambda: ops.elementwise(SILU_PROGRAM, [gt, ut, one], (T, F), out=ht)
    norm = lambda: ops.elementwise(NORM_PROGRAM, [x, r, gamma], (T, H), out=y)
    with ClockSampler(0) as ck:
        t0 = time.time()
        ms = _time(silu, steps, warmup)
        t1 = time.time()
    ms_norm = _time(norm, steps, warmup, flush=flush)
    os.environ["KVM_SM100_EW_JIT"] = "0"
    try:
        ms_i = _time(silu, max(steps // 4, 3), warmup)
        ms_norm_i = _time(norm, max(steps // 4, 3), warmup, flush=flush)
    finally:
        del os.environ["KVM_SM100_EW_JIT"]
    byt = 3 * 2 * T * F
    gbs = byt / (ms / 1e3) / 1e9
    norm_bytes = 2 * 2 * T * H + 4 * T + 2 * H
    n_cpu = 1 << 22
    cpu = _cpu_job("elementwise",
                   (SILU_PROGRAM, [(_bits(gt.view(-1)[:n_cpu]), "bf16"),
                                   (_bits(ut.view(-1)[:n_cpu]), "bf16"),
                                   (one.view(1).cpu().numpy(), "f32")],
                    [(n_cpu, 1), (n_cpu, 1), (1, 1)], "bf16", 7, n_cpu),
                   6.0 * n_cpu / 1e9, "GB/s",
                   f"the program over {n_cpu} of the {T * F} elements", max_reps=5)
    _line(args, ck, t0, t1, metric="fused elementwise GB/s", value=gbs, unit="GB/s",
          ms_per_step=ms, dtype="f32 registers, bf16 in/out", cpu_baseline=cpu,
          config={"workload": f"silu_gate_program_{T}x{F}_bf16",
                  "bytes_per_step": byt, "l2": f"{byt / 1e9:.2f} GB per step > L2",
                  "interpreter_ms": ms_i,
                  "rmsnorm_scale_program": {"shape": [T, H], "ms": ms_norm,
                                            "gbs": norm_bytes / (ms_norm / 1e3) / 1e9,
                                            "interpreter_ms": ms_norm_i,
                                            "l2": "flushed before each launch"}},
          roofline={"bound": "hbm", "achieved": gbs, "peak": peaks["hbm"], "unit": "GB/s",
                    "frac": gbs / peaks["hbm"],
                    "traffic": _traffic("fused_elementwise_silu_8192x14336"),
                    "traffic_src": _traffic_src("fused_elementwise_silu_8192x14336"),
                    "kernel": "kvm_ew (generated)"},
          gpu_launches=steps)
    return 0


def run(args, peaks, ClockSampler) -> int:
    if args.workload == "tp":
        return run_tp(args, peaks, ClockSampler)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    steps, warmup = args.steps, max(args.warmup, 3)
    if args.workload == "gemm":
        a = torch.randn((1024, 1024), generator=g, device=dev).to(torch.bfloat16)
        b = torch.randn((1024, 1024), generator=g, device=dev).to(torch.bfloat16)
        d = torch.empty((1024, 1024), dtype=torch.bfloat16, device=dev)
        flush = _l2_flusher(dev)
        with ClockSampler(0) as ck:
            t0 = time.time()
            ms = _time(lambda: ops.matmul(a, b, out=d), steps, warmup, flush=flush)
            t1 = time.time()
        flop = 2.0 * 1024 ** 3
        tf = flop / (ms / 1e3) / 1e12
        cpu = _cpu_job("gemm", (_bits(a), _bits(b)), flop / 1e12, "TFLOP/s",
                       "the whole 1024^3 product")
        _line(args, ck, t0, t1, metric="GEMM TFLOP/s", value=tf, unit="TFLOP/s",
              ms_per_step=ms, dtype="bf16", cpu_baseline=cpu,
              config={"workload": "bf16_matmul_1024x1024x1024",
                      "l2": "flushed before each launch (256 MB read)"},
              roofline={"bound": "tensor", "achieved": tf, "peak": peaks["bf16"],
                        "unit": "TFLOP/s", "frac": tf / peaks["bf16"],
                        "traffic": _traffic("gemm_bf16_1024x1024x1024"),
                        "traffic_src": _traffic_src("gemm_bf16_1024x1024x1024")},
              gpu_launches=steps)
        return 0
    if args.workload == "decode":
        return run_decode(args, peaks, ClockSampler, dev, g)
    if args.workload == "ew":
        return run_ew(args, peaks, ClockSampler, dev, g)
    if args.workload == "attn":
        return run_attn(args, peaks, ClockSampler, dev, g)
    if args.workload == "mlp":
        T, H, F = 4096, 4096, 14336
        x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
        wg = (torch.randn((F, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wu = (torch.randn((F, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wd = (torch.randn((H, F), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w13 = ops.pack_gate_up(wg, wu, layout="nk")
        wg_keep, wu_keep = wg, wu  # for the CPU leg
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
        rows = 128
        cpu = _cpu_job("mlp_rows", (_bits(x[:rows]), _bits(wg_keep), _bits(wu_keep), _bits(wd)),
                       2.0 * rows * H * F * 3 / 1e12, "TFLOP/s",
                       f"{rows} of the {T} token rows through the block (rows are independent)")
        _line(args, ck, t0, t1, metric="gated MLP block TFLOP/s", value=tf, unit="TFLOP/s",
              ms_per_step=ms, dtype="bf16",
              cpu_baseline=cpu,
              config={"workload": "gated_mlp_T4096_H4096_F14336", "l2": "weights 352 MB > L2"},
              roofline={"bound": "tensor", "achieved": gu_tf, "peak": _bf16_peak(peaks, ms, steps)[0],
                        "unit": "TFLOP/s", "frac": gu_tf / _bf16_peak(peaks, ms, steps)[0],
                        "peak_src": _bf16_peak(peaks, ms, steps)[1],
                        "traffic": _traffic("gated_mlp_T4096_H4096_F14336"),
                        "traffic_src": _traffic_src("gated_mlp_T4096_H4096_F14336"),
                        "kernel": "gate/up GEMM + fused SiLU-gate",
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
            from ._lib import lib
            wsz = int(lib().kvm_sm100_gemm_fp8_workspace(M, N, K))
            ws = torch.empty(max(wsz, 16), dtype=torch.uint8, device=dev)
            ms = _time(lambda: ops.matmul_fp8(aq, sa, wq, sw, out=d, workspace=ws), steps,
                       warmup)
            flop = 2.0 * M * N * K
            byt = M * K + K * N + 4 * (sa.numel() + sw.numel()) + 2 * M * N
            res[M] = {"ms": ms, "tflops": flop / (ms / 1e3) / 1e12,
                      "gbs": byt / (ms / 1e3) / 1e9, "bytes": byt, "flop": flop}
        t1 = time.time()
    fp8_peak = 2 * peaks["bf16"]   # dense fp8 rate is twice bf16 on this part
    rows = {str(M): dict(r, frac_hbm=r["gbs"] / peaks["hbm"],
                         frac_fp8=r["tflops"] / fp8_peak) for M, r in res.items()}
    r16 = res[16]
    a16 = torch.randn((16, K), generator=g, device=dev)
    aq16, sa16 = ops.quantize_e4m3(a16)
    cpu = _cpu_job("gemm_fp8_blockscaled", (aq16.cpu().numpy(), sa16.cpu().numpy(),
                                            wq.cpu().numpy(), sw.cpu().numpy()),
                   r16["bytes"] / 1e9, "GB/s", "the whole M = 16 product", max_reps=5)
    _line(args, ck, t0, t1, metric="FP8 W8A8 GEMM GB/s (M=16, HBM-bound)",
          value=r16["gbs"], unit="GB/s", ms_per_step=r16["ms"], dtype="e4m3",
          cpu_baseline=cpu,
          config={"workload": "fp8_w8a8_blockscaled_K8192_N28672", "per_m": rows,
                  "fp8_peak_tflops": f"{fp8_peak:.0f} (2 x measured bf16)"},
          roofline={"bound": "hbm", "achieved": r16["gbs"], "peak": peaks["hbm"],
                    "unit": "GB/s", "frac": r16["gbs"] / peaks["hbm"],
                    "traffic": _traffic("fp8_gemm_K8192_N28672"),
                        "traffic_src": _traffic_src("fp8_gemm_K8192_N28672")},
          gpu_launches=3 * steps)
    return 0
