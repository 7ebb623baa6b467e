#!/usr/bin/env python
"""MoE-layer throughput benchmark (tokens/s) for the B200 execution backend.

Workload (one step = one MoE layer forward over one batch):
    tokens [8192, 4096] bf16 ~ N(0,1); router W [4096, 64] ~ N(0, 0.02);
    softmax top-2 over 64 experts; each expert a gated FFN 4096 -> 1408 -> 4096
    with weights ~ N(0, 0.02); dispatch, grouped GEMM, weighted combine.
Inputs are synthetic, seeded (torch generator seed 0), generated on the
device; weights are random-init with the layer's shapes. The working set
(2.2 GB of expert weights + 0.5 GB of activations per step) is far larger
than the 126 MB L2, so no flush is needed between timed steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torch.distributed (one process per GPU, NCCL): each rank
holds 8192 tokens (weak scaling) and the experts are sharded over the ranks
(expert parallel) with an all-to-all exchange of the routed token rows.

--impl reference times the CPU restatement of the layer (the reference
toolkit itself has no execution path) on this machine's host cores, on a
bounded token sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

TOKENS, HIDDEN, EXPERTS, FFN, TOP_K = 8192, 4096, 64, 1408, 2
METRIC = "MoE-layer tokens/s"
UNIT = "tokens/s"
CONFIG_NAME = "moe_layer_T8192_H4096_E64_F1408_top2"


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU baseline leg (rank 0, N=1)")
    ap.add_argument("--tokens", type=int, default=TOKENS,
                    help="tokens per rank (default: the headline 8192; smaller "
                         "values are profiling cases, not bench lines)")
    ap.add_argument("--experts", type=int, default=EXPERTS,
                    help="experts (default 64; profiling cases may use fewer)")
    ap.add_argument("--workload", choices=["moe", "gemm", "mlp", "fp8", "tp", "attn", "decode", "ew"],
                    default="moe",
                    help="moe (default, the headline line); gemm: bf16 1024^3 matmul; "
                         "mlp: gated MLP block 4096x4096->14336; fp8: W8A8 block-scaled "
                         "GEMM [M,8192]x[8192,28672] for M in 16,128,1024; tp: "
                         "tensor-parallel decoder layer (hidden 8192, batch 4 x 2048); "
                         "attn: the decoder layer's fused causal attention alone; "
                         "decode: paged decode attention, --seqs sequences x 4096 keys; "
                         "ew: generated fused elementwise programs (SiLU-gate, RMSNorm "
                         "scaling) vs the interpreter")
    ap.add_argument("--ep-exchange", choices=["overlap", "serial"], default="overlap",
                    help="N > 1: the all-to-all fused into the grouped GEMMs (default) "
                         "or the serial exchange kernels (for comparison)")
    ap.add_argument("--seqs", type=int, default=64,
                    help="decode workload: sequences per step (64; smaller values are "
                         "profiling cases)")
    args = ap.parse_args(argv)
    globals()["TOKENS"] = args.tokens
    globals()["EXPERTS"] = args.experts
    return args


def config_name() -> str:
    if TOKENS == 8192 and EXPERTS == 64:
        return CONFIG_NAME
    return f"profiling_case_T{TOKENS}_H{HIDDEN}_E{EXPERTS}_F{FFN}_top{TOP_K}"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"],
                    bf16_sustained=d["bf16_tflops_sustained"], src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, src="fallback")


# ----------------------------------------------------------- clock sampler ---

class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons in the background."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu_index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self

        def reader():
            for line in self.proc.stdout:
                self.samples.append((time.time(), [x.strip() for x in line.split(",")]))
        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self, t0: float, t1: float) -> dict:
        inside = [s for t, s in self.samples if t0 <= t <= t1]
        if not inside:   # timed region shorter than the sampling period
            inside = [s for t, s in self.samples if t0 - 0.25 <= t <= t1 + 0.25]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(s[1]) for s in inside if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in inside if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in inside for n, v in zip(names, s[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside)}


# --------------------------------------------------------------- our arm ---

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_weights(torch, dev, gen):
    wr = (torch.randn((EXPERTS, HIDDEN), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    w13 = torch.empty((EXPERTS, 2 * FFN, HIDDEN), dtype=torch.bfloat16, device=dev)
    w2 = torch.empty((EXPERTS, HIDDEN, FFN), dtype=torch.bfloat16, device=dev)
    for e in range(EXPERTS):   # chunked to bound the fp32 temporaries
        w13[e] = (torch.randn((2 * FFN, HIDDEN), generator=gen, device=dev) * 0.02)
        w2[e] = (torch.randn((HIDDEN, FFN), generator=gen, device=dev) * 0.02)
    return wr, w13, w2


def cpu_baseline_leg(x_dev, wr, w13, w2, min_s: float = 10.0) -> dict:
    """The oracle (CPU restatement of the layer) timed on the host cores: the
    whole token batch through the layer, repeated until >= min_s of work
    (at most 3 passes)."""
    import numpy as np
    import torch
    import oracle

    def bits(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

    xs, wrs, w13s, w2s = bits(x_dev), bits(wr), bits(w13), bits(w2)
    oracle.moe_layer(xs[:16], wrs, w13s, w2s, TOP_K)          # warm-up
    done, t0 = 0, time.perf_counter()
    while True:
        oracle.moe_layer(xs, wrs, w13s, w2s, TOP_K)
        done += 1
        dt = time.perf_counter() - t0
        if dt >= min_s or done >= 3:
            break
    n = done * xs.shape[0]
    return {"value": n / dt, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
            "sample": f"all {xs.shape[0]} tokens through the whole layer x{done} "
                      f"(same inputs and weights), {dt:.1f} s"}


def cpu_job(name, args, kw, units, unit, sample, max_reps, min_s=3.0):
    """CPU baseline of a kernel workload line: the oracle's `name` on the host
    cores over a bounded sample, repeated until min_s of work (at most
    max_reps); `units` of the line's unit per call."""
    import oracle
    if name == "mlp_rows":
        x, wg, wu, wd = args
        fn = lambda: oracle.gemm(oracle.gemm_silu_gate(oracle.rmsnorm(x, None, 1e-5), wg, wu),
                                 wd, b_layout="nk")
    else:
        f = getattr(oracle, name)
        fn = lambda: f(*args, **kw)
    fn()  # warm-up
    done, t0 = 0, time.perf_counter()
    while True:
        fn()
        done += 1
        dt = time.perf_counter() - t0
        if dt >= min_s or done >= max_reps:
            break
    return {"value": units * done / dt, "unit": unit, "cores": oracle.num_threads(),
            "kind": "port", "sample": f"{sample}, x{done} in {dt:.1f} s"}


# DRAM bytes (read + write) of one launch of the dominant kernel, from an ncu
# capture, with where the figure comes from (the summary file under profiles/
# gives the command that produced it).
GATE_UP_TRAFFIC = {
    "bytes": 1808847360.0,
    "src": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one gemm_pair_kernel<2> "
           "launch of this workload at full size (one-pass capture): "
           "profiles/moe_layer_kernels_T8192.md",
}


def roofline_entry(name, ms, flop=None, nbytes=None, pk=None, peak_kind="burst"):
    """One kernel's roofline: the binding bound (tensor if FLOP / peak takes
    longer than bytes / HBM peak, else HBM) and achieved = work / ms."""
    bf16 = pk["bf16_sustained"] if peak_kind == "sustained" else pk["bf16"]
    t_tensor = flop / (bf16 * 1e12) if flop else 0.0
    t_hbm = nbytes / (pk["hbm"] * 1e9) if nbytes else 0.0
    t = ms / 1e3
    if t_tensor >= t_hbm:
        e = {"bound": "tensor", "achieved": flop / t / 1e12, "peak": bf16, "unit": "TFLOP/s"}
        src = f"{pk['src']} ({peak_kind} bf16)"
    else:
        e = {"bound": "hbm", "achieved": nbytes / t / 1e9, "peak": pk["hbm"], "unit": "GB/s"}
        src = f"{pk['src']} (hbm copy)"
    e["frac"] = e["achieved"] / e["peak"]
    e.update({"kernel": name, "ms": ms, "flop": flop, "bytes": nbytes, "peak_src": src})
    return e


def layer_rooflines(phases: dict, world: int, pk: dict, peak_kind: str) -> list:
    """Roofline entries of the layer's kernels from their mean event times.
    Algorithmic work per launch (T tokens of this rank, k slots, E experts,
    E/P local, R = rows the rank's experts receive = T*k on average):
      router   x [T,H] + Wr [E,H] read, logits [T,E] f32 + top-k [T,k] (i32+f32)
               written; 2*T*H*E FLOP (HBM-bound)
      gate_up  2*R*2F*H FLOP; W13 [E/P,2F,H] + rows [R,H] read, H [R,F] written
      down     2*R*H*F FLOP;  W2 [E/P,H,F] + H [R,F] read, Y [R,H] written
      scatter  x [T,H] read, [T*k,H] written
      combine  [T*k,H] read, out [T,H] written
      ep_dispatch / ep_combine: the same bytes as scatter / combine, (P-1)/P of
               them over NVLink."""
    T, H, E, F, k = TOKENS, HIDDEN, EXPERTS, FFN, TOP_K
    R = T * k
    el = E // world
    work = {
        "router": (2.0 * T * H * E, T * H * 2 + E * H * 2 + T * E * 4 + T * k * 8),
        "gate_up": (2.0 * R * 2 * F * H, el * 2 * F * H * 2 + R * H * 2 + R * F * 2),
        "down": (2.0 * R * H * F, el * H * F * 2 + R * F * 2 + R * H * 2),
        "scatter": (None, T * H * 2 + R * H * 2),
        "combine": (None, R * H * 2 + T * H * 2),
        "ep_dispatch": (None, T * H * 2 + R * H * 2),
        "ep_combine": (None, R * H * 2 + T * H * 2),
    }
    # the overlapped exchange runs the all-to-all inside the grouped GEMMs
    work["ep_dispatch_gate_up"] = work["gate_up"]
    work["ep_down_push"] = work["down"]
    out = []
    for name, (flop, nbytes) in work.items():
        if name in phases and phases[name] > 0:
            out.append(roofline_entry(name, phases[name], flop, nbytes, pk, peak_kind))
    return out


def ep_parity(layer, x, wr, w13, w2, rank, world, n=256):
    """Bit-exact check of the expert-parallel layer: the first n tokens of
    every rank's batch, gathered on rank 0, through the one-GPU layer (which
    holds all E experts). Every rank takes part in the gather; rank 0 returns
    the comparison, the others None."""
    import torch
    import torch.distributed as dist
    from kvm_b200.moe import MoELayer
    out = layer(x)[:n].contiguous()
    xs = x[:n].contiguous()
    gx = [torch.empty_like(xs) for _ in range(world)]
    gy = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(gx, xs)
    dist.all_gather(gy, out)
    if rank != 0:
        return None
    ref_layer = MoELayer(wr, w13, w2, TOP_K, n * world)
    ref = ref_layer(torch.cat(gx))
    got = torch.cat(gy)
    same = torch.equal(ref.view(torch.int16), got.view(torch.int16))
    diff = (ref.float() - got.float()).abs().max().item()
    return {"bitexact": bool(same), "tokens_checked": n * world, "max_abs_diff": diff}


def graph_leg(args):
    """The same layer as a .kvm program through the drop-in path: the
    reference's parser and kernel->task transform with the sm_100a Device
    target, then the executor's launches (kvm_run, one process, its own
    seeded inputs of the graph's shapes), timed with CUDA events over
    args.steps runs. None when the host side is not built or the workload is
    a profiling case."""
    exe = ROOT / "kvm_b200" / "_build" / "host" / "kvm_run"
    g = ROOT / "kvm_b200" / "graphs" / "moe_layer.kvm"
    if not exe.exists() or TOKENS != 8192 or EXPERTS != 64:
        return None
    r = subprocess.run([str(exe), str(g), "--warmup", str(max(args.warmup, 3)),
                        "--iters", str(args.steps)], capture_output=True, text=True,
                       timeout=600)
    if r.returncode != 0:
        return {"error": (r.stderr or "").strip()[-300:]}
    d = json.loads(r.stdout.strip().splitlines()[-1])
    ms = d["ms_per_run"]
    return {"graph": "kvm_b200/graphs/moe_layer.kvm", "ms_per_run": ms,
            "tokens_per_s": TOKENS / (ms / 1e3), "launches_per_run": d["launch_steps"],
            "steps": d["steps"], "runs": d["iters"],
            "path": ".kvm text -> reference parser -> reference kernel->task transform "
                    "(sm_100a Device target) -> executor -> C ABI kernels"}


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world != args.gpus:
        print(f"--gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
        return 2
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        return 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)

    from kvm_b200 import _lib
    from kvm_b200.moe import MoELayer
    from kvm_b200.timing import PhaseProbe

    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    wr, w13, w2 = make_weights(torch, dev, gen)
    gen.manual_seed(1000 + rank)
    x = torch.randn((TOKENS, HIDDEN), generator=gen, device=dev).to(torch.bfloat16)

    if world > 1:
        from kvm_b200.ep import ExpertParallelMoE
        layer = ExpertParallelMoE(wr, w13, w2, top_k=TOP_K, max_tokens=TOKENS,
                                  rank=rank, world=world,
                                  overlap=args.ep_exchange == "overlap")
        if rank != 0:      # rank 0 keeps all experts for the parity check
            w13 = w2 = None
    else:
        layer = MoELayer(wr, w13, w2, TOP_K, TOKENS)
        w13 = w2 = None
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    probe = PhaseProbe(args.steps, layer.PHASES)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # ---- device-resident timing
    for _ in range(args.warmup):
        layer(x)
    _lib.device_status()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        wall0 = time.time()
        ev0.record(stream)
        for i in range(args.steps):
            layer(x)
        ev1.record(stream)
        torch.cuda.synchronize()
        wall1 = time.time()
        barrier()
    _lib.device_status()
    ms = ev0.elapsed_time(ev1)
    # per-launch times in a second pass of the same steps: events between the
    # launches would serialise them (no programmatic dependent launch), so the
    # timed loop above records none. The ranks start it together (stopping the
    # clock sampler takes a different time on each), else the first exchange
    # of the pass would absorb the difference.
    barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        layer(x, probe=probe.next_call())
    torch.cuda.synchronize()
    barrier()
    _lib.device_status()
    phases = probe.mean_ms()
    if world > 1:
        names = list(phases)
        t = torch.tensor([ms] + [phases[n] for n in names], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
        phases = {n: float(v) for n, v in zip(names, t[1:].tolist())}
    ms_per_step = ms / args.steps
    value = TOKENS * world * args.steps / (ms / 1e3)

    # ---- end to end through the public API: pinned host batches in, pinned
    # host results out, each step's copies overlapped with its neighbours'
    # compute (kvm_b200.pipeline.HostPipeline); every step still copies its
    # whole input in and its whole result out inside the timed region
    from kvm_b200.pipeline import HostPipeline
    pipe = HostPipeline(layer, TOKENS, HIDDEN, depth=2, device=dev)
    x_host = [x.cpu().pin_memory() for _ in range(2)]
    out_host = [torch.empty((TOKENS, HIDDEN), dtype=torch.bfloat16).pin_memory()
                for _ in range(2)]
    # at least 50 steps, so that filling and draining the three-stream
    # pipeline (one step's copy in, compute, copy out) is a small part
    e2e_steps = min(max(args.steps, 50), 200)
    for i in range(3):
        pipe.submit(x_host[i % 2], out_host[i % 2])
    pipe.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(pipe.h2d)
    for i in range(e2e_steps):
        pipe.submit(x_host[i % 2], out_host[i % 2])
    e1.record(pipe.d2h)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    e2e_value = TOKENS * world * e2e_steps / (e2e_ms / 1e3)
    _lib.device_status()

    parity = None
    if world > 1:
        parity = ep_parity(layer, x, wr, w13, w2, rank, world)
        _lib.device_status()

    # ---- roofline of the dominant kernel (grouped gate/up GEMM + SiLU-gate)
    # and of the others; the burst bf16 peak applies to a timed region of
    # under 2 s, the sustained one (power-capped clocks) to longer ones
    pk = peaks()
    peak_kind = "sustained" if ms / 1e3 >= 2.0 else "burst"
    entries = layer_rooflines(phases, world, pk, peak_kind)
    roof = dict(next(e for e in entries if e["kernel"] in ("gate_up", "ep_dispatch_gate_up")))
    roof["kernel"] = ("grouped gate/up GEMM + fused SiLU-gate on SM pairs (gemm_pair_kernel<2>)"
                      if roof["kernel"] == "gate_up" else
                      "dispatch all-to-all fused with the grouped gate/up GEMM + SiLU-gate "
                      "on SM pairs (gemm_pair_kernel<2, 1>)")
    headline = TOKENS == 8192 and EXPERTS == 64 and world == 1
    roof["traffic"] = GATE_UP_TRAFFIC["bytes"] if headline else None
    roof["traffic_src"] = GATE_UP_TRAFFIC["src"] if headline else None
    roof["timed_region_s"] = ms / 1e3

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_leg(x, layer.w_router, layer.w13, layer.w2)
    graph = graph_leg(args) if rank == 0 and world == 1 else None

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded torch.randn, random-init weights)",
            "config": {"workload": config_name(), "tokens_per_rank": TOKENS, "hidden": HIDDEN,
                       "experts": EXPERTS, "ffn": FFN, "top_k": TOP_K,
                       "parallelism": f"ep{world}" if world > 1 else "single",
                       **({"ep_exchange": args.ep_exchange} if world > 1 else {}),
                       "l2": "inputs larger than L2 (2.2 GB weights per step)"},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": TOKENS * HIDDEN * 2,
                    "d2h_bytes_per_step": TOKENS * HIDDEN * 2, "steps": e2e_steps,
                    "copies": "pinned host <-> HBM on two copy streams, overlapped with "
                              "the neighbouring steps' compute (HostPipeline, depth 2)"},
            "gpu_launches": layer.LAUNCHES_PER_CALL * args.steps,
            "roofline": roof,
            "kernels_ms": {n: round(v, 5) for n, v in phases.items()},
            "kernels_ms_src": "a second pass of the same steps with an event after each launch",
            "roofline_kernels": [{k: e[k] for k in ("kernel", "bound", "achieved", "peak",
                                                   "unit", "frac", "ms")}
                                 for e in entries],
            "cpu_baseline": cpu,
            "clocks": clocks.summary(wall0, wall1),
        }
        if parity is not None:
            line["ep_bitexact"] = parity["bitexact"]
            line["ep_parity"] = parity
        if graph is not None:
            line["kvm_graph"] = graph
        print(json.dumps(line), flush=True)
    if world > 1:
        layer.close()
        barrier()
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------- reference arm ---

def run_reference(args) -> int:
    """CPU restatement of the layer on the host cores, bounded sample/step."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    import numpy as np
    import oracle

    rng = np.random.default_rng(0)
    x = oracle.normal_bf16(rng, (1024, HIDDEN))
    wr = oracle.normal_bf16(rng, (EXPERTS, HIDDEN), 0.02)
    w13 = oracle.normal_bf16(rng, (EXPERTS, 2 * FFN, HIDDEN), 0.02)
    w2 = oracle.normal_bf16(rng, (EXPERTS, HIDDEN, FFN), 0.02)
    t = time.perf_counter()
    oracle.moe_layer(x[:64], wr, w13, w2, TOP_K)
    per_tok = (time.perf_counter() - t) / 64
    total_steps = args.steps + args.warmup
    sample = int(max(8, min(1024, 90.0 / total_steps / max(per_tok, 1e-6))))
    for _ in range(args.warmup):
        oracle.moe_layer(x[:sample], wr, w13, w2, TOP_K)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.moe_layer(x[:sample], wr, w13, w2, TOP_K)
    dt = time.perf_counter() - t0
    value = sample * args.steps / dt
    cores = oracle.num_threads()
    desc = (f"{sample} of the 8192 tokens per step through the whole layer; "
            "the reference has no execution path, so this is the oracle's C restatement")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": config_name(), "tokens_per_step_sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.workload != "moe":
        from kvm_b200 import bench_kernels
        if not args.no_cpu_baseline and int(os.environ.get("RANK", "0")) == 0:
            bench_kernels.CPU_LEG = cpu_job
        return bench_kernels.run(args, peaks(), ClockSampler)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
