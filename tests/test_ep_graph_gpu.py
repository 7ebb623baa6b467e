"""Expert parallelism through the graph executor: a MoE-layer graph whose
comm.moe_dispatch / comm.moe_combine name several ranks (src/ir/dialect/
kernel/ops.h:87-88; the rank list survives lowering, src/device/
device.cpp:108-121) run by kvm_run as one process per GPU. Each rank routes
its own tokens; the experts are split evenly over the ranks; the dispatch
result is the rank's receive buffer (T*top_k*ranks rows of capacity). Every
rank's output must equal, bit for bit, the same graph over one rank on that
rank's tokens (the GEMMs' per-row arithmetic does not depend on which rows
share a tile). Fusion passes on and off. Skipped with fewer GPUs than ranks."""
import json
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle

ROOT = Path(__file__).resolve().parent.parent
KVM_RUN = ROOT / "kvm_b200" / "_build" / "host" / "kvm_run"
T, H, E, F, K = 384, 256, 16, 128, 2

pytestmark = pytest.mark.gpu


def _t(dtype, shape):
    return f"kernel.tensor<dtype={dtype}, shape=[{','.join(map(str, shape))}]>"


def moe_graph(world):
    """The MoE layer graph over `world` ranks (world = 1: the one-GPU graph)."""
    ranks = ",".join(str(r) for r in range(world))
    R = T * K * world
    bf = "bf16"
    return f"""graph {{
  config {{ ranks = [{ranks}] }}
  ^moe(%x: {_t(bf, [T, H])}, %wr: {_t(bf, [H, E])}, %w1: {_t(bf, [E, H, F])}, %w3: {_t(bf, [E, H, F])}, %w2: {_t(bf, [E, F, H])}, %one: {_t(bf, [1])} {{fill = 1.0}}) {{
    %g: {_t('f32', [T, E])} = kernel.matmul(%x, %wr)
    %d: {_t(bf, [R, H])} = kernel.comm.moe_dispatch<ranks=[{ranks}]> {{top_k = {K}}} (%x, %g)
    %a: {_t(bf, [R, F])} = kernel.matmul(%d, %w1)
    %b: {_t(bf, [R, F])} = kernel.matmul(%d, %w3)
    %n: {_t(bf, [R, F])} = kernel.neg(%a)
    %e: {_t(bf, [R, F])} = kernel.exp(%n)
    %p: {_t(bf, [R, F])} = kernel.add(%e, %one)
    %s: {_t(bf, [R, F])} = kernel.div(%a, %p)
    %h: {_t(bf, [R, F])} = kernel.mul(%s, %b)
    %y: {_t(bf, [R, H])} = kernel.matmul(%h, %w2)
    %out: {_t(bf, [T, H])} = kernel.comm.moe_combine<ranks=[{ranks}]> (%y, %g)
    return %out
  }}
}}"""


def _run(graph, world, ind, outd, cdir, fuse):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", KVM_EXEC_NO_FUSION="0" if fuse else "1")
    cmd = [str(KVM_RUN), str(graph), "--inputs", str(ind), "--out", str(outd),
           "--warmup", "1", "--iters", "2"]
    if world > 1:
        procs = [subprocess.Popen(cmd + ["--rank", str(rk), "--world", str(world),
                                         "--comm-dir", str(cdir)],
                                  stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                                  env=env) for rk in range(world)]
    else:
        procs = [subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                  text=True, env=env)]
    outs = []
    try:
        for p in procs:
            outs.append(p.communicate(timeout=240))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, e
    return [json.loads(o.strip().splitlines()[-1]) for o, _ in outs]


@pytest.mark.parametrize("fuse", [True, False])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_graph_matches_one_rank(cuda, tmp_path, world, fuse):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    rng = np.random.default_rng(world)
    w = {"wr": oracle.normal_bf16(rng, (H, E), 0.05),
         "w1": oracle.normal_bf16(rng, (E, H, F), 0.05),
         "w3": oracle.normal_bf16(rng, (E, H, F), 0.05),
         "w2": oracle.normal_bf16(rng, (E, F, H), 0.05)}
    xs = [oracle.normal_bf16(rng, (T, H)) for _ in range(world)]
    ge = tmp_path / "ep.kvm"
    ge.write_text(moe_graph(world))
    g1 = tmp_path / "one.kvm"
    g1.write_text(moe_graph(1))
    ind, outd, cdir = tmp_path / "in", tmp_path / "out", tmp_path / "comm"
    cdir.mkdir()
    for rk in range(world):
        for d in (ind / f"r{rk}", outd / f"r{rk}", ind / f"one{rk}", outd / f"one{rk}"):
            d.mkdir(parents=True)
        for sub in (f"r{rk}", f"one{rk}"):
            xs[rk].tofile(ind / sub / "x.bin")
            for k, v in w.items():
                v.tofile(ind / sub / f"{k}.bin")
    summaries = _run(ge, world, ind, outd, cdir, fuse)
    steps = summaries[0]["steps"]
    assert "ep_dispatch" in steps and "ep_combine" in steps
    assert ("grouped_gemm_silu_gate" in steps) == fuse
    for rk in range(world):
        _run(g1, 1, ind / f"one{rk}", outd / f"one{rk}", cdir, fuse)
        got = np.fromfile(outd / f"r{rk}" / "out.bin", dtype=np.uint16)
        ref = np.fromfile(outd / f"one{rk}" / "out.bin", dtype=np.uint16)
        assert np.array_equal(got, ref), rk
