"""The kernel dialect's collectives (comm.all_reduce.sum/max, all_gather,
all_to_all, broadcast, send/recv; src/ir/dialect/kernel/dialect.cpp:58-64)
run by kvm_run as one process per GPU over NCCL, compared bit-exactly with
the same exchange done on the host: every case moves or compares values
without rounding (a sum of two f32 values is the same in either order)."""
import json
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle

ROOT = Path(__file__).resolve().parent.parent
KVM_RUN = ROOT / "kvm_b200" / "_build" / "host" / "kvm_run"
N = 4096      # f32 elements per rank


def _t(dtype, shape):
    return f"kernel.tensor<dtype={dtype}, shape=[{','.join(map(str, shape))}]>"


def comm_graph(world, n=N):
    ranks = ",".join(str(r) for r in range(world))
    f, b = "f32", "bf16"
    last = world - 1
    to = ",".join(str(r) for r in range(world) if r != last)
    return f"""graph {{
  config {{ ranks = [{ranks}] }}
  ^c(%x: {_t(f, [n])}, %z: {_t(b, [world, 512])}) {{
    %s: {_t(f, [n])} = kernel.comm.all_reduce.sum<ranks=[{ranks}]> (%x)
    %m: {_t(f, [n])} = kernel.comm.all_reduce.max<ranks=[{ranks}]> (%x)
    %g: {_t(f, [world, n])} = kernel.comm.all_gather<ranks=[{ranks}]> (%x)
    %a: {_t(b, [world, 512])} = kernel.comm.all_to_all<ranks=[{ranks}]> (%z)
    %b: {_t(f, [n])} = kernel.comm.broadcast<from={last}, to=[{to}]> (%x)
    %t: {_t(f, [n])} = kernel.comm.send<from=0, to={last}> (%x)
    %r: {_t(f, [n])} = kernel.comm.recv<from=0, to={last}> (%x)
    %p: {_t(f, [n])} = kernel.comm.all_reduce.sum<ranks=[0]> (%x)
    return %s, %m, %g, %a, %b, %t, %r, %p
  }}
}}"""


def test_comm_graph_lowers(tmp_path):
    """Every collective of the kernel dialect parses and lowers (task.comm.*)
    with its rank attributes intact; no GPU needed."""
    if not KVM_RUN.exists():
        pytest.fail("kvm_run is not built (python -c 'import __graft_entry__ as g; g.build()')")
    g = tmp_path / "c.kvm"
    g.write_text(comm_graph(2, 256))
    r = subprocess.run([str(KVM_RUN), str(g), "--lower-only", "--dump-task"],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert json.loads(r.stdout.strip().splitlines()[-1])["task_ops"] == 8
    for op in ("task.comm.all_reduce.sum<ranks=[0,1]>", "task.comm.all_gather<ranks=[0,1]>",
               "task.comm.broadcast<from=1, to=[0]>", "task.comm.send<from=0, to=1>",
               "task.comm.recv<from=0, to=1>", "task.comm.all_to_all<ranks=[0,1]>"):
        assert op in r.stderr
    r = subprocess.run([str(KVM_RUN), str(g), "--world", "2", "--rank", "1"],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "--comm-dir" in r.stderr


def _expected(xs, zs, world):
    last = world - 1
    out = []
    for rk in range(world):
        a = np.stack([zs[p][rk] for p in range(world)])
        out.append({
            "s": np.sum(np.stack(xs), axis=0, dtype=np.float32) if world == 2 else None,
            "m": np.max(np.stack(xs), axis=0),
            "g": np.stack(xs),
            "a": a,
            "b": xs[last],
            "t": xs[rk],
            "r": xs[0] if rk == last else xs[rk],
            "p": xs[rk],
        })
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_collectives_over_nccl(cuda, tmp_path, world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    g = tmp_path / "c.kvm"
    g.write_text(comm_graph(world))
    rng = np.random.default_rng(5)
    xs = [rng.standard_normal(N).astype(np.float32) for _ in range(world)]
    zs = [oracle.f32_to_bf16(rng.standard_normal((world, 512)).astype(np.float32))
          for _ in range(world)]
    ind, outd, cdir = tmp_path / "in", tmp_path / "out", tmp_path / "comm"
    cdir.mkdir()
    for rk in range(world):
        (ind / f"r{rk}").mkdir(parents=True)
        (outd / f"r{rk}").mkdir(parents=True)
        xs[rk].tofile(ind / f"r{rk}" / "x.bin")
        zs[rk].tofile(ind / f"r{rk}" / "z.bin")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([str(KVM_RUN), str(g), "--inputs", str(ind), "--out", str(outd),
                               "--warmup", "1", "--iters", "2", "--rank", str(rk),
                               "--world", str(world), "--comm-dir", str(cdir)],
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                              env=env)
             for rk in range(world)]
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
    steps = json.loads(outs[0][0].strip().splitlines()[-1])["steps"]
    assert "comm_all_reduce_sum" in steps and "comm_send" in steps
    want = _expected(xs, zs, world)
    names = ["s", "m", "g", "a", "b", "t", "r", "p"]
    for rk in range(world):
        d = outd / f"r{rk}"
        for k in names:
            path = d / f"{k}.bin"
            dt = np.uint16 if k == "a" else np.float32
            got = np.fromfile(path, dtype=dt)
            w = want[rk][k]
            if w is None:  # f32 sums of more than two ranks depend on NCCL's order
                ref = np.sum(np.stack(xs), axis=0, dtype=np.float64)
                np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
                continue
            assert np.array_equal(got, np.asarray(w).reshape(-1)), (rk, k)


@pytest.mark.gpu
def test_expert_parallel_graph_ops_fail_loudly(cuda, tmp_path):
    """moe_dispatch over more than one rank is expert parallelism: run as a
    single process (no communicator), the graph executor refuses it instead
    of computing one rank's share (tests/test_ep_graph_gpu.py runs it over
    several processes)."""
    if not KVM_RUN.exists():
        pytest.fail("kvm_run is not built")
    T, H, E = 64, 128, 8
    g = tmp_path / "ep.kvm"
    g.write_text(f"""graph {{
  config {{ ranks = [0, 1] }}
  ^ep(%x: {_t('bf16', [T, H])}, %g: {_t('f32', [T, E])}) {{
    %d: {_t('bf16', [2 * T, H])} = kernel.comm.moe_dispatch<ranks=[0,1]> {{top_k = 2}} (%x, %g)
    return %d
  }}
}}""")
    r = subprocess.run([str(KVM_RUN), str(g)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 1 and "needs a communicator" in r.stderr, r.stderr
