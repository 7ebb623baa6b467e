"""Graphs through the whole drop-in path on a B200: .kvm text -> reference
parser -> reference transform with the sm_100a Device target -> executor ->
C ABI kernels (kvm_run), compared with the oracle composed op by op (each
kernel op's output rounded to its declared dtype). bf16 tolerance: relative
L2 error <= 1e-2."""
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from helpers import rel_err

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
KVM_RUN = ROOT / "kvm_b200" / "_build" / "host" / "kvm_run"


def _t(dtype, shape):
    return f"kernel.tensor<dtype={dtype}, shape=[{','.join(map(str, shape))}]>"


def _run(tmp_path, text, inputs, iters=2, fuse=True):
    if not KVM_RUN.exists():
        pytest.fail("kvm_run is not built (python -c 'import __graft_entry__ as g; g.build()')")
    g = tmp_path / "g.kvm"
    g.write_text(text)
    ind, outd = tmp_path / "in", tmp_path / "out"
    ind.mkdir()
    outd.mkdir()
    for name, arr in inputs.items():
        np.ascontiguousarray(arr).tofile(ind / f"{name}.bin")
    import os
    env = dict(os.environ, KVM_EXEC_NO_FUSION="0" if fuse else "1")
    r = subprocess.run([str(KVM_RUN), str(g), "--inputs", str(ind), "--out", str(outd),
                        "--warmup", "1", "--iters", str(iters)],
                       capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr
    summary = json.loads(r.stdout.strip().splitlines()[-1])
    return summary, outd


def _bf(x):
    return oracle.f32_to_bf16(np.asarray(x, dtype=np.float32))


def _f(b):
    return oracle.bf16_to_f32(b).astype(np.float32)


def mlp_graph(T, H, F):
    """The gated-MLP block graph (RMSNorm and SiLU-gate as kernel-op
    composites) at the given sizes; kvm_b200/graphs/mlp_block.kvm is this
    graph at T = H = 4096, F = 14336."""
    bf, f32 = "bf16", "f32"
    return f"""graph {{
  config {{ ranks = [0] }}
  ^mlp(%x: {_t(bf, [T, H])}, %gamma: {_t(bf, [H])}, %invh: {_t(bf, [H, 1])} {{fill = {1.0 / H!r}}}, %eps: {_t(f32, [1])} {{fill = 1e-5}}, %one: {_t(bf, [1])} {{fill = 1.0}}, %wg: {_t(bf, [H, F])}, %wu: {_t(bf, [H, F])}, %wd: {_t(bf, [F, H])}) {{
    %sq: {_t(bf, [T, H])} = kernel.mul(%x, %x)
    %ms: {_t(f32, [T, 1])} = kernel.matmul(%sq, %invh)
    %ve: {_t(f32, [T, 1])} = kernel.add(%ms, %eps)
    %r: {_t(f32, [T, 1])} = kernel.rsqrt(%ve)
    %xn: {_t(bf, [T, H])} = kernel.mul(%x, %r)
    %xg: {_t(bf, [T, H])} = kernel.mul(%xn, %gamma)
    %g: {_t(bf, [T, F])} = kernel.matmul(%xg, %wg)
    %u: {_t(bf, [T, F])} = kernel.matmul(%xg, %wu)
    %n: {_t(bf, [T, F])} = kernel.neg(%g)
    %e: {_t(bf, [T, F])} = kernel.exp(%n)
    %p: {_t(bf, [T, F])} = kernel.add(%e, %one)
    %s: {_t(bf, [T, F])} = kernel.div(%g, %p)
    %h: {_t(bf, [T, F])} = kernel.mul(%s, %u)
    %o: {_t(bf, [T, H])} = kernel.matmul(%h, %wd)
    return %o
  }}
}}"""


def test_matmul_and_gemm_graph(cuda, tmp_path):
    rng = np.random.default_rng(0)
    M, K, N = 256, 512, 384
    a, b = oracle.normal_bf16(rng, (M, K)), oracle.normal_bf16(rng, (K, N))
    c = oracle.normal_bf16(rng, (M, N))
    text = f"""graph {{
  ^g(%a: {_t('bf16', [M, K])}, %b: {_t('bf16', [K, N])}, %c: {_t('bf16', [M, N])}) {{
    %d: {_t('bf16', [M, N])} = kernel.matmul(%a, %b)
    %e: {_t('bf16', [M, N])} = kernel.gemm(%a, %b, %c)
    return %d, %e
  }}
}}"""
    s, outd = _run(tmp_path, text, {"a": a, "b": b, "c": c})
    assert s["steps"] == ["gemm_bf16", "gemm_bf16"]
    d = np.fromfile(outd / "d.bin", dtype=np.uint16).reshape(M, N)
    e = np.fromfile(outd / "e.bin", dtype=np.uint16).reshape(M, N)
    assert rel_err(_f(d), _f(oracle.gemm(a, b))) < 1e-2
    assert rel_err(_f(e), _f(oracle.gemm(a, b, c=c))) < 1e-2


def test_elementwise_broadcast_graph(cuda, tmp_path):
    rng = np.random.default_rng(1)
    T, H = 64, 96
    x = oracle.normal_bf16(rng, (T, H))
    y = oracle.normal_bf16(rng, (T, H))
    col = (rng.random((T, 1)) + 0.5).astype(np.float32)
    row = oracle.normal_bf16(rng, (H,))
    text = f"""graph {{
  ^g(%x: {_t('bf16', [T, H])}, %y: {_t('bf16', [T, H])}, %col: {_t('f32', [T, 1])}, %row: {_t('bf16', [H])}) {{
    %s: {_t('bf16', [T, H])} = kernel.add(%x, %y)
    %m: {_t('f32', [T, H])} = kernel.mul(%s, %col)
    %q: {_t('bf16', [T, H])} = kernel.div(%m, %row)
    %r: {_t('f32', [T, 1])} = kernel.rsqrt(%col)
    %z: {_t('bf16', [T, H])} = kernel.max(%q, %x)
    %k: {_t('bf16', [T, H])} = kernel.cmp.gt(%x, %y)
    return %z, %r, %k
  }}
}}"""
    s, outd = _run(tmp_path, text, {"x": x, "y": y, "col": col, "row": row})
    sref = _f(_bf(_f(x) + _f(y)))
    mref = sref * col
    qref = _f(_bf(mref / _f(row)))
    zref = _f(_bf(np.maximum(qref, _f(x))))
    z = _f(np.fromfile(outd / "z.bin", dtype=np.uint16).reshape(T, H))
    assert np.array_equal(z, zref)
    r = np.fromfile(outd / "r.bin", dtype=np.float32).reshape(T, 1)
    np.testing.assert_allclose(r, 1 / np.sqrt(col), rtol=1e-6)
    k = _f(np.fromfile(outd / "k.bin", dtype=np.uint16).reshape(T, H))
    assert np.array_equal(k, (_f(x) > _f(y)).astype(np.float32))


@pytest.mark.parametrize("fuse", [True, False])
def test_moe_graph(cuda, tmp_path, fuse):
    rng = np.random.default_rng(2)
    T, H, E, F, k = 512, 256, 8, 128, 2
    x = oracle.normal_bf16(rng, (T, H))
    wr = oracle.normal_bf16(rng, (H, E), 0.05)
    w1 = oracle.normal_bf16(rng, (E, H, F), 0.05)
    w3 = oracle.normal_bf16(rng, (E, H, F), 0.05)
    w2 = oracle.normal_bf16(rng, (E, F, H), 0.05)
    one = _bf(np.ones(1))
    text = f"""graph {{
  config {{ ranks = [0] }}
  ^moe(%x: {_t('bf16', [T, H])}, %wr: {_t('bf16', [H, E])}, %w1: {_t('bf16', [E, H, F])}, %w3: {_t('bf16', [E, H, F])}, %w2: {_t('bf16', [E, F, H])}, %one: {_t('bf16', [1])} {{fill = 1.0}}) {{
    %g: {_t('f32', [T, E])} = kernel.matmul(%x, %wr)
    %d: {_t('bf16', [T * k, H])} = kernel.comm.moe_dispatch<ranks=[0]> {{top_k = {k}}} (%x, %g)
    %a: {_t('bf16', [T * k, F])} = kernel.matmul(%d, %w1)
    %b: {_t('bf16', [T * k, F])} = kernel.matmul(%d, %w3)
    %n: {_t('bf16', [T * k, F])} = kernel.neg(%a)
    %e: {_t('bf16', [T * k, F])} = kernel.exp(%n)
    %p: {_t('bf16', [T * k, F])} = kernel.add(%e, %one)
    %s: {_t('bf16', [T * k, F])} = kernel.div(%a, %p)
    %h: {_t('bf16', [T * k, F])} = kernel.mul(%s, %b)
    %y: {_t('bf16', [T * k, H])} = kernel.matmul(%h, %w2)
    %out: {_t('bf16', [T, H])} = kernel.comm.moe_combine<ranks=[0]> (%y, %g)
    return %out, %g
  }}
}}"""
    s, outd = _run(tmp_path, text, {"x": x, "wr": wr, "w1": w1, "w3": w3, "w2": w2,
                                    "one": one}, fuse=fuse)
    # g is also a graph output, so the router GEMM is not fused into top-k
    assert s["steps"][:4] == ["gemm_bf16", "moe_topk", "moe_permute", "moe_scatter_rows"]
    assert ("grouped_gemm_silu_gate" in s["steps"]) == fuse
    g = np.fromfile(outd / "g.bin", dtype=np.float32).reshape(T, E)
    assert rel_err(g, oracle.gemm(x, wr, out_f32=True)) < 1e-5
    # oracle composed op by op, routed on the GPU's own logits
    idx, tw = oracle.moe_topk(g, k)
    off, pos, _ = oracle.moe_permute(idx, E)
    d = oracle.moe_scatter_rows(x, pos, k)
    tr = lambda w: np.ascontiguousarray(w.transpose(0, 2, 1))
    a = oracle.grouped_gemm(d, tr(w1), off)
    b = oracle.grouped_gemm(d, tr(w3), off)
    n = _bf(-_f(a))
    e = _bf(np.exp(_f(n)))
    p = _bf(_f(e) + 1.0)
    sv = _bf(_f(a) / _f(p))
    h = _bf(_f(sv) * _f(b))
    y = oracle.grouped_gemm(h, tr(w2), off)
    ref = oracle.moe_combine(y, pos, tw)
    out = np.fromfile(outd / "out.bin", dtype=np.uint16).reshape(T, H)
    assert rel_err(_f(out), _f(ref)) < 1e-2


@pytest.mark.parametrize("fuse", [True, False])
def test_rmsnorm_mlp_graph(cuda, tmp_path, fuse):
    rng = np.random.default_rng(3)
    T, H, F = 256, 512, 1024
    x = oracle.normal_bf16(rng, (T, H))
    gamma = oracle.normal_bf16(rng, (H,))
    invh = _bf(np.full((H, 1), 1.0 / H))
    eps = np.array([1e-5], dtype=np.float32)
    one = _bf(np.ones(1))
    wg = oracle.normal_bf16(rng, (H, F), 0.05)
    wu = oracle.normal_bf16(rng, (H, F), 0.05)
    wd = oracle.normal_bf16(rng, (F, H), 0.05)
    text = mlp_graph(T, H, F)
    s, outd = _run(tmp_path, text, {"x": x, "gamma": gamma, "invh": invh, "eps": eps,
                                    "one": one, "wg": wg, "wu": wu, "wd": wd}, fuse=fuse)
    if fuse:
        assert s["steps"] == ["rmsnorm", "gemm_silu_gate", "gemm_bf16"]
    else:
        assert "gemv_bf16" in s["steps"] and len(s["steps"]) == 14
    sq = _bf(_f(x) * _f(x))
    ms = oracle.gemm(sq, invh, out_f32=True)          # [T, 1]
    r = 1.0 / np.sqrt(ms + eps[0])
    xn = _bf(_f(x) * r)
    xg = _bf(_f(xn) * _f(gamma))
    g = oracle.gemm(xg, wg)
    u = oracle.gemm(xg, wu)
    n = _bf(-_f(g))
    e = _bf(np.exp(_f(n)))
    p = _bf(_f(e) + 1.0)
    sv = _bf(_f(g) / _f(p))
    h = _bf(_f(sv) * _f(u))
    ref = oracle.gemm(h, wd)
    o = np.fromfile(outd / "o.bin", dtype=np.uint16).reshape(T, H)
    assert rel_err(_f(o), _f(ref)) < 1e-2


def test_moe_graph_router_fused(cuda, tmp_path):
    """With the logits only feeding dispatch/combine, the router GEMM, softmax
    and top-k run as one kernel; results match the unfused run."""
    rng = np.random.default_rng(4)
    T, H, E, F, k = 256, 256, 16, 128, 2
    ins = {"x": oracle.normal_bf16(rng, (T, H)), "wr": oracle.normal_bf16(rng, (H, E), 0.05),
           "w1": oracle.normal_bf16(rng, (E, H, F), 0.05),
           "w3": oracle.normal_bf16(rng, (E, H, F), 0.05),
           "w2": oracle.normal_bf16(rng, (E, F, H), 0.05), "one": _bf(np.ones(1))}
    text = (ROOT / "kvm_b200" / "graphs" / "moe_layer.kvm").read_text()
    for a, b in [("[8192,4096]", f"[{T},{H}]"), ("[4096,64]", f"[{H},{E}]"),
                 ("[64,4096,1408]", f"[{E},{H},{F}]"), ("[64,1408,4096]", f"[{E},{F},{H}]"),
                 ("[8192,64]", f"[{T},{E}]"), ("[16384,4096]", f"[{T * k},{H}]"),
                 ("[16384,1408]", f"[{T * k},{F}]")]:
        text = text.replace(a, b)
    s1, o1 = _run(tmp_path / "a", text, ins) if (tmp_path / "a").mkdir() is None else None
    s2, o2 = _run(tmp_path / "b", text, ins, fuse=False) if (tmp_path / "b").mkdir() is None else None
    assert s1["steps"][0] == "moe_router_topk" and s2["steps"][0] == "gemm_bf16"
    a = _f(np.fromfile(o1 / "out.bin", dtype=np.uint16))
    b = _f(np.fromfile(o2 / "out.bin", dtype=np.uint16))
    assert rel_err(a, b) < 1e-2
