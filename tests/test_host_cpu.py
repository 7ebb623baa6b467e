"""C++ host side on CPU: the reference's own test binaries (graph, parser,
dialects, decomp) linked against the sm_100a Device target instead of the
reference's src/device/device.cpp, and lowering of the configuration graphs
through the reference parser and transform (kvm_run --lower-only)."""
import json
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HOST = ROOT / "kvm_b200" / "_build" / "host"
GRAPHS = ROOT / "kvm_b200" / "graphs"
REF_TESTS = ["value", "graph", "attr", "serialize", "parse", "kernel_dialect",
             "task_dialect", "tile_dialect", "decomp"]


@pytest.fixture(scope="module")
def host_bin():
    if not (HOST / "kvm_run").exists():
        from kvm_b200.host import build_host
        if not build_host.build():
            pytest.skip("host binaries not built and the reference sources are absent")
    return HOST


@pytest.mark.parametrize("name", REF_TESTS)
def test_reference_tests_pass_on_sm100_device(host_bin, name):
    r = subprocess.run([str(host_bin / f"test_{name}")], capture_output=True, text=True,
                       timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all tests passed" in r.stdout


@pytest.mark.parametrize("graph,ops,fusions", [
    ("matmul_1024", 4, []),
    ("moe_layer", 37, ["silu_gate", "router"]),
    ("moe_layer_ep8", 37, ["silu_gate", "router"]),
    ("mlp_block", 54, ["rmsnorm", "silu_gate"])])
def test_config_graphs_lower(host_bin, graph, ops, fusions):
    r = subprocess.run([str(host_bin / "kvm_run"), str(GRAPHS / f"{graph}.kvm"),
                        "--lower-only", "--dump-task"], capture_output=True, text=True,
                       timeout=60)
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    assert out["task_ops"] == ops
    assert [f.split(":")[0] for f in out["fusions"]] == fusions
    # the dump is itself a parseable task graph with the expected units
    assert "task.tc.mma" in r.stderr and "loc=shared" in r.stderr


def test_unlowerable_op_fails_loudly(host_bin, tmp_path):
    g = tmp_path / "attn.kvm"
    g.write_text("""graph {
  ^a(%q: kernel.tensor<dtype=bf16, shape=[8,64]>, %m: kernel.attn_meta<q={off=[0,8],pos=[0]}, kv={off=[0,8],pos=[0],blocks=[[0]]}, mask=causal>) {
    %r: kernel.tensor<dtype=bf16, shape=[8,64]> = kernel.attn.rope(%q, %m)
    return %r
  }
}
""")
    r = subprocess.run([str(host_bin / "kvm_run"), str(g), "--lower-only"],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode != 0


def test_fusion_can_be_disabled(host_bin):
    import os
    env = dict(os.environ, KVM_EXEC_NO_FUSION="1")
    r = subprocess.run([str(host_bin / "kvm_run"), str(GRAPHS / "moe_layer.kvm"),
                        "--lower-only"], capture_output=True, text=True, timeout=60, env=env)
    assert r.returncode == 0 and json.loads(r.stdout)["fusions"] == []


# ------------------------------------------------------- task -> tile pass ---

def _tile_run(host_bin, *args, timeout=120):
    r = subprocess.run([str(host_bin / "kvm_run"), *map(str, args)], capture_output=True,
                       text=True, timeout=timeout)
    return r


def test_tile_lowering_matmul_matches_gemm_tiles(host_bin):
    """kernel.matmul 1024^3 -> one tile.tc.mma(_acc) per tcgen05 instruction of
    the one-SM GEMM's 128x128 tiles (64 tiles x 64 K-steps of 16), all legal."""
    r = _tile_run(host_bin, GRAPHS / "matmul_1024.kvm", "--tile")
    assert r.returncode == 0, r.stderr
    s = json.loads(r.stdout)
    assert s["mma"] == 8 * 8 * 64 and s["loads"] == 2 * s["mma"] and s["stores"] == 64
    assert s["illegal"] == 0 and s["copied"] == 0
    assert "64 tiles of 128x128" in s["tiled"][0]


def test_tile_lowering_moe_layer(host_bin):
    """The router product tiles as 128x64 (the router kernel's tile); the
    routed expert products keep their task shape (tiles chosen on the GPU)."""
    r = _tile_run(host_bin, GRAPHS / "moe_layer.kvm", "--tile")
    assert r.returncode == 0, r.stderr
    s = json.loads(r.stdout)
    assert s["illegal"] == 0 and s["dynamic_mma"] == 3
    assert any("tiles of 128x64" in t for t in s["tiled"])


def test_tile_graph_text_round_trip(host_bin, tmp_path):
    out = tmp_path / "tile.kvm"
    r = subprocess.run([str(host_bin / "kvm_run"), str(GRAPHS / "matmul_1024.kvm"), "--tile",
                        "--dump-tile"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0
    out.write_text(r.stderr)
    s = json.loads(r.stdout)
    v = _tile_run(host_bin, "--verify-tile", out)
    assert v.returncode == 0, v.stdout + v.stderr
    assert json.loads(v.stdout) == {"tile_ops": s["tile_ops"], "illegal": 0, "first_error": ""}


def _mma_graph(m, n, k, a_dt="bf16", b_dt="bf16", b_loc="shared", d_dt="f32"):
    return f"""graph {{
  config {{ ranks = [0] }}
  ^t(%a: tile.tensor<dtype={a_dt}, loc=shared, shape=[{m},{k}]>, %b: tile.tensor<dtype={b_dt}, loc={b_loc}, shape=[{k},{n}]>) {{
    %d: tile.tensor<dtype={d_dt}, loc=register, shape=[{m},{n}]> = tile.tc.mma<m={m}, n={n}, k={k}>(%a, %b)
    return %d
  }}
}}
"""


@pytest.mark.parametrize("m,n,k,kw,ok", [
    (128, 256, 16, {}, True),                  # the one-SM GEMM tile
    (256, 144, 16, {}, True),                  # an SM-pair tile of 144 tokens
    (64, 8, 16, {}, True),
    (128, 64, 16, {"a_dt": "f16", "b_dt": "f16"}, True),
    (128, 200, 16, {}, False),                 # N not a multiple of 16
    (96, 128, 16, {}, False),                  # no M = 96 instruction
    (128, 128, 32, {}, False),                 # kind::f16 has K = 16
    (128, 128, 16, {"b_loc": "register"}, False),
    (128, 128, 16, {"a_dt": "f16"}, False),    # A and B of one type
    (128, 128, 16, {"a_dt": "f32", "b_dt": "f32"}, False),
])
def test_legal_tile_table(host_bin, tmp_path, m, n, k, kw, ok):
    g = tmp_path / "one.kvm"
    g.write_text(_mma_graph(m, n, k, **kw))
    r = _tile_run(host_bin, "--verify-tile", g)
    s = json.loads(r.stdout)
    assert (s["illegal"] == 0) == ok, s
    assert (r.returncode == 0) == ok
