"""Fused elementwise programs (kvm_sm100_elementwise): kernels generated per
program and compiled by NVRTC for sm_100a, against the oracle's fp32
restatement (oracle.elementwise) and against the interpreter kernel
(KVM_SM100_EW_JIT=0).

Bit-exact for programs of correctly rounded ops (add sub mul div max min neg
abs rcp sqrt, compares, casts), except that NaN payloads and the sign of a
zero are not compared (x86 and the GPU make different default NaNs, and
max/min of +0 and -0 may return either); exp / log / rsqrt are CUDA's fp32
math functions, checked against the exact value within CUDA's documented
bounds (2 ulp for expf and rsqrtf, 1 ulp for logf)."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle
from kvm_b200 import _lib

EXACT = ["add", "sub", "mul", "div", "max", "min", "neg", "abs", "rcp", "sqrt", "cmp.eq",
         "cmp.ne", "cmp.lt", "cmp.le", "cmp.gt", "cmp.ge", "round.bf16", "round.f16",
         "trunc.i32"]
UNARY = {"neg", "abs", "rcp", "sqrt", "exp", "log", "rsqrt", "round.bf16", "round.f16",
         "trunc.i32"}
SILU = [("load", 0, 0, 0), ("load", 1, 0, 1), ("neg", 0, 0, 2), ("exp", 2, 0, 3),
        ("load", 2, 0, 4), ("add", 3, 4, 5), ("div", 0, 5, 6), ("mul", 6, 1, 7)]


def _prepare(instrs, dtypes, bcast, out_dtype, n, out_addr=1 << 20, align=16):
    p = _lib.ew_program(instrs, dtypes, bcast, out_dtype, instrs[-1][3])
    ins = _lib.EwInputs()
    for i in range(len(dtypes)):
        ins.ptr[i] = (1 << 24) * (i + 1) + (0 if align == 16 else 2)
    rc = _lib.lib().kvm_sm100_elementwise_prepare(C.byref(p), C.byref(ins),
                                                   C.c_void_p(out_addr), C.c_int64(n))
    return rc, _lib.lib().kvm_sm100_last_error().decode()


@pytest.mark.parametrize("out_dtype", ["bf16", "f32", "f16", "i32"])
@pytest.mark.parametrize("in_dtype", ["bf16", "f32", "f16", "i32"])
def test_codegen_compiles_every_dtype(in_dtype, out_dtype):
    """The generated source compiles for sm_100a (NVRTC runs without a GPU):
    8-wide form with contiguous, row-broadcast, column-broadcast and scalar
    inputs of each dtype into each output dtype."""
    n = 64 * 1024
    bc = [(n, 1), (1024, 1), (64, 1024), (1, 1)]
    instrs = [("load", 0, 0, 0), ("load", 1, 0, 1), ("load", 2, 0, 2), ("load", 3, 0, 3),
              ("mul", 0, 1, 4), ("add", 4, 2, 5), ("max", 5, 3, 6)]
    rc, err = _prepare(instrs, [in_dtype] * 4, bc, out_dtype, n)
    assert rc == 0, err


@pytest.mark.parametrize("op", sorted(set(EXACT) | {"exp", "log", "rsqrt"}))
def test_codegen_compiles_every_op(op):
    instrs = [("load", 0, 0, 0), ("load", 1, 0, 1), (op, 0, 1, 2)]
    rc, err = _prepare(instrs, ["bf16", "f32"], [(4096, 1), (4096, 1)], "bf16", 4096)
    assert rc == 0, err


def test_codegen_compiles_narrow_and_wide_forms():
    # odd sizes and a misaligned pointer take the 1-per-thread form
    rc, err = _prepare(SILU, ["bf16", "bf16", "f32"], [(1001, 1), (1001, 1), (1, 1)],
                       "bf16", 1001)
    assert rc == 0, err
    rc, err = _prepare(SILU, ["bf16", "bf16", "f32"], [(4096, 1), (4096, 1), (1, 1)],
                       "bf16", 4096, align=2)
    assert rc == 0, err
    rc, err = _prepare(SILU, ["bf16", "bf16", "f32"], [(12, 3), (36, 1), (1, 1)], "f32", 72)
    assert rc == 0, err
    # 64-bit indices past 2^31 elements
    n = (1 << 31) + 1024
    rc, err = _prepare([("load", 0, 0, 0), ("neg", 0, 0, 1)], ["f32"], [(1024, 1)], "bf16", n)
    assert rc == 0, err


def test_prepare_rejects_bad_programs():
    rc, err = _prepare([("load", 3, 0, 0)], ["bf16"], [(64, 1)], "bf16", 64)
    assert rc != 0 and "missing input" in err
    rc, err = _prepare([("load", 0, 0, 0)], ["bf16"], [(48, 1)], "bf16", 64)
    assert rc != 0 and "divide" in err


def test_oracle_silu_program():
    rng = np.random.default_rng(0)
    g = oracle.normal_bf16(rng, (512,), 3.0)
    u = oracle.normal_bf16(rng, (512,))
    one = np.ones(1, np.float32)
    got = oracle.elementwise(SILU, [(g, "bf16"), (u, "bf16"), (one, "f32")],
                             [(512, 1), (512, 1), (1, 1)], "bf16", 7, 512)
    assert np.array_equal(got, oracle.silu_mul(g, u)) or \
        np.abs(oracle.bf16_to_f32(got) - oracle.bf16_to_f32(oracle.silu_mul(g, u))).max() < 0.05


# ------------------------------------------------------------------ GPU ---

def _torch_in(arr, dt, cuda):
    import torch
    arr = np.array(arr, copy=True)  # numpy scalars become 0-d arrays
    if dt in ("bf16", "f16"):
        t = torch.from_numpy(arr.view(np.int16)).to(cuda)
        return t.view(torch.bfloat16 if dt == "bf16" else torch.float16)
    return torch.from_numpy(arr).to(cuda)


def _rand_input(rng, dt, shape):
    x = (np.asarray(rng.standard_normal(shape), dtype=np.float32) * 2).reshape(shape)
    if dt == "bf16":
        return oracle.f32_to_bf16(x)
    if dt == "f16":
        return x.astype(np.float16).view(np.uint16)
    if dt == "i32":
        return np.round(x * 4).astype(np.int32)
    return x


def _run(instrs, arrays, dtypes, out_shape, out_dtype, cuda):
    import torch
    from kvm_b200 import ops
    tin = [_torch_in(a, d, cuda) for a, d in zip(arrays, dtypes)]
    tdt = {"bf16": torch.bfloat16, "f32": torch.float32, "f16": torch.float16,
           "i32": torch.int32}[out_dtype]
    out = ops.elementwise(instrs, tin, out_shape, tdt)
    ops.device_status()
    o = out.cpu()
    if out_dtype in ("bf16", "f16"):
        return o.view(torch.int16).numpy().view(np.uint16).reshape(-1)
    return o.numpy().reshape(-1)


def _same(got, want, dtype):
    """Equal bits, or both NaN, or both zero."""
    got, want = np.asarray(got).reshape(-1), np.asarray(want).reshape(-1)
    if dtype == "i32":
        return np.array_equal(got, want)
    if dtype == "bf16":
        g, w = oracle.bf16_to_f32(got), oracle.bf16_to_f32(want)
    elif dtype == "f16":
        g, w = got.view(np.float16).astype(np.float32), want.view(np.float16).astype(np.float32)
    else:
        g, w = got.astype(np.float32), want.astype(np.float32)
    same = (got.view(np.uint8).reshape(len(got), -1) ==
            want.view(np.uint8).reshape(len(want), -1)).all(axis=1)
    ok = same | (np.isnan(g) & np.isnan(w)) | ((g == 0) & (w == 0))
    return bool(ok.all())


def _random_program(rng, n_inputs, ops_pool, length):
    instrs = [("load", i, 0, i) for i in range(n_inputs)]
    live = list(range(n_inputs))
    reg = n_inputs
    for _ in range(length):
        op = ops_pool[rng.integers(len(ops_pool))]
        a = live[rng.integers(len(live))]
        b = live[rng.integers(len(live))]
        dst = reg % 16
        instrs.append((op, a, 0 if op in UNARY else b, dst))
        if dst not in live:
            live.append(dst)
        reg += 1
    return instrs


SHAPES = [  # output shape, input shapes (broadcast patterns)
    ((256, 1024), [(256, 1024), (1024,), (256, 1), ()]),
    ((8, 16, 64), [(8, 16, 64), (16, 64), (8, 16, 1), (64,)]),
    ((3, 7, 5), [(3, 7, 5), (7, 5), (3, 1, 1), (5,)]),       # 1-per-thread form
    ((1000,), [(1000,), (1000,), (), ()]),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(len(SHAPES)))
@pytest.mark.parametrize("out_dtype", ["bf16", "f32", "f16", "i32"])
def test_random_exact_programs(cuda, case, out_dtype):
    """Random chains of correctly rounded ops over every broadcast pattern:
    the generated kernel equals the oracle bit for bit, and the interpreter."""
    out_shape, in_shapes = SHAPES[case]
    n = int(np.prod(out_shape))
    rng = np.random.default_rng(100 * case + len(out_dtype))
    for trial in range(6):
        dtypes = [["bf16", "f32", "f16", "i32"][(trial + j) % 4] for j in range(4)]
        arrays = [_rand_input(rng, d, s) for d, s in zip(dtypes, in_shapes)]
        instrs = _random_program(rng, 4, EXACT, 10)
        bc = [_lib.broadcast_of(s, out_shape) for s in in_shapes]
        want = oracle.elementwise(instrs, list(zip(arrays, dtypes)), bc, out_dtype,
                                  instrs[-1][3], n)
        got = _run(instrs, arrays, dtypes, out_shape, out_dtype, cuda)
        assert _same(got, want, out_dtype), (trial, instrs)
        os.environ["KVM_SM100_EW_JIT"] = "0"
        try:
            interp = _run(instrs, arrays, dtypes, out_shape, out_dtype, cuda)
        finally:
            del os.environ["KVM_SM100_EW_JIT"]
        assert _same(interp, got, out_dtype), (trial, instrs)


@pytest.mark.gpu
def test_transcendental_programs(cuda):
    """exp / log / rsqrt: within CUDA's documented error bound of the exact
    value (float64), and bit equal to the interpreter (same CUDA math calls)."""
    rng = np.random.default_rng(7)
    n = 1 << 16
    x = np.abs(rng.standard_normal(n).astype(np.float32)) + 0.1
    x64 = x.astype(np.float64)
    truth = {"exp": np.exp(x64), "log": np.log(x64), "rsqrt": 1.0 / np.sqrt(x64)}
    bound = {"exp": 2, "log": 1, "rsqrt": 2}  # CUDA's documented maximum ulp errors
    for op in ("exp", "log", "rsqrt"):
        instrs = [("load", 0, 0, 0), (op, 0, 0, 1)]
        got = _run(instrs, [x], ["f32"], (n,), "f32", cuda)
        ulp = np.spacing(np.abs(truth[op]).astype(np.float32)).astype(np.float64)
        assert np.all(np.abs(got - truth[op]) <= bound[op] * ulp), op
        os.environ["KVM_SM100_EW_JIT"] = "0"
        try:
            interp = _run(instrs, [x], ["f32"], (n,), "f32", cuda)
        finally:
            del os.environ["KVM_SM100_EW_JIT"]
        assert np.array_equal(interp, got), op


@pytest.mark.gpu
@pytest.mark.parametrize("n", [8, 4096 * 14336 // 8, 1000])
def test_silu_program_matches_fused_kernel_semantics(cuda, n):
    """The SiLU-gate expression as a generic program, bf16 in and out, against
    the oracle (the per-op fp32 chain; bit-exact except exp's <= 2 ulp)."""
    rng = np.random.default_rng(n)
    g = oracle.normal_bf16(rng, (n,), 3.0)
    u = oracle.normal_bf16(rng, (n,))
    one = np.ones(1, np.float32)
    got = _run(SILU, [g, u, one], ["bf16", "bf16", "f32"], (n,), "bf16", cuda)
    want = oracle.elementwise(SILU, [(g, "bf16"), (u, "bf16"), (one, "f32")],
                              [(n, 1), (n, 1), (1, 1)], "bf16", 7, n)
    gf, wf = oracle.bf16_to_f32(got), oracle.bf16_to_f32(want)
    # a 2-ulp exp difference can flip a bf16 rounding: at most one bf16 ulp
    assert np.all(np.abs(gf - wf) <= np.abs(wf) * 2 ** -7 + 1e-30)
    assert np.mean(got != want) < 1e-3


@pytest.mark.gpu
def test_wide_index_past_2g_elements(cuda):
    """n >= 2^31 takes the 64-bit index form: a row-broadcast input of 1024
    f32 values negated into 2^31 + 1024 bf16 outputs (4 GiB), sampled."""
    import torch
    from kvm_b200 import ops
    n = (1 << 31) + 1024
    row = torch.arange(1024, dtype=torch.float32, device=cuda)
    out = ops.elementwise([("load", 0, 0, 0), ("neg", 0, 0, 1)], [row], (n // 1024, 1024),
                          torch.bfloat16)
    ops.device_status()
    idx = torch.tensor([0, 1, 1023, 1024, (1 << 31) - 1, 1 << 31, n - 1], device=cuda)
    got = out.view(-1)[idx].float().cpu().numpy()
    want = oracle.bf16_to_f32(oracle.f32_to_bf16(-(idx.cpu().numpy() % 1024).astype(np.float32)))
    assert np.array_equal(got, want)
    del out
    torch.cuda.empty_cache()
