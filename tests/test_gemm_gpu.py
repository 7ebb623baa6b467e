"""tcgen05 GEMM parity against the oracle (kernel.matmul / kernel.gemm).

Tolerance (bf16 outputs): relative L2 error <= 1e-2 and max |err| <= 2% of the
output's max |ref| -- both sides accumulate in fp32; differences come from
summation order and bf16 output rounding.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import from_bits, rel_err, to_bits
from kvm_b200 import ops

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 256, 64),      # one tile
    (256, 512, 1024),
    (1000, 776, 520),    # ragged M, N, K (masking, partial TMA boxes)
    (1, 64, 8),          # tiny
    (1024, 1024, 1024),  # the single-matmul graph's shape
    (4736, 2048, 256),   # more tiles than SMs: persistent loop, 2 TMEM buffers
    # On 148 SMs the last wave of these runs as half-width items:
    (1280, 1920, 256),   # 150 tiles of 128 x 128: the last 2 as 4 halves of 64
    (4096, 2560, 128),   # 320 tiles of 128 x 256: the last 24 as 48 halves
    (4000, 2408, 200),   # ragged; the very last half lies wholly past N
]


def _check_bf16(got_bits, ref_bits, tol=1e-2):
    g = oracle.bf16_to_f32(got_bits)
    r = oracle.bf16_to_f32(ref_bits)
    assert np.isfinite(g).all()
    assert rel_err(g, r) <= tol
    assert np.abs(g - r).max() <= 0.02 * max(np.abs(r).max(), 1e-3)


@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_matmul_bf16(cuda, M, N, K, layout):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = oracle.normal_bf16(rng, (M, K))
    b = oracle.normal_bf16(rng, (K, N) if layout == "kn" else (N, K))
    ref = oracle.gemm(a, b, b_layout=layout)
    d = ops.matmul(from_bits(a, cuda), from_bits(b, cuda), b_layout=layout)
    ops.device_status()
    _check_bf16(to_bits(d), ref)


@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("M,N,K", [(384, 640, 512), (1280, 1920, 256)])
def test_gemm_f32_with_addend(cuda, layout, M, N, K):
    rng = np.random.default_rng(11)
    a = oracle.normal_bf16(rng, (M, K))
    b = oracle.normal_bf16(rng, (K, N) if layout == "kn" else (N, K))
    c = rng.standard_normal((M, N), dtype=np.float32)
    ref = oracle.gemm(a, b, b_layout=layout, c=c, out_f32=True)
    d = ops.gemm(from_bits(a, cuda), from_bits(b, cuda), torch.from_numpy(c).to(cuda),
                 b_layout=layout)
    ops.device_status()
    assert rel_err(d.cpu().numpy(), ref) < 1e-5


def test_gemm_bf16_addend_and_strided_rows(cuda):
    rng = np.random.default_rng(12)
    M, N, K = 300, 512, 256
    a_full = oracle.normal_bf16(rng, (M, K + 64))
    b = oracle.normal_bf16(rng, (N, K))
    c = oracle.normal_bf16(rng, (M, N))
    ref = oracle.gemm(np.ascontiguousarray(a_full[:, :K]), b, b_layout="nk", c=c)
    a_dev = from_bits(a_full, cuda)[:, :K]          # row stride K + 64
    d = ops.gemm(a_dev, from_bits(b, cuda), from_bits(c, cuda), b_layout="nk")
    ops.device_status()
    _check_bf16(to_bits(d), ref)


def test_output_canaries_untouched(cuda):
    """Rows/cols outside the output view must not be written."""
    rng = np.random.default_rng(13)
    M, N, K = 200, 136, 128
    a = oracle.normal_bf16(rng, (M, K))
    b = oracle.normal_bf16(rng, (N, K))
    big = torch.full((M + 8, N + 24), 7.0, dtype=torch.bfloat16, device=cuda)
    out = big[:M, :N]
    ops.matmul(from_bits(a, cuda), from_bits(b, cuda), b_layout="nk", out=out)
    ops.device_status()
    _check_bf16(to_bits(out), oracle.gemm(a, b, b_layout="nk"))
    assert torch.all(big[M:, :] == 7.0) and torch.all(big[:, N:] == 7.0)


def test_silu_gate_gemm(cuda):
    rng = np.random.default_rng(14)
    M, F, K = 300, 384, 512
    a = oracle.normal_bf16(rng, (M, K))
    wg = oracle.normal_bf16(rng, (F, K), 0.05)
    wu = oracle.normal_bf16(rng, (F, K), 0.05)
    ref = oracle.gemm_silu_gate(a, wg, wu)
    w13 = ops.pack_gate_up(from_bits(wg, cuda), from_bits(wu, cuda), layout="nk")
    assert np.array_equal(to_bits(w13), oracle.pack_gate_up(wg[None], wu[None])[0])
    h = ops.silu_gate_matmul(from_bits(a, cuda), w13)
    ops.device_status()
    _check_bf16(to_bits(h), ref)


def test_pack_gate_up_from_kn_layout(cuda):
    rng = np.random.default_rng(15)
    G, K, F = 3, 96, 256
    wg = oracle.normal_bf16(rng, (G, K, F))
    wu = oracle.normal_bf16(rng, (G, K, F))
    got = ops.pack_gate_up(from_bits(wg, cuda), from_bits(wu, cuda), layout="kn")
    ref = oracle.pack_gate_up(np.ascontiguousarray(wg.transpose(0, 2, 1)),
                              np.ascontiguousarray(wu.transpose(0, 2, 1)))
    assert np.array_equal(to_bits(got), ref)
    t = ops.transpose(from_bits(wg, cuda))
    assert np.array_equal(to_bits(t), wg.transpose(0, 2, 1))
