"""FP8 e4m3 block quantiser (bit-exact) and W8A8 block-scaled GEMM (relative
L2 error <= 3e-2, the FP8 tolerance) against the oracle."""
import numpy as np
import pytest
import torch

import oracle
from helpers import rel_err, to_bits
from kvm_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("R,C", [(256, 384), (200, 300), (16, 8192), (1, 128)])
def test_quantiser_bit_exact(cuda, R, C):
    rng = np.random.default_rng(R * C)
    x = (rng.standard_normal((R, C)) * 3).astype(np.float32)
    q, s = ops.quantize_e4m3(torch.from_numpy(x).to(cuda))
    ops.device_status()
    rq, rs = oracle.quantize_e4m3_block128(x)
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(q.cpu().numpy(), rq)


def test_quantiser_from_bf16(cuda):
    rng = np.random.default_rng(3)
    xb = oracle.normal_bf16(rng, (128, 256))
    xt = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    q, s = ops.quantize_e4m3(xt)
    rq, rs = oracle.quantize_e4m3_block128(oracle.bf16_to_f32(xb))
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


@pytest.mark.parametrize("M,N,K", [(16, 1024, 2048), (128, 512, 1024), (300, 256, 640),
                                   (1024, 1280, 1024), (1, 256, 512), (33, 384, 1024),
                                   (64, 128 * 150, 256), (16, 28672, 1024),
                                   (200, 128 * 37, 384), (300, 128 * 100, 256)])
def test_fp8_gemm(cuda, M, N, K):
    """Every launch form: the swapped form for M <= 64 (16/32/64-token tiles)
    and the 128-row form, each with stream-K tiles cut between CTAs (partials
    + reduction) or held whole, and round-robin waves before a stream-K tail
    (300 tiles on 148 SMs)."""
    rng = np.random.default_rng(M + N + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((N, K)).astype(np.float32)
    aq, sa = oracle.quantize_e4m3_block128(a)
    wq, sw = oracle.quantize_e4m3_block128(w)
    ref = oracle.bf16_to_f32(oracle.gemm_fp8_blockscaled(aq, sa, wq, sw))
    d = ops.matmul_fp8(torch.from_numpy(aq).to(cuda), torch.from_numpy(sa).to(cuda),
                       torch.from_numpy(wq).to(cuda), torch.from_numpy(sw).to(cuda))
    ops.device_status()
    got = oracle.bf16_to_f32(to_bits(d))
    assert np.isfinite(got).all()
    assert rel_err(got, ref) < 3e-2
    assert rel_err(got, ref) < 2e-3     # in practice: bf16 rounding flips only


def test_fp8_weights_from_kn_layout(cuda):
    """Weights given [K, N] with [K/128, N/128] scales are re-laid out once."""
    rng = np.random.default_rng(9)
    M, N, K = 64, 256, 512
    a = rng.standard_normal((M, K)).astype(np.float32)
    w_kn = rng.standard_normal((K, N)).astype(np.float32)
    wq_kn, sw_kn = oracle.quantize_e4m3_block128(w_kn)
    aq, sa = oracle.quantize_e4m3_block128(a)
    wq = ops.transpose_u8(torch.from_numpy(wq_kn).to(cuda))
    sw = ops.transpose_f32(torch.from_numpy(sw_kn).to(cuda))
    assert np.array_equal(wq.cpu().numpy(), wq_kn.T)
    d = ops.matmul_fp8(torch.from_numpy(aq).to(cuda), torch.from_numpy(sa).to(cuda), wq, sw)
    ref = oracle.bf16_to_f32(oracle.gemm_fp8_blockscaled(
        aq, sa, np.ascontiguousarray(wq_kn.T), np.ascontiguousarray(sw_kn.T)))
    assert rel_err(oracle.bf16_to_f32(to_bits(d)), ref) < 3e-2
