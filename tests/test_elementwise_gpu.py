"""RMSNorm and SiLU-gate kernels against the oracle (bf16 tolerance 1e-2;
in practice differences are single bf16 rounding flips)."""
import numpy as np
import pytest

import oracle
from helpers import from_bits, rel_err, to_bits
from kvm_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,H", [(4096, 4096), (3, 8192), (17, 24), (5, 12288)])
@pytest.mark.parametrize("with_gamma", [False, True])
def test_rmsnorm(cuda, rows, H, with_gamma):
    rng = np.random.default_rng(rows + H)
    x = oracle.normal_bf16(rng, (rows, H))
    g = oracle.normal_bf16(rng, (H,)) if with_gamma else None
    ref = oracle.rmsnorm(x, g, 1e-5)
    y = ops.rmsnorm(from_bits(x, cuda), None if g is None else from_bits(g, cuda), 1e-5)
    ops.device_status()
    got = oracle.bf16_to_f32(to_bits(y))
    r = oracle.bf16_to_f32(ref)
    assert rel_err(got, r) < 1e-2
    # at most a one-ulp bf16 difference per element
    assert np.abs(got - r).max() <= np.abs(r).max() * 2 ** -7


@pytest.mark.parametrize("n", [8, 4096 * 14336 // 64, 1000])
def test_silu_mul(cuda, n):
    rng = np.random.default_rng(n)
    g = oracle.normal_bf16(rng, (n,), 3.0)
    u = oracle.normal_bf16(rng, (n,))
    ref = oracle.silu_mul(g, u)
    h = ops.silu_mul(from_bits(g, cuda), from_bits(u, cuda))
    ops.device_status()
    assert rel_err(oracle.bf16_to_f32(to_bits(h)), oracle.bf16_to_f32(ref)) < 1e-2
