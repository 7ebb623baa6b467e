"""Causal grouped-query attention and rotary embedding against the oracle
(bf16 tolerance: relative L2 <= 1e-2)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import from_bits, rel_err, to_bits
from kvm_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,L,HQ,HKV", [(2, 256, 4, 2), (1, 384, 8, 1), (2, 200, 2, 2),
                                        (1, 1024, 16, 2), (3, 128, 3, 1)])
def test_attention_prefill(cuda, B, L, HQ, HKV):
    rng = np.random.default_rng(B * 1000 + L + HQ)
    hd = 128
    q = oracle.normal_bf16(rng, (B * L, HQ * hd))
    k = oracle.normal_bf16(rng, (B * L, HKV * hd))
    v = oracle.normal_bf16(rng, (B * L, HKV * hd))
    ref = oracle.attention(q, k, v, B, HQ, HKV)
    out = ops.attention_prefill(from_bits(q, cuda), from_bits(k, cuda), from_bits(v, cuda),
                                batch=B, heads_q=HQ, heads_kv=HKV)
    ops.device_status()
    got = oracle.bf16_to_f32(to_bits(out))
    assert np.isfinite(got).all()
    assert rel_err(got, oracle.bf16_to_f32(ref)) < 1e-2


def test_attention_on_strided_views(cuda):
    """q, k, v as column slices of one fused QKV matrix (the decoder layer's
    layout), output into a wider buffer."""
    rng = np.random.default_rng(7)
    B, L, HQ, HKV, hd = 2, 256, 4, 1, 128
    qkv = oracle.normal_bf16(rng, (B * L, (HQ + 2 * HKV) * hd))
    q = np.ascontiguousarray(qkv[:, :HQ * hd])
    k = np.ascontiguousarray(qkv[:, HQ * hd:(HQ + HKV) * hd])
    v = np.ascontiguousarray(qkv[:, (HQ + HKV) * hd:])
    ref = oracle.attention(q, k, v, B, HQ, HKV)
    t = from_bits(qkv, cuda)
    big = torch.zeros((B * L, HQ * hd + 256), dtype=torch.bfloat16, device=cuda)
    out = big[:, :HQ * hd]
    ops.attention_prefill(t[:, :HQ * hd], t[:, HQ * hd:(HQ + HKV) * hd],
                          t[:, (HQ + HKV) * hd:], batch=B, heads_q=HQ, heads_kv=HKV, out=out)
    ops.device_status()
    assert rel_err(oracle.bf16_to_f32(to_bits(out)), oracle.bf16_to_f32(ref)) < 1e-2
    assert torch.all(big[:, HQ * hd:] == 0)


@pytest.mark.parametrize("rows,L,heads", [(512, 256, 4), (2048, 2048, 2)])
def test_rope(cuda, rows, L, heads):
    rng = np.random.default_rng(rows + heads)
    x = oracle.normal_bf16(rng, (rows, heads * 128 + 64))   # wider rows: a view
    ref = oracle.rope(np.ascontiguousarray(x[:, :heads * 128]), L, heads)
    t = from_bits(x, cuda)
    ops.rope_(t[:, :heads * 128], seq_len=L, heads=heads)
    ops.device_status()
    got = to_bits(t)
    assert np.array_equal(got[:, heads * 128:], x[:, heads * 128:])   # untouched
    g, r = oracle.bf16_to_f32(got[:, :heads * 128]), oracle.bf16_to_f32(ref)
    assert rel_err(g, r) < 1e-2
    assert np.mean(got[:, :heads * 128] != ref) < 0.01   # at most rare 1-ulp flips


def test_attention_rescales_when_later_keys_dominate(cuda):
    """Keys of a later tile with 8x the scale raise each row's running max by
    far more than 2^8, so the fused kernel rescales its TMEM accumulator."""
    rng = np.random.default_rng(11)
    B, L, HQ, HKV, hd = 1, 512, 2, 1, 128
    q = oracle.normal_bf16(rng, (B * L, HQ * hd))
    kf = oracle.bf16_to_f32(oracle.normal_bf16(rng, (B * L, HKV * hd)))
    kf[384:512] *= 8.0
    kf[200:210] *= 4.0
    k = oracle.f32_to_bf16(kf)
    v = oracle.normal_bf16(rng, (B * L, HKV * hd))
    ref = oracle.attention(q, k, v, B, HQ, HKV)
    out = ops.attention_prefill(from_bits(q, cuda), from_bits(k, cuda), from_bits(v, cuda),
                                batch=B, heads_q=HQ, heads_kv=HKV)
    ops.device_status()
    got = oracle.bf16_to_f32(to_bits(out))
    assert np.isfinite(got).all()
    assert rel_err(got, oracle.bf16_to_f32(ref)) < 1e-2

