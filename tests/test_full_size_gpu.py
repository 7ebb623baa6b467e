"""Parity at the full sizes of the benchmark configurations, against the
oracle. Where rows (MLP, FP8 GEMM) or heads (attention) are independent, the
oracle computes a subset of them and only that subset is compared; the MoE
layer and the paged decode step are compared whole. Tolerances as elsewhere:
routing bit-exact given the GPU's logits (tokens whose top-k differs between
the GPU's and the oracle's own fp32 logits are counted and must be ties to
within 1e-4), bf16 relative L2 <= 1e-2, FP8 <= 3e-2."""
import numpy as np
import pytest
import torch

import oracle
from helpers import check_moe_routing_and_layer, rel_err, to_bits
from kvm_b200 import ops

pytestmark = pytest.mark.gpu


def _randn(g, shape, std, dev):
    """bf16 N(0, std^2) on the GPU, generated in slabs of at most 2^28 values."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    flat = out.view(-1)
    step = 1 << 28
    for i in range(0, flat.numel(), step):
        n = min(step, flat.numel() - i)
        flat[i:i + n] = (torch.randn(n, generator=g, device=dev) * std).to(torch.bfloat16)
    return out


def test_moe_layer_full_size(cuda, record_property):
    """8192 tokens, hidden 4096, 64 experts of 4096 -> 1408 -> 4096, top-2."""
    from kvm_b200.moe import MoELayer
    T, H, E, F, k = 8192, 4096, 64, 1408, 2
    g = torch.Generator(device=cuda)
    g.manual_seed(0)
    x = _randn(g, (T, H), 1.0, cuda)
    wr = _randn(g, (E, H), 0.02, cuda)
    w13 = _randn(g, (E, 2 * F, H), 0.02, cuda)
    w2 = _randn(g, (E, H, F), 0.02, cuda)
    layer = MoELayer(wr, w13, w2, k, T)
    out = layer(x)
    ops.device_status()
    n = check_moe_routing_and_layer(layer, to_bits(x), to_bits(w13), to_bits(w2),
                                    to_bits(wr), out, k, record_property)
    assert n <= T // 100


def test_gated_mlp_full_size(cuda):
    """x [4096, 4096], gate/up [4096 -> 14336], down [14336 -> 4096]: the GPU
    runs all rows, the oracle the first and last 128."""
    T, H, F = 4096, 4096, 14336
    g = torch.Generator(device=cuda)
    g.manual_seed(1)
    x = _randn(g, (T, H), 1.0, cuda)
    wg = _randn(g, (F, H), 0.02, cuda)
    wu = _randn(g, (F, H), 0.02, cuda)
    wd = _randn(g, (H, F), 0.02, cuda)
    w13 = ops.pack_gate_up(wg, wu, layout="nk")
    xn = ops.rmsnorm(x, None, 1e-5)
    h = ops.silu_gate_matmul(xn, w13)
    y = ops.matmul(h, wd, b_layout="nk")
    ops.device_status()
    got = oracle.bf16_to_f32(to_bits(y))
    wgb, wub, wdb = to_bits(wg), to_bits(wu), to_bits(wd)
    xb = to_bits(x)
    for rows in (slice(0, 128), slice(T - 128, T)):
        xr = oracle.rmsnorm(xb[rows], None, 1e-5)
        hr = oracle.gemm_silu_gate(xr, wgb, wub)
        yr = oracle.gemm(hr, wdb, b_layout="nk")
        assert rel_err(got[rows], oracle.bf16_to_f32(yr)) < 1e-2


@pytest.mark.parametrize("M", [16, 128, 1024])
def test_fp8_gemm_full_size(cuda, M):
    """[M, 8192] x [8192, 28672] e4m3 with 128 x 128 fp32 block scales: the
    GPU computes every row, the oracle the first and the last 16."""
    K, N = 8192, 28672
    g = torch.Generator(device=cuda)
    g.manual_seed(2 + M)
    w = torch.randn((N, K), generator=g, device=cuda)
    wq, sw = ops.quantize_e4m3(w)
    del w
    a = torch.randn((M, K), generator=g, device=cuda)
    aq, sa = ops.quantize_e4m3(a)
    d = ops.matmul_fp8(aq, sa, wq, sw)
    ops.device_status()
    got = oracle.bf16_to_f32(to_bits(d))
    assert np.isfinite(got).all()
    aqh, sah = aq.cpu().numpy(), sa.cpu().numpy()
    wqh, swh = wq.cpu().numpy(), sw.cpu().numpy()
    for r0 in sorted({0, M - 16}):
        blk = r0 // 128
        ref = oracle.gemm_fp8_blockscaled(aqh[r0:r0 + 16], sah[blk:blk + 1], wqh, swh)
        assert rel_err(got[r0:r0 + 16], oracle.bf16_to_f32(ref)) < 3e-2


def test_attention_full_size(cuda):
    """Causal GQA, batch 4 x 2048, 64 query / 8 kv heads of 128: the GPU
    computes all heads, the oracle the 8 query heads of kv head 0 and of kv
    head 7."""
    B, L, HQ, HKV, hd = 4, 2048, 64, 8, 128
    g = torch.Generator(device=cuda)
    g.manual_seed(3)
    q = _randn(g, (B * L, HQ * hd), 1.0, cuda)
    k = _randn(g, (B * L, HKV * hd), 1.0, cuda)
    v = _randn(g, (B * L, HKV * hd), 1.0, cuda)
    out = ops.attention_prefill(q, k, v, batch=B, heads_q=HQ, heads_kv=HKV)
    ops.device_status()
    got = oracle.bf16_to_f32(to_bits(out))
    qb, kb, vb = to_bits(q), to_bits(k), to_bits(v)
    grp = HQ // HKV
    for kh in (0, HKV - 1):
        qs = slice(kh * grp * hd, (kh + 1) * grp * hd)
        ks = slice(kh * hd, (kh + 1) * hd)
        ref = oracle.attention(qb[:, qs], kb[:, ks], vb[:, ks], B, grp, 1)
        assert rel_err(got[:, qs], oracle.bf16_to_f32(ref)) < 1e-2, kh


def test_paged_decode_full_size(cuda):
    """The decode step of the benchmark: 64 sequences x 4096 cached keys + one
    new token, 64 query / 8 kv heads, 16-token pages at random places; cache
    contents bit-exact, attention within 1e-2, every sequence checked."""
    from test_kvcache_gpu import _run
    _run(cuda, np.random.default_rng(11), layout="page_first", bs=16, HQ=64, HKV=8,
         ctx=[4096] * 64, nq=[1] * 64, layers=1, layer=0)


def test_tp_decoder_layer_full_size(cuda):
    """The tensor-parallel decoder layer's configuration on one GPU: hidden
    8192, 64 query / 8 kv heads of 128, FFN 28672 gated, batch 4 x 2048,
    RMSNorm gains 1. The GPU computes all 8192 tokens; the oracle computes the
    first and the last 16 tokens of sequence 3 (its keys and values for the
    whole sequence, queries only for those rows), composed op by op like the
    layer: RMSNorm, QKV, RoPE, causal attention, O + residual, RMSNorm,
    SiLU-gate FFN, down + residual."""
    from kvm_b200.tp import TPDecoderLayer
    B, L, H, HQ, HKV, F, hd = 4, 2048, 8192, 64, 8, 28672, 128
    g = torch.Generator(device=cuda)
    g.manual_seed(4)
    x = _randn(g, (B * L, H), 1.0, cuda)
    wq = _randn(g, (HQ * hd, H), 0.02, cuda)
    wk = _randn(g, (HKV * hd, H), 0.02, cuda)
    wv = _randn(g, (HKV * hd, H), 0.02, cuda)
    wo = _randn(g, (H, HQ * hd), 0.02, cuda)
    wg = _randn(g, (F, H), 0.02, cuda)
    wu = _randn(g, (F, H), 0.02, cuda)
    w2 = _randn(g, (H, F), 0.02, cuda)
    ones = torch.ones(H, dtype=torch.bfloat16, device=cuda)
    layer = TPDecoderLayer.from_full(wq, wk, wv, wo, wg, wu, w2, ones, ones, batch=B,
                                     seq_len=L, heads_q=HQ, heads_kv=HKV)
    out = layer(x)
    ops.device_status()
    s0 = 3 * L
    rows = np.r_[0:16, L - 16:L]
    got = oracle.bf16_to_f32(to_bits(out[s0:s0 + L]))[rows]
    del layer, out

    xs = to_bits(x[s0:s0 + L])
    gam = to_bits(ones)
    xn = oracle.rmsnorm(xs, gam, 1e-5)
    kv = oracle.gemm(xn, np.concatenate([to_bits(wk), to_bits(wv)]), b_layout="nk")
    k = oracle.rope(np.ascontiguousarray(kv[:, :HKV * hd]), L, HKV)
    v = np.ascontiguousarray(kv[:, HKV * hd:])
    q = np.zeros((L, HQ * hd), dtype=np.uint16)      # only the checked rows matter
    q[rows] = oracle.gemm(xn[rows], to_bits(wq), b_layout="nk")
    q = oracle.rope(q, L, HQ)
    a = oracle.attention(q, k, v, 1, HQ, HKV)[rows]
    h1 = oracle.gemm(a, to_bits(wo), b_layout="nk", c=xs[rows])
    h1n = oracle.rmsnorm(h1, gam, 1e-5)
    act = oracle.gemm_silu_gate(h1n, to_bits(wg), to_bits(wu))
    ref = oracle.gemm(act, to_bits(w2), b_layout="nk", c=h1)
    assert np.isfinite(got).all()
    assert rel_err(got, oracle.bf16_to_f32(ref)) < 1e-2
