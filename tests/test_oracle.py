"""CPU checks of the oracle itself (test infrastructure): bf16 rounding against
torch, GEMM/norm/SiLU against float64 numpy restatements, and the MoE routing,
permutation and combine definitions on hand-made cases."""
import numpy as np
import pytest
import torch

import oracle
from helpers import rel_err


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(100000).astype(np.float32) * 10,
        np.array([0.0, -0.0, 1.0, 65504.0, 3.3895314e38, 1e-40, np.inf, -np.inf],
                 dtype=np.float32),
        # exact ties: mantissa low half 0x8000 (even and odd upper halves)
        np.array([0x3F808000, 0x3F818000, 0xBF808000], dtype=np.uint32).view(np.float32),
    ])
    ours = oracle.f32_to_bf16(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)
    nan = oracle.f32_to_bf16(np.array([np.nan], dtype=np.float32))
    assert np.isnan(oracle.bf16_to_f32(nan))[0]


@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_gemm_matches_float64(layout):
    rng = np.random.default_rng(1)
    M, N, K = 37, 53, 70
    a = oracle.normal_bf16(rng, (M, K))
    b = oracle.normal_bf16(rng, (K, N) if layout == "kn" else (N, K))
    got = oracle.gemm(a, b, b_layout=layout, out_f32=True)
    bf = oracle.bf16_to_f32(b).astype(np.float64)
    ref = oracle.bf16_to_f32(a).astype(np.float64) @ (bf if layout == "kn" else bf.T)
    assert rel_err(got, ref) < 1e-6
    got16 = oracle.gemm(a, b, b_layout=layout)
    assert np.array_equal(got16, oracle.f32_to_bf16(got))


def test_gemm_with_addend():
    rng = np.random.default_rng(2)
    a = oracle.normal_bf16(rng, (16, 32))
    b = oracle.normal_bf16(rng, (32, 24))
    c = oracle.normal_bf16(rng, (16, 24))
    d = oracle.gemm(a, b, c=c)
    acc = oracle.gemm(a, b, out_f32=True)
    assert np.array_equal(d, oracle.f32_to_bf16(acc + oracle.bf16_to_f32(c)))


def test_rmsnorm_matches_float64():
    rng = np.random.default_rng(3)
    x = oracle.normal_bf16(rng, (9, 4096))
    g = oracle.normal_bf16(rng, (4096,))
    y = oracle.rmsnorm(x, g, 1e-5)
    xf = oracle.bf16_to_f32(x).astype(np.float64)
    ref = xf / np.sqrt((xf ** 2).mean(-1, keepdims=True) + 1e-5) * oracle.bf16_to_f32(g)
    assert rel_err(oracle.bf16_to_f32(y), ref) < 4e-3


def test_silu_mul_matches_float64():
    rng = np.random.default_rng(4)
    g = oracle.normal_bf16(rng, (4096,), 3.0)
    u = oracle.normal_bf16(rng, (4096,))
    h = oracle.silu_mul(g, u)
    gf = oracle.bf16_to_f32(g).astype(np.float64)
    ref = gf / (1 + np.exp(-gf)) * oracle.bf16_to_f32(u)
    assert rel_err(oracle.bf16_to_f32(h), ref) < 4e-3


def test_gemm_silu_gate_and_packing():
    rng = np.random.default_rng(5)
    M, F, K = 20, 256, 64
    a = oracle.normal_bf16(rng, (M, K))
    wg = oracle.normal_bf16(rng, (1, F, K))
    wu = oracle.normal_bf16(rng, (1, F, K))
    h = oracle.gemm_silu_gate(a, wg[0], wu[0])
    w13 = oracle.pack_gate_up(wg, wu)
    assert np.array_equal(w13[0, 0:64], wg[0, 0:64])
    assert np.array_equal(w13[0, 64:128], wu[0, 0:64])
    assert np.array_equal(w13[0, 128:192], wg[0, 64:128])
    assert np.array_equal(w13[0, 448:512], wu[0, 192:256])
    off = np.array([0, M], dtype=np.int32)
    h2 = oracle.grouped_gemm(a, w13, off, silu_gate=True)
    assert np.array_equal(h, h2)


def test_topk_ties_pick_lower_index_and_weights_are_softmax():
    logits = np.zeros((3, 8), dtype=np.float32)
    logits[0] = [1, 5, 5, 0, 0, 0, 0, 5]
    logits[1] = np.arange(8, dtype=np.float32)
    logits[2] = 0.0  # all equal
    idx, w = oracle.moe_topk(logits, 2)
    assert idx.tolist() == [[1, 2], [7, 6], [0, 1]]
    p = np.exp(logits[1] - logits[1].max())
    p /= p.sum()
    assert np.allclose(w[1], [p[7], p[6]], rtol=1e-6)
    assert np.allclose(w[2], [1 / 8, 1 / 8])


def test_permute_is_stable_expert_major():
    idx = np.array([[3, 1], [1, 0], [3, 2], [1, 3]], dtype=np.int32)
    off, pos, src = oracle.moe_permute(idx, 5)
    assert off.tolist() == [0, 1, 4, 5, 8, 8]
    # pairs (t,j) in expert order: e0:(1,1) e1:(0,1),(1,0),(3,0) e2:(2,1) e3:(0,0),(2,0),(3,1)
    assert pos.tolist() == [5, 1, 2, 0, 6, 4, 3, 7]
    assert src.tolist() == [1, 0, 1, 3, 2, 0, 2, 3]
    with pytest.raises(ValueError):
        oracle.moe_permute(np.array([[5, 0]], dtype=np.int32), 5)


def test_scatter_then_combine_round_trip():
    rng = np.random.default_rng(6)
    T, k, H, E = 11, 2, 16, 4
    x = oracle.normal_bf16(rng, (T, H))
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    off, pos, src = oracle.moe_permute(idx, E)
    xp = oracle.moe_scatter_rows(x, pos, k)
    assert np.array_equal(xp[pos.reshape(T, k)[:, 0]], x)
    assert np.array_equal(src, np.repeat(np.arange(T), k)[np.argsort(pos)])
    w = np.full((T, k), 0.5, dtype=np.float32)
    out = oracle.moe_combine(xp, pos, w)   # 0.5*x + 0.5*x == x exactly
    assert np.array_equal(out, x)


def test_moe_layer_composes_the_steps():
    rng = np.random.default_rng(7)
    T, H, E, F, k = 32, 64, 8, 128, 2
    x = oracle.normal_bf16(rng, (T, H))
    wr = oracle.normal_bf16(rng, (E, H), 0.02)
    w13 = oracle.normal_bf16(rng, (E, 2 * F, H), 0.02)
    w2 = oracle.normal_bf16(rng, (E, H, F), 0.02)
    out, logits, idx, tw = oracle.moe_layer(x, wr, w13, w2, k)
    assert np.array_equal(logits, oracle.gemm(x, wr, b_layout="nk", out_f32=True))
    idx2, tw2 = oracle.moe_topk(logits, k)
    assert np.array_equal(idx, idx2) and np.array_equal(tw, tw2)
    off, pos, _ = oracle.moe_permute(idx, E)
    xp = oracle.moe_scatter_rows(x, pos, k)
    h = oracle.grouped_gemm(xp, w13, off, silu_gate=True)
    y = oracle.grouped_gemm(h, w2, off)
    assert np.array_equal(out, oracle.moe_combine(y, pos, tw))


def test_attention_oracle_matches_float64():
    rng = np.random.default_rng(8)
    B, L, HQ, HKV, hd = 2, 40, 4, 2, 128
    q = oracle.normal_bf16(rng, (B * L, HQ * hd))
    k = oracle.normal_bf16(rng, (B * L, HKV * hd))
    v = oracle.normal_bf16(rng, (B * L, HKV * hd))
    out = oracle.bf16_to_f32(oracle.attention(q, k, v, B, HQ, HKV))
    qf, kf, vf = (oracle.bf16_to_f32(a).astype(np.float64) for a in (q, k, v))
    ref = np.zeros_like(out, dtype=np.float64)
    for b in range(B):
        for h in range(HQ):
            kh = h // (HQ // HKV)
            Q = qf[b * L:(b + 1) * L, h * hd:(h + 1) * hd]
            K = kf[b * L:(b + 1) * L, kh * hd:(kh + 1) * hd]
            V = vf[b * L:(b + 1) * L, kh * hd:(kh + 1) * hd]
            S = Q @ K.T / np.sqrt(hd)
            S[np.triu_indices(L, 1)] = -np.inf
            P = np.exp(S - S.max(1, keepdims=True))
            P /= P.sum(1, keepdims=True)
            ref[b * L:(b + 1) * L, h * hd:(h + 1) * hd] = P @ V
    assert rel_err(out, ref) < 1e-2


def test_rope_oracle_matches_float64():
    rng = np.random.default_rng(9)
    L, heads, hd = 16, 2, 128
    x = oracle.normal_bf16(rng, (2 * L, heads * hd))
    got = oracle.bf16_to_f32(oracle.rope(x, L, heads))
    xf = oracle.bf16_to_f32(x).astype(np.float64)
    ref = np.empty_like(xf)
    for r in range(2 * L):
        pos = r % L
        for h in range(heads):
            v = xf[r, h * hd:(h + 1) * hd]
            th = pos * 10000.0 ** (-2.0 * np.arange(hd // 2) / hd)
            a, b = v[:hd // 2], v[hd // 2:]
            ref[r, h * hd:h * hd + hd // 2] = a * np.cos(th) - b * np.sin(th)
            ref[r, h * hd + hd // 2:(h + 1) * hd] = b * np.cos(th) + a * np.sin(th)
    assert rel_err(got, ref) < 4e-3


def test_paged_kv_oracle_matches_dense_attention():
    """Writing a sequence into shuffled pages, reading it back and decoding
    every row over the pages equals the dense causal attention oracle."""
    rng = np.random.default_rng(9)
    HKV, HQ, L, bs, pages, layers = 2, 4, 70, 16, 12, 2
    W = HKV * 128
    for layout in ("page_first", "layer_first"):
        st = oracle.kv_strides(layout, pages, layers, bs, W)
        pool = np.zeros(pages * layers * 2 * bs * W, dtype=np.uint16)
        bt = rng.permutation(pages)[:5].astype(np.int32)
        k = oracle.normal_bf16(rng, (L, W))
        v = oracle.normal_bf16(rng, (L, W))
        q = oracle.normal_bf16(rng, (L, HQ * 128))
        pool = oracle.kvcache_write(pool, st, bs, 1, k, v, [0, L], [0], bt, [0, 5])
        kr, vr = oracle.kvcache_read(pool, st, bs, 1, W, [0, L], bt, [0, 5])
        assert np.array_equal(kr, k) and np.array_equal(vr, v)
        out = oracle.attention_decode(q, pool, st, bs, 1, [0, L], [0], bt, [0, 5], HQ, HKV)
        ref = oracle.attention(q, k, v, 1, HQ, HKV)
        assert rel_err(oracle.bf16_to_f32(out), oracle.bf16_to_f32(ref)) < 1e-2
        # layer 0 untouched
        other = oracle.kvcache_read(pool, st, bs, 0, W, [0, L], bt, [0, 5])[0]
        assert not other.any()


def test_moe_layer_given_routing_matches_the_whole_layer():
    """The composed post-routing oracle (permute, scatter, grouped GEMMs,
    combine) reproduces orc_moe_layer bit for bit when given its routing, and
    the router logits the layer tests compute separately are the layer's."""
    rng = np.random.default_rng(5)
    T, H, E, F, k = 96, 64, 8, 128, 2
    x = oracle.normal_bf16(rng, (T, H))
    wr = oracle.normal_bf16(rng, (E, H), 0.02)
    w13 = oracle.normal_bf16(rng, (E, 2 * F, H), 0.02)
    w2 = oracle.normal_bf16(rng, (E, H, F), 0.02)
    out, logits, idx, tw = oracle.moe_layer(x, wr, w13, w2, k)
    assert np.array_equal(oracle.moe_layer_given_routing(x, w13, w2, idx, tw), out)
    lg = oracle.gemm(x, wr, b_layout="nk", out_f32=True)
    assert np.array_equal(lg.view(np.uint32), logits.view(np.uint32))
    gaps = oracle.topk_gap(logits, k)
    s = np.sort(logits, axis=1)
    assert np.allclose(gaps, s[:, -k] - s[:, -k - 1])
