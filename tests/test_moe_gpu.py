"""MoE dispatch / grouped GEMM / combine parity against the oracle.

Routing indices, permutation, offsets and the scatter copy are compared
bit-exactly given the same inputs (the GPU's logits are fed to the oracle's
top-k, since fp32 logits from different accumulation orders can differ in the
last bits). Combine is bit-exact given the same expert outputs. GEMM outputs
use the bf16 tolerance: relative L2 error <= 1e-2.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import check_moe_routing_and_layer, from_bits, rel_err, to_bits
from kvm_b200 import ops

pytestmark = pytest.mark.gpu


def _weights(rng, E, H, F):
    wr = oracle.normal_bf16(rng, (E, H), 0.02)
    w13 = oracle.normal_bf16(rng, (E, 2 * F, H), 0.02)
    w2 = oracle.normal_bf16(rng, (E, H, F), 0.02)
    return wr, w13, w2


@pytest.mark.parametrize("T,k,E", [(512, 2, 64), (1, 2, 64), (300, 1, 64), (129, 8, 64),
                                   (700, 2, 16), (64, 3, 5),
                                   # tiles of 56, 32 and 88 rows on 148 SMs, ragged
                                   # last tiles
                                   (8192, 2, 64), (4099, 2, 64), (12000, 2, 64),
                                   # more than 64 experts: 128- and 256-column tiles
                                   (1024, 2, 96), (600, 8, 128), (300, 2, 200),
                                   (256, 4, 256)])
def test_router_topk_bit_exact_given_logits(cuda, T, k, E):
    rng = np.random.default_rng(T + k)
    H = 256
    x = oracle.normal_bf16(rng, (T, H))
    wr = oracle.normal_bf16(rng, (E, H), 0.02)
    r = ops.moe_route(from_bits(x, cuda), from_bits(wr, cuda), top_k=k)
    ops.device_status()
    logits = r.logits.cpu().numpy()
    ref_logits = oracle.gemm(x, wr, b_layout="nk", out_f32=True)
    assert rel_err(logits, ref_logits) < 1e-5
    idx, w = oracle.moe_topk(logits, k)
    assert np.array_equal(r.topk_idx.cpu().numpy(), idx)
    np.testing.assert_allclose(r.topk_w.cpu().numpy(), w, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("H", [4096, 200, 64])
def test_router_logits_do_not_depend_on_the_batch(cuda, H):
    """A token's logits are the same bits whichever batch (and so tile and
    CTA) it is routed in: the expert-parallel layer relies on it. H = 200
    ends in a partial K block; H = 64 is a single one."""
    rng = np.random.default_rng(H)
    T, E, k = 8192, 64, 2
    x = from_bits(oracle.normal_bf16(rng, (T, H)), cuda)
    wr = from_bits(oracle.normal_bf16(rng, (E, H), 0.02), cuda)
    full = ops.moe_route(x, wr, top_k=k)
    part = ops.moe_route(x[T - 300:].contiguous(), wr, top_k=k)
    ops.device_status()
    a = full.logits[T - 300:].cpu().numpy().view(np.uint32)
    b = part.logits.cpu().numpy().view(np.uint32)
    assert np.array_equal(a, b)
    assert np.array_equal(full.topk_idx[T - 300:].cpu().numpy(), part.topk_idx.cpu().numpy())
    ref = oracle.gemm(to_bits(x[:64]), to_bits(wr), b_layout="nk", out_f32=True)
    assert rel_err(full.logits[:64].cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("T,H,E,k", [
    # one K block: the second CTA of each SM pair has no K half (its partial
    # is zero), and 157 tiles of 128 rows give the pairs two or three tiles
    # each (the exchange buffers of both tile parities in use)
    (20000, 64, 37, 3),
    # one expert; an odd number of 64-deep K blocks (K halves of 2 and 1)
    (333, 192, 1, 1),
    # a partial last K block in the second half, all 8 of 64 experts taken
    (5000, 4000, 64, 8)])
def test_router_sm_pairs_edge_shapes(cuda, T, H, E, k):
    """The E <= 64 router (SM pairs, K split in two) at shapes that reach its
    corner paths, against the oracle."""
    rng = np.random.default_rng(T + H + E)
    x = oracle.normal_bf16(rng, (T, H))
    wr = oracle.normal_bf16(rng, (E, H), 0.05)
    r = ops.moe_route(from_bits(x, cuda), from_bits(wr, cuda), top_k=k)
    ops.device_status()
    logits = r.logits.cpu().numpy()
    assert rel_err(logits, oracle.gemm(x, wr, b_layout="nk", out_f32=True)) < 1e-5
    idx, w = oracle.moe_topk(logits, k)
    assert np.array_equal(r.topk_idx.cpu().numpy(), idx)
    np.testing.assert_allclose(r.topk_w.cpu().numpy(), w, rtol=1e-5, atol=1e-7)


def test_router_ties_take_lower_expert(cuda):
    T, H, E = 128, 64, 64
    x = np.zeros((T, H), dtype=np.uint16)
    x[:, 0] = oracle.f32_to_bf16(np.ones(T, dtype=np.float32))
    wr = np.zeros((E, H), dtype=np.uint16)  # every logit 0 except a few equal maxima
    wr[[5, 9, 40], 0] = oracle.f32_to_bf16(np.full(3, 2.0, dtype=np.float32))
    r = ops.moe_route(from_bits(x, cuda), from_bits(wr, cuda), top_k=4)
    ops.device_status()
    assert (r.topk_idx.cpu().numpy() == np.array([5, 9, 40, 0])).all()


@pytest.mark.parametrize("T,k,E,skew", [(4096, 2, 64, False), (1000, 2, 64, True),
                                        (7, 3, 64, False), (2048, 8, 16, False),
                                        (513, 1, 1, False),
                                        # more experts than threads per block
                                        (600, 2, 300, False),
                                        # count matrix over 16K cells: separate scan
                                        (40000, 2, 64, False)])
def test_permute_and_scatter_bit_exact(cuda, T, k, E, skew):
    rng = np.random.default_rng(T * 3 + k)
    if skew:   # most pairs on two experts, many experts empty
        idx = np.where(rng.random((T, k)) < 0.9, rng.integers(0, 2, (T, k)),
                       rng.integers(0, E, (T, k))).astype(np.int32)
    else:
        idx = rng.integers(0, E, (T, k)).astype(np.int32)
    off, pos, src = oracle.moe_permute(idx, E)
    d = ops.moe_permute(torch.from_numpy(idx).to(cuda), E)
    ops.device_status()
    assert np.array_equal(d.offsets.cpu().numpy(), off)
    assert np.array_equal(d.pos.cpu().numpy(), pos)
    assert np.array_equal(d.src_token.cpu().numpy(), src)
    H = 136
    x = oracle.normal_bf16(rng, (T, H))
    xp = ops.moe_scatter_rows(from_bits(x, cuda), d.pos, k)
    ops.device_status()
    assert np.array_equal(to_bits(xp), oracle.moe_scatter_rows(x, pos, k))


def test_permute_rejects_bad_expert_index(cuda):
    idx = torch.tensor([[0, 70]], dtype=torch.int32, device=cuda)
    ops.moe_permute(idx, 64)
    from kvm_b200._lib import KvmError
    with pytest.raises(KvmError):
        ops.device_status()


@pytest.mark.parametrize("silu", [False, True])
def test_grouped_gemm(cuda, silu):
    rng = np.random.default_rng(21 + silu)
    G, K = 12, 320
    N = 512 if silu else 384
    counts = rng.integers(0, 300, G)
    counts[3] = 0          # empty group
    counts[7] = 1          # single row
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    rows = int(off[-1])
    a = oracle.normal_bf16(rng, (rows, K))
    w = oracle.normal_bf16(rng, (G, N, K), 0.05)
    ref = oracle.grouped_gemm(a, w, off, silu_gate=silu)
    got = ops.grouped_matmul(from_bits(a, cuda), from_bits(w, cuda),
                             torch.from_numpy(off).to(cuda), silu_gate=silu)
    ops.device_status()
    g, r = oracle.bf16_to_f32(to_bits(got)), oracle.bf16_to_f32(ref)
    assert rel_err(g, r) < 1e-2


@pytest.mark.parametrize("silu", [False, True])
def test_grouped_gemm_wide_groups(cuda, silu):
    """Groups around and past the 256-token MMA width and the 512-token pair
    tile: one and two MMAs per tile, several tiles per group, ragged ends."""
    rng = np.random.default_rng(23 + silu)
    K = 192
    N = 512 if silu else 384
    counts = np.array([0, 1, 255, 256, 257, 300, 511, 512, 513, 1000, 1537, 16, 17])
    G = len(counts)
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    rows = int(off[-1])
    a = oracle.normal_bf16(rng, (rows, K))
    w = oracle.normal_bf16(rng, (G, N, K), 0.05)
    ref = oracle.grouped_gemm(a, w, off, silu_gate=silu)
    got = ops.grouped_matmul(from_bits(a, cuda), from_bits(w, cuda),
                             torch.from_numpy(off).to(cuda), silu_gate=silu)
    ops.device_status()
    g, r = oracle.bf16_to_f32(to_bits(got)), oracle.bf16_to_f32(ref)
    assert rel_err(g, r) < 1e-2
    # every group's rows, checked separately (a wrong tile shows up per group)
    for i in range(G):
        lo, hi = off[i], off[i + 1]
        if hi > lo:
            assert rel_err(g[lo:hi], r[lo:hi]) < 1e-2, i


@pytest.mark.parametrize("silu", [False, True])
def test_grouped_gemm_groups_just_past_one_tile(cuda, silu):
    """Groups of 257..289 tokens (two token tiles of 136..152 columns) beside
    groups of every other size class, each group checked on its own rows, and
    nothing written past the last row."""
    rng = np.random.default_rng(29 + silu)
    K = 256
    N = 512 if silu else 768
    counts = np.array([257, 264, 270, 272, 273, 280, 287, 288, 289, 256, 255, 1, 0, 300,
                       258, 520])
    G = len(counts)
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    rows = int(off[-1])
    a = oracle.normal_bf16(rng, (rows, K))
    w = oracle.normal_bf16(rng, (G, N, K), 0.05)
    ref = oracle.grouped_gemm(a, w, off, silu_gate=silu)
    out_n = N // 2 if silu else N
    canary = torch.full((rows + 64, out_n), 7.0, dtype=torch.bfloat16, device=cuda)
    got = ops.grouped_matmul(from_bits(a, cuda), from_bits(w, cuda),
                             torch.from_numpy(off).to(cuda), silu_gate=silu,
                             out=canary[:rows])
    ops.device_status()
    assert torch.all(canary[rows:] == 7.0)  # nothing written past the last row
    g, r = oracle.bf16_to_f32(to_bits(got)), oracle.bf16_to_f32(ref)
    for i in range(G):
        lo, hi = off[i], off[i + 1]
        if hi > lo:
            assert rel_err(g[lo:hi], r[lo:hi]) < 1e-2, (i, counts[i])


def test_combine_bit_exact(cuda):
    rng = np.random.default_rng(31)
    T, k, H, E = 777, 2, 512, 64
    idx = rng.integers(0, E, (T, k)).astype(np.int32)
    off, pos, _ = oracle.moe_permute(idx, E)
    y = oracle.normal_bf16(rng, (T * k, H))
    w = rng.random((T, k), dtype=np.float32)
    ref = oracle.moe_combine(y, pos, w)
    got = ops.moe_combine(from_bits(y, cuda), torch.from_numpy(pos).to(cuda),
                          torch.from_numpy(w).to(cuda))
    ops.device_status()
    assert np.array_equal(to_bits(got), ref)


def test_moe_layer_end_to_end(cuda):
    from kvm_b200.moe import MoELayer
    rng = np.random.default_rng(41)
    T, H, E, F, k = 1024, 512, 64, 256, 2
    x = oracle.normal_bf16(rng, (T, H))
    wr, w13, w2 = _weights(rng, E, H, F)
    ref, ref_logits, ref_idx, _ = oracle.moe_layer(x, wr, w13, w2, k)
    layer = MoELayer.from_packed(from_bits(wr, cuda), from_bits(w13, cuda),
                                 from_bits(w2, cuda), top_k=k, max_tokens=T)
    out = layer(from_bits(x, cuda))
    ops.device_status()
    n = check_moe_routing_and_layer(layer, x, w13, w2, wr, out, k)
    assert n <= T // 100
    # the layer's own top-k agrees with the oracle's whole layer off the ties
    same = (layer.last_routing.topk_idx.cpu().numpy() == ref_idx).all(axis=1)
    assert rel_err(oracle.bf16_to_f32(to_bits(out))[same],
                   oracle.bf16_to_f32(ref)[same]) < 1e-2


def test_host_pipeline_matches_layer(cuda):
    """HostPipeline (pinned host batches, copies overlapped with compute on
    three streams) returns, for every batch, exactly what the layer returns
    for that batch on one stream -- including a ragged last batch and more
    batches than device slots."""
    from kvm_b200.moe import MoELayer
    from kvm_b200.pipeline import HostPipeline
    rng = np.random.default_rng(43)
    T, H, E, F, k = 512, 512, 16, 256, 2
    wr, w13, w2 = _weights(rng, E, H, F)
    layer = MoELayer.from_packed(from_bits(wr, cuda), from_bits(w13, cuda),
                                 from_bits(w2, cuda), top_k=k, max_tokens=T)
    sizes = [512, 512, 300, 512, 7]
    xs = [oracle.normal_bf16(rng, (n, H)) for n in sizes]
    want = [to_bits(layer(from_bits(x, cuda)).clone()) for x in xs]
    pipe = HostPipeline(layer, T, H, depth=2, device=cuda)
    hin = [from_bits(x, "cpu").pin_memory() for x in xs]
    hout = [torch.empty((n, H), dtype=torch.bfloat16).pin_memory() for n in sizes]
    for a, b in zip(hin, hout):
        pipe.submit(a, b)
    pipe.synchronize()
    ops.device_status()
    for i, (w, o) in enumerate(zip(want, hout)):
        assert np.array_equal(to_bits(o), w), i
    with pytest.raises(ValueError):
        pipe.submit(torch.empty((4, H), dtype=torch.bfloat16), hout[0][:4])
