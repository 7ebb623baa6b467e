"""Paged KV cache (kvcache.write / kvcache.read) and decode attention over it
against the oracle: the cache contents and gathers bit-exact, attention
within bf16 tolerance (relative L2 <= 1e-2)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import from_bits, rel_err, to_bits
from kvm_b200 import ops
from kvm_b200.kvcache import PagedKVCache

pytestmark = pytest.mark.gpu


def _tables(rng, pages, bs, lens):
    """Distinct random pages for each sequence (lens = tokens it will hold)."""
    need = [(n + bs - 1) // bs for n in lens]
    ids = rng.permutation(pages)[:sum(need)].astype(np.int32)
    off = np.concatenate([[0], np.cumsum(need)]).astype(np.int32)
    return ids, off


def _i32(a, dev):
    return torch.from_numpy(np.asarray(a, dtype=np.int32)).to(dev)


def _run(cuda, rng, *, layout, bs, HQ, HKV, ctx, nq, layers=2, layer=1, garbage=False):
    W = HKV * 128
    S = len(ctx)
    total = [c + n for c, n in zip(ctx, nq)]
    need_pages = sum((t + bs - 1) // bs for t in total)
    pages = need_pages + 5
    cache = PagedKVCache(pages=pages, layers=layers, block_size=bs, heads_kv=HKV,
                         layout=layout, device=cuda)
    if garbage:  # stale NaN bits everywhere a token was never written
        cache.pool.view(torch.int16).fill_(0x7FC0)
    pool = to_bits(cache.pool)
    bt, bt_off = _tables(rng, pages, bs, total)
    strides = cache.strides
    # 1) the context tokens, 2) the new tokens
    ctx_off = np.concatenate([[0], np.cumsum(ctx)]).astype(np.int32)
    new_off = np.concatenate([[0], np.cumsum(nq)]).astype(np.int32)
    kc = oracle.normal_bf16(rng, (int(ctx_off[-1]), W))
    vc = oracle.normal_bf16(rng, (int(ctx_off[-1]), W))
    kn = oracle.normal_bf16(rng, (int(new_off[-1]), W))
    vn = oracle.normal_bf16(rng, (int(new_off[-1]), W))
    q = oracle.normal_bf16(rng, (int(new_off[-1]), HQ * 128))
    zeros = np.zeros(S, dtype=np.int32)
    pool = oracle.kvcache_write(pool, strides, bs, layer, kc, vc, ctx_off, zeros, bt, bt_off)
    pool = oracle.kvcache_write(pool, strides, bs, layer, kn, vn, new_off,
                                np.asarray(ctx, dtype=np.int32), bt, bt_off)
    bt_d, bto_d = _i32(bt, cuda), _i32(bt_off, cuda)
    if ctx_off[-1] > 0:
        cache.write(layer, from_bits(kc, cuda), from_bits(vc, cuda), _i32(ctx_off, cuda),
                    _i32(zeros, cuda), bt_d, bto_d)
    cache.write(layer, from_bits(kn, cuda), from_bits(vn, cuda), _i32(new_off, cuda),
                _i32(ctx, cuda), bt_d, bto_d)
    ops.device_status()
    assert np.array_equal(to_bits(cache.pool), pool)
    # gather everything back
    kv_off = np.concatenate([[0], np.cumsum(total)]).astype(np.int32)
    k_ref, v_ref = oracle.kvcache_read(pool, strides, bs, layer, W, kv_off, bt, bt_off)
    k_got, v_got = cache.read(layer, _i32(kv_off, cuda), bt_d, bto_d, int(kv_off[-1]))
    ops.device_status()
    assert np.array_equal(to_bits(k_got), k_ref) and np.array_equal(to_bits(v_got), v_ref)
    # decode the new rows
    ref = oracle.attention_decode(q, pool, strides, bs, layer, new_off,
                                  np.asarray(ctx, dtype=np.int32), bt, bt_off, HQ, HKV)
    out = cache.decode(layer, from_bits(q, cuda), _i32(new_off, cuda), _i32(ctx, cuda),
                       bt_d, bto_d, heads_q=HQ, max_q_rows=max(nq), max_keys=max(total))
    ops.device_status()
    got = oracle.bf16_to_f32(to_bits(out))
    assert np.isfinite(got).all()
    r = oracle.bf16_to_f32(ref)
    assert rel_err(got, r) < 1e-2
    for s in range(S):   # each sequence on its own
        lo, hi = new_off[s], new_off[s + 1]
        assert rel_err(got[lo:hi], r[lo:hi]) < 1e-2, s


def test_paged_decode_page_first_gqa8(cuda):
    """16-token pages; a fresh sequence, one spanning two key chunks with
    six new rows (two query groups of four at 8 heads per kv head)."""
    _run(cuda, np.random.default_rng(1), layout="page_first", bs=16, HQ=16, HKV=2,
         ctx=[0, 1030, 200], nq=[1, 6, 3])


def test_paged_decode_layer_first_big_pages(cuda):
    """256-token pages (a 128-key tile inside one page), one query head per kv
    head, 40 new rows (two query groups of 32)."""
    _run(cuda, np.random.default_rng(2), layout="layer_first", bs=256, HQ=4, HKV=4,
         ctx=[2100, 77], nq=[1, 40])


def test_paged_decode_ignores_stale_slots(cuda):
    """Slots never written hold NaN bits; the partially filled last page must
    not leak them into the output."""
    _run(cuda, np.random.default_rng(3), layout="page_first", bs=32, HQ=8, HKV=1,
         ctx=[45, 130], nq=[2, 1], garbage=True)


def test_kvcache_write_rejects_bad_page(cuda):
    from kvm_b200._lib import KvmError
    cache = PagedKVCache(pages=4, layers=1, block_size=16, heads_kv=1, device=cuda)
    k = torch.zeros((1, 128), dtype=torch.bfloat16, device=cuda)
    cache.write(0, k, k, _i32([0, 1], cuda), _i32([0], cuda), _i32([9], cuda),
                _i32([0, 1], cuda))
    with pytest.raises(KvmError):
        ops.device_status()
