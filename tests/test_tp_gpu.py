"""Tensor-parallel decoder layer: one GPU against the oracle composed op by op,
and 2+ GPUs (column/row-parallel shards with NCCL all-reduce) against one GPU.
bf16 tolerance: relative L2 <= 1e-2."""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from helpers import from_bits, rel_err, to_bits

pytestmark = pytest.mark.gpu
B, L, H, HQ, HKV, F = 2, 256, 512, 4, 2, 1024


def _full(seed=11, hq=HQ, hkv=HKV):
    rng = np.random.default_rng(seed)
    w = dict(wq=oracle.normal_bf16(rng, (hq * 128, H), 0.05),
             wk=oracle.normal_bf16(rng, (hkv * 128, H), 0.05),
             wv=oracle.normal_bf16(rng, (hkv * 128, H), 0.05),
             wo=oracle.normal_bf16(rng, (H, hq * 128), 0.05),
             wg=oracle.normal_bf16(rng, (F, H), 0.05),
             wu=oracle.normal_bf16(rng, (F, H), 0.05),
             w2=oracle.normal_bf16(rng, (H, F), 0.05),
             g1=oracle.normal_bf16(rng, (H,)), g2=oracle.normal_bf16(rng, (H,)))
    x = oracle.normal_bf16(rng, (B * L, H))
    return w, x


def _oracle_layer(w, x, hq=HQ, hkv=HKV):
    xn = oracle.rmsnorm(x, w["g1"], 1e-5)
    qkv = oracle.gemm(xn, np.concatenate([w["wq"], w["wk"], w["wv"]]), b_layout="nk")
    q = np.ascontiguousarray(qkv[:, :hq * 128])
    k = np.ascontiguousarray(qkv[:, hq * 128:(hq + hkv) * 128])
    v = np.ascontiguousarray(qkv[:, (hq + hkv) * 128:])
    q, k = oracle.rope(q, L, hq), oracle.rope(k, L, hkv)
    a = oracle.attention(q, k, v, B, hq, hkv)
    h1 = oracle.gemm(a, w["wo"], b_layout="nk", c=x)
    h1n = oracle.rmsnorm(h1, w["g2"], 1e-5)
    act = oracle.gemm_silu_gate(h1n, w["wg"], w["wu"])
    return oracle.gemm(act, w["w2"], b_layout="nk", c=h1)


def _layer(w, dev, rank=0, world=1, hq=HQ, hkv=HKV):
    from kvm_b200.tp import TPDecoderLayer
    t = {k: from_bits(v, dev) for k, v in w.items()}
    return TPDecoderLayer.from_full(t["wq"], t["wk"], t["wv"], t["wo"], t["wg"], t["wu"],
                                    t["w2"], t["g1"], t["g2"], batch=B, seq_len=L,
                                    heads_q=hq, heads_kv=hkv, rank=rank, world=world)


def test_decoder_layer_single_gpu(cuda):
    from kvm_b200 import ops
    w, x = _full()
    ref = _oracle_layer(w, x)
    out = _layer(w, cuda)(from_bits(x, cuda))
    ops.device_status()
    assert rel_err(oracle.bf16_to_f32(to_bits(out)), oracle.bf16_to_f32(ref)) < 1e-2


def _worker(rank, world, outdir, hq, hkv):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # file rendezvous in the test's own directory: no port to race for
    dist.init_process_group("nccl", init_method=f"file://{outdir}/rendezvous", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        w, x = _full(hq=hq, hkv=hkv)
        out = _layer(w, dev, rank, world, hq, hkv)(from_bits(x, dev))
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"out{rank}.npy"), to_bits(out))
    finally:
        dist.destroy_process_group()



@pytest.mark.parametrize("world,hq,hkv", [(2, 4, 2), (4, 8, 4), (8, 16, 8)])
def test_decoder_layer_tensor_parallel(world, hq, hkv):
    """Heads split hq/world and hkv/world per rank (one kv head per rank at 8)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    w, x = _full(hq=hq, hkv=hkv)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, d, hq, hkv), nprocs=world,
                           start_method="spawn")
        outs = [np.load(os.path.join(d, f"out{r}.npy")) for r in range(world)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])   # all-reduce: same on all
    ref = _oracle_layer(w, x, hq, hkv)
    assert rel_err(oracle.bf16_to_f32(outs[0]), oracle.bf16_to_f32(ref)) < 1e-2
