"""Expert-parallel MoE exchange logic on CPU ranks (gloo), with the oracle as
each rank's local compute. Every output row depends only on its own token and
the expert weights, so the sharded layer must equal the single-process oracle
layer on the concatenated tokens bit for bit."""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from kvm_b200.ep import ExpertParallelMoENccl, make_plan

T, H, E, F, K = 48, 64, 8, 128, 2


def _weights():
    rng = np.random.default_rng(99)
    wr = oracle.normal_bf16(rng, (E, H), 0.5)
    w13 = oracle.normal_bf16(rng, (E, 2 * F, H), 0.05)
    w2 = oracle.normal_bf16(rng, (E, H, F), 0.05)
    return wr, w13, w2


def _tokens(rank):
    return oracle.normal_bf16(np.random.default_rng(1000 + rank), (T, H))


def _i16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16))


class OracleCompute:
    """One rank's local compute through the oracle (CPU tensors of bf16 bits)."""

    def __init__(self, wr, w13_local, w2_local, world):
        self.wr, self.w13, self.w2 = wr, w13_local, w2_local
        self.recv = torch.zeros((T * K * world, H), dtype=torch.int16)
        self.yback = torch.zeros((T * K, H), dtype=torch.int16)

    def dispatch_local(self, x):
        xb = x.numpy().view(np.uint16)
        logits = oracle.gemm(xb, self.wr, b_layout="nk", out_f32=True)
        idx, self.w = oracle.moe_topk(logits, K)
        off, self.pos, _ = oracle.moe_permute(idx, E)
        xp = oracle.moe_scatter_rows(xb, self.pos, K)
        return _i16(xp), torch.from_numpy(off)

    def experts(self, rows, local_offsets):
        off = np.asarray(local_offsets, dtype=np.int32)
        a = np.ascontiguousarray(self.recv[:rows].numpy().view(np.uint16))
        h = oracle.grouped_gemm(a, self.w13, off, silu_gate=True)
        y = oracle.grouped_gemm(h, self.w2, off)
        out = torch.zeros((max(rows, 1), H), dtype=torch.int16)
        out[:rows] = _i16(y)
        return out

    def combine_local(self, n):
        yb = self.yback.numpy().view(np.uint16)
        return _i16(oracle.moe_combine(yb, self.pos, self.w))


def _worker(rank, world, outdir):
    # file rendezvous in the test's own directory: no port to race for
    dist.init_process_group("gloo", init_method=f"file://{outdir}/rendezvous", rank=rank,
                            world_size=world)
    try:
        wr, w13, w2 = _weights()
        epr = E // world
        sl = slice(rank * epr, (rank + 1) * epr)
        comp = OracleCompute(wr, np.ascontiguousarray(w13[sl]),
                             np.ascontiguousarray(w2[sl]), world)
        layer = ExpertParallelMoENccl(_i16(wr), _i16(w13), _i16(w2), top_k=K, max_tokens=T,
                                  rank=rank, world=world, compute=comp)
        out = layer(_i16(_tokens(rank)))
        np.save(os.path.join(outdir, f"out{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_matches_single_process(world):
    wr, w13, w2 = _weights()
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, d), nprocs=world,
                           start_method="spawn")
        outs = [np.load(os.path.join(d, f"out{r}.npy")).view(np.uint16)
                for r in range(world)]
    x_all = np.concatenate([_tokens(r) for r in range(world)])
    ref, *_ = oracle.moe_layer(x_all, wr, w13, w2, K)
    assert np.array_equal(np.concatenate(outs), ref)


def test_plan_orders_messages_by_expert_and_source():
    # 2 ranks, 4 experts (2 per rank). This is rank 1.
    send_offsets = [0, 3, 3, 7, 9]          # rows for experts 0..3
    recv_counts = [2, 0, 4, 2]              # from rank0: e2=2,e3=0; from rank1: e2=4,e3=2
    p = make_plan(1, 2, 4, send_offsets, recv_counts)
    assert p.send == [(0, 0, 3), (1, 3, 4), (1, 7, 2)]
    assert p.local_offsets == [0, 6, 8]
    assert p.recv == [(0, 0, 2), (1, 2, 4), (1, 6, 2)]
    assert p.recv_rows == 8
