"""Tensor-parallel decoder layer on the sm_100a kernels (one process per GPU).

    h1  = x + O( attn( rope(Q), rope(K), V ) )     Q, K, V = RMSNorm(x) . Wqkv
    out = h1 + Wd( SiLU(RMSNorm(h1) . Wg) * (RMSNorm(h1) . Wu) )

Column-parallel: Wqkv (each rank owns HQ/P query heads and HKV/P kv heads)
and the gate/up projection (FFN/P columns). Row-parallel: the output and down
projections, each followed by a sum all-reduce of the [T, hidden] partials
(`comm.all_reduce.sum`, src/ir/dialect/kernel/dialect.cpp:62, over NCCL on
NVLink). The residual adds ride in the row-parallel GEMMs' addend on rank 0
only, so after the sum they count once. Attention and RoPE are
`attn.prefill` / `attn.rope` (dialect.cpp:38-40) for equal-length sequences.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


class TPDecoderLayer:
    """Weights (bf16, this rank's shards, K-contiguous):
        wqkv [(hq + 2*hkv) * 128, H]  query heads, then key heads, then value heads
        wo   [H, hq * 128]
        w13  [2 * ffn_r, H]           gate/up packed by ops.pack_gate_up
        w2   [H, ffn_r]
        g1, g2 [H]                     RMSNorm gains
    """

    def __init__(self, wqkv, wo, w13, w2, g1, g2, *, batch: int, seq_len: int,
                 heads_q: int, heads_kv: int, rank: int = 0, world: int = 1, group=None,
                 eps: float = 1e-5, rope_base: float = 10000.0):
        if heads_q % world or heads_kv % world:
            raise ValueError("heads must divide over the ranks")
        self.B, self.L = batch, seq_len
        self.hq, self.hkv = heads_q // world, heads_kv // world
        self.rank, self.world, self.group = rank, world, group
        self.eps, self.base = eps, rope_base
        self.wqkv, self.wo, self.w13, self.w2, self.g1, self.g2 = wqkv, wo, w13, w2, g1, g2
        H = wo.shape[0]
        self.H = H
        T = batch * seq_len
        dev = wqkv.device
        bf = torch.bfloat16
        self.xn = torch.empty((T, H), dtype=bf, device=dev)
        self.qkv = torch.empty((T, wqkv.shape[0]), dtype=bf, device=dev)
        self.attn = torch.empty((T, self.hq * 128), dtype=bf, device=dev)
        self.h1 = torch.empty((T, H), dtype=bf, device=dev)
        self.h1n = torch.empty((T, H), dtype=bf, device=dev)
        self.act = torch.empty((T, w13.shape[0] // 2), dtype=bf, device=dev)
        self.out = torch.empty((T, H), dtype=bf, device=dev)
        from ._lib import lib
        ws = int(lib().kvm_sm100_attention_workspace(batch, seq_len, self.hq, self.hkv))
        self.ws = torch.empty(ws, dtype=torch.uint8, device=dev)

    @classmethod
    def from_full(cls, wq, wk, wv, wo, wg, wu, w2, g1, g2, *, batch, seq_len, heads_q,
                  heads_kv, rank=0, world=1, group=None):
        """Shard full weights given K-contiguous: wq [HQ*128, H], wk/wv
        [HKV*128, H], wo [H, HQ*128], wg/wu [FFN, H], w2 [H, FFN]."""
        hq, hkv = heads_q // world, heads_kv // world
        F = wg.shape[0] // world
        qs = slice(rank * hq * 128, (rank + 1) * hq * 128)
        ks = slice(rank * hkv * 128, (rank + 1) * hkv * 128)
        fs = slice(rank * F, (rank + 1) * F)
        wqkv = torch.cat([wq[qs], wk[ks], wv[ks]]).contiguous()
        w13 = ops.pack_gate_up(wg[fs].contiguous(), wu[fs].contiguous(), layout="nk")
        return cls(wqkv, wo[:, qs].contiguous(), w13, w2[:, fs].contiguous(), g1, g2,
                   batch=batch, seq_len=seq_len, heads_q=heads_q, heads_kv=heads_kv,
                   rank=rank, world=world, group=group)

    # kernels of our own per call: 2 RMSNorm, 4 GEMM, 2 RoPE, 1 fused attention
    def launches(self) -> int:
        return 9

    def __call__(self, x: torch.Tensor, probe=None) -> torch.Tensor:
        hq, hkv, L = self.hq, self.hkv, self.L
        ops.rmsnorm(x, self.g1, self.eps, out=self.xn)
        ops.matmul(self.xn, self.wqkv, b_layout="nk", out=self.qkv)
        q = self.qkv[:, :hq * 128]
        k = self.qkv[:, hq * 128:(hq + hkv) * 128]
        v = self.qkv[:, (hq + hkv) * 128:]
        ops.rope_(q, seq_len=L, heads=hq, base=self.base)
        ops.rope_(k, seq_len=L, heads=hkv, base=self.base)
        if probe is not None:
            probe[0].record()
        ops.attention_prefill(q, k, v, batch=self.B, heads_q=hq, heads_kv=hkv,
                              out=self.attn, workspace=self.ws)
        if probe is not None:
            probe[1].record()
        ops.matmul(self.attn, self.wo, b_layout="nk", c=x if self.rank == 0 else None,
                   out=self.h1)
        if self.world > 1:
            dist.all_reduce(self.h1, group=self.group)
        ops.rmsnorm(self.h1, self.g2, self.eps, out=self.h1n)
        ops.silu_gate_matmul(self.h1n, self.w13, out=self.act)
        ops.matmul(self.act, self.w2, b_layout="nk", c=self.h1 if self.rank == 0 else None,
                   out=self.out)
        if self.world > 1:
            dist.all_reduce(self.out, group=self.group)
        return self.out
