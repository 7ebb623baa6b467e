"""The MoE layer of a kernel-dialect graph executed on one GPU:

    comm.moe_dispatch(x, g)  ->  route (router GEMM + softmax + top-k),
                                 permute (expert-major order), scatter rows
    kernel.gemm on 3-D expert weights
                             ->  grouped GEMM gate/up with fused SiLU-gate,
                                 grouped GEMM down
    comm.moe_combine(y, g)   ->  weighted combine

(reference ops: src/ir/dialect/kernel/dialect.cpp:35,65-66; the pass-through
lowering of dispatch/combine is src/device/device.cpp:143-147.)

All buffers are allocated once, at construction, for ``max_tokens``; a call
launches seven or eight kernels (LAUNCHES_PER_CALL) on the current stream and
allocates nothing, so the call can be captured in a CUDA graph.
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import call, lib


def permute_launches(n_pairs: int, E: int) -> int:
    """Kernels kvm_sm100_moe_permute launches for n_pairs (token, expert)
    pairs: a count pass and a rank pass that also forms the offsets when the
    per-block count matrix (ceil(n_pairs / 256) x E) has at most 16384
    entries, else count, scan and rank."""
    blocks = (n_pairs + 255) // 256
    return 2 if blocks * E <= 16 * 1024 else 3


def _out_buffer(out, own, T, H):
    if out is None:
        return own
    if (out.dtype != torch.bfloat16 or not out.is_cuda or not out.is_contiguous()
            or out.dim() != 2 or out.shape[0] < T or out.shape[1] != H):
        raise ValueError(f"out must be a contiguous bf16 CUDA tensor [>= {T}, {H}]")
    return out


class MoELayer:
    """Top-k MoE layer with gated (SiLU) experts: H -> F -> H per expert.

    Weights (bf16, device):
      w_router [E, H]      one row per expert
      w13      [E, 2F, H]  gate/up packed by ops.pack_gate_up
      w2       [E, H, F]   down projection, one [H, F] matrix per expert
    """

    def __init__(self, w_router: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor,
                 top_k: int, max_tokens: int):
        E, H = w_router.shape
        F = w13.shape[1] // 2
        if w13.shape != (E, 2 * F, H) or w2.shape != (E, H, F):
            raise ValueError("expected w13 [E, 2F, H] and w2 [E, H, F]")
        for t, n in ((w_router, "w_router"), (w13, "w13"), (w2, "w2")):
            if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{n} must be a contiguous bf16 CUDA tensor")
        self.E, self.H, self.F, self.k = E, H, F, top_k
        self.max_tokens = max_tokens
        self.w_router, self.w13, self.w2 = w_router, w13, w2
        dev = w_router.device
        T, k = max_tokens, top_k
        self.logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        self.topk_idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        self.topk_w = torch.empty((T, k), dtype=torch.float32, device=dev)
        self.offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        self.pos = torch.empty(T * k, dtype=torch.int32, device=dev)
        self.src_token = torch.empty(T * k, dtype=torch.int32, device=dev)
        ws = int(lib().kvm_sm100_moe_permute_workspace(T, k, E))
        self.workspace = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        self.xp = torch.empty((T * k, H), dtype=torch.bfloat16, device=dev)
        self.h = torch.empty((T * k, F), dtype=torch.bfloat16, device=dev)
        self.y = torch.empty((T * k, H), dtype=torch.bfloat16, device=dev)
        self.out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)

    @classmethod
    def from_packed(cls, w_router, w13, w2, *, top_k: int, max_tokens: int) -> "MoELayer":
        return cls(w_router, w13, w2, top_k, max_tokens)

    @classmethod
    def from_graph_weights(cls, w_router_hk: torch.Tensor, w1: torch.Tensor,
                           w3: torch.Tensor, w2: torch.Tensor, *, top_k: int,
                           max_tokens: int) -> "MoELayer":
        """Weights in the graph's kernel.matmul layout: router [H, E],
        w1/w3 [E, H, F] (gate/up), w2 [E, F, H]; re-laid out once on the GPU."""
        wr = ops.transpose(w_router_hk)
        w13 = ops.pack_gate_up(w1, w3, layout="kn")
        w2t = ops.transpose(w2)
        return cls(wr, w13, w2t, top_k, max_tokens)

    @property
    def last_routing(self) -> ops.Routing:
        n = self._n
        return ops.Routing(self.logits[:n], self.topk_idx[:n], self.topk_w[:n])

    @property
    def last_dispatch(self) -> ops.Dispatch:
        n = self._n * self.k
        return ops.Dispatch(self.offsets, self.pos[:n], self.src_token[:n])

    # phase marks of a call (kvm_b200.timing.PhaseProbe): one per launch
    PHASES = ["start", "router", "permute", "scatter", "gate_up", "down", "combine"]

    def __call__(self, x: torch.Tensor, probe=None, out: torch.Tensor | None = None
                 ) -> torch.Tensor:
        """Run the layer on x [T, H]; `probe` (a kvm_b200.timing.PhaseProbe
        over PHASES) records a CUDA event before the first launch and after
        each launch, for per-kernel timing; `out` (contiguous bf16 [>= T, H])
        receives the result instead of the layer's own buffer."""
        mark = probe.mark if probe is not None else (lambda name: None)
        T, H = x.shape
        if H != self.H or T > self.max_tokens or T <= 0:
            raise ValueError(f"x must be [T<= {self.max_tokens}, {self.H}]")
        if x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous():
            raise ValueError("x must be a contiguous bf16 CUDA tensor")
        self._n = T
        st = torch.cuda.current_stream().cuda_stream
        E, F, k = self.E, self.F, self.k
        dst = _out_buffer(out, self.out, T, H)
        mark("start")
        call("kvm_sm100_moe_router_topk", x.data_ptr(), self.w_router.data_ptr(),
             self.logits.data_ptr(), self.topk_idx.data_ptr(), self.topk_w.data_ptr(),
             T, H, E, k, st)
        mark("router")
        call("kvm_sm100_moe_permute", self.topk_idx.data_ptr(), T, k, E,
             self.offsets.data_ptr(), self.pos.data_ptr(), self.src_token.data_ptr(),
             self.workspace.data_ptr(), st)
        mark("permute")
        call("kvm_sm100_moe_scatter_rows", x.data_ptr(), self.pos.data_ptr(),
             self.xp.data_ptr(), T, k, H, st)
        mark("scatter")
        call("kvm_sm100_grouped_gemm_bf16", self.xp.data_ptr(), self.w13.data_ptr(),
             self.h.data_ptr(), self.offsets.data_ptr(), E, T * k, 2 * F, H, 2, st)
        mark("gate_up")
        call("kvm_sm100_grouped_gemm_bf16", self.h.data_ptr(), self.w2.data_ptr(),
             self.y.data_ptr(), self.offsets.data_ptr(), E, T * k, H, F, 0, st)
        mark("down")
        call("kvm_sm100_moe_combine", self.y.data_ptr(), self.pos.data_ptr(),
             self.topk_w.data_ptr(), dst.data_ptr(), T, k, H, st)
        mark("combine")
        return dst[:T]

    @property
    def LAUNCHES_PER_CALL(self) -> int:
        """Kernels one call on max_tokens tokens launches: router 1, permute
        2 or 3, scatter 1, grouped GEMMs 2, combine 1."""
        return 5 + permute_launches(self.max_tokens * self.k, self.E)
