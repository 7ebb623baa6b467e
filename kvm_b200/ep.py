"""Expert-parallel MoE layer: experts sharded over the ranks of a process
group. Two exchanges are provided: ExpertParallelMoE (peer memory over NVLink,
no host synchronisation, the production path) and ExpertParallelMoENccl
(torch.distributed point-to-point messages; runs on gloo too, so its exchange
logic is tested on CPU ranks).

This executes `kernel.comm.moe_dispatch` / `kernel.comm.moe_combine` with
their `ranks` operand (src/ir/dialect/kernel/ops.h:87-88, carried onto the
task ops by src/device/device.cpp:108-121) when the ranks span several GPUs.

Rank r owns experts [r*E/P, (r+1)*E/P). One forward:

  1. route + permute + scatter the rank's own tokens (local kernels); the
     permuted rows are expert-major, hence destination-rank-major;
  2. exchange per-expert row counts (all_to_all of int32 [P, E/P]);
  3. one device->host copy of the counts and offsets; the host plans one
     message per (peer, expert) pair with rows, so every rank receives its
     rows already expert-major (grouped by local expert, then by source rank);
  4. dispatch: batched isend/irecv of those messages (local pairs are
     device copies);
  5. grouped gate/up GEMM with fused SiLU-gate, grouped down GEMM over the
     local experts;
  6. combine exchange: the reverse messages return each expert output row to
     the rank that owns the token, at the row its local permutation gave it;
  7. weighted combine (local kernel).

Every rank issues the same collectives in the same order; messages between
a pair are issued in ascending expert order on both sides.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class Plan:
    """Message plan of one forward (host-side, all sizes in rows)."""
    send: list      # (peer, src_row, n_rows) from the permuted send buffer
    recv: list      # (peer, dst_row, n_rows) into the expert-major receive buffer
    local_offsets: list  # [E/P + 1] row offsets of the local experts
    recv_rows: int


def make_plan(rank: int, world: int, experts: int, send_offsets, recv_counts) -> Plan:
    """Pure host logic (tested on CPU).

    send_offsets: [E+1] offsets of this rank's permuted rows by global expert.
    recv_counts:  [P * E/P]; recv_counts[s*Epr + e] = rows rank s sends for
                  local expert e.
    Messages to/from one peer are listed in ascending local-expert order.
    """
    epr = experts // world
    send, recv = [], []
    for d in range(world):
        for e in range(epr):
            g = d * epr + e
            n = int(send_offsets[g + 1] - send_offsets[g])
            if n:
                send.append((d, int(send_offsets[g]), n))
    local = [0]
    for e in range(epr):
        local.append(local[-1] + sum(int(recv_counts[s * epr + e]) for s in range(world)))
    for e in range(epr):
        row = local[e]
        for s in range(world):
            n = int(recv_counts[s * epr + e])
            if n:
                recv.append((s, row, n))
                row += n
    return Plan(send, recv, local, local[-1])


class CudaCompute:
    """Local compute of one rank on the sm_100a kernels."""

    @property
    def LAUNCHES(self) -> int:
        """Kernels per call on max_tokens tokens: router 1, permute 2 or 3,
        scatter 1, grouped GEMMs 2, combine 1."""
        from .moe import permute_launches
        return 5 + permute_launches(self.max_tokens * self.k, self.E)

    def __init__(self, w_router, w13_local, w2_local, top_k, max_tokens, world):
        from ._lib import lib
        self.wr, self.w13, self.w2 = w_router, w13_local, w2_local
        self.E, self.H = w_router.shape
        self.F = w13_local.shape[1] // 2
        self.k = top_k
        self.max_tokens = max_tokens
        dev = w_router.device
        T, k, E, H, F = max_tokens, top_k, self.E, self.H, self.F
        self.logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        self.idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        self.topw = torch.empty((T, k), dtype=torch.float32, device=dev)
        self.offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        self.pos = torch.empty(T * k, dtype=torch.int32, device=dev)
        self.src = torch.empty(T * k, dtype=torch.int32, device=dev)
        ws = int(lib().kvm_sm100_moe_permute_workspace(T, k, E))
        self.ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        self.xp = torch.empty((T * k, H), dtype=torch.bfloat16, device=dev)
        cap = T * k * world            # every row of every rank on this rank
        self.recv = torch.empty((cap, H), dtype=torch.bfloat16, device=dev)
        self.h = torch.empty((cap, F), dtype=torch.bfloat16, device=dev)
        self.y = torch.empty((cap, H), dtype=torch.bfloat16, device=dev)
        self.yback = torch.empty((T * k, H), dtype=torch.bfloat16, device=dev)
        self.out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        self.loc_off = torch.empty(w13_local.shape[0] + 1, dtype=torch.int32, device=dev)
        self.loc_off_host = torch.empty(w13_local.shape[0] + 1, dtype=torch.int32).pin_memory()

    def dispatch_local(self, x):
        from ._lib import call
        T, H = x.shape
        st = torch.cuda.current_stream().cuda_stream
        E, k = self.E, self.k
        call("kvm_sm100_moe_router_topk", x.data_ptr(), self.wr.data_ptr(),
             self.logits.data_ptr(), self.idx.data_ptr(), self.topw.data_ptr(),
             T, H, E, k, st)
        call("kvm_sm100_moe_permute", self.idx.data_ptr(), T, k, E, self.offsets.data_ptr(),
             self.pos.data_ptr(), self.src.data_ptr(), self.ws.data_ptr(), st)
        call("kvm_sm100_moe_scatter_rows", x.data_ptr(), self.pos.data_ptr(),
             self.xp.data_ptr(), T, k, H, st)
        return self.xp, self.offsets

    def experts(self, rows: int, local_offsets: list):
        from ._lib import call
        n = len(local_offsets)
        self.loc_off_host[:n] = torch.tensor(local_offsets, dtype=torch.int32)
        self.loc_off[:n].copy_(self.loc_off_host[:n], non_blocking=True)
        if rows == 0:
            return self.y
        st = torch.cuda.current_stream().cuda_stream
        G, H, F = n - 1, self.H, self.F
        call("kvm_sm100_grouped_gemm_bf16", self.recv.data_ptr(), self.w13.data_ptr(),
             self.h.data_ptr(), self.loc_off.data_ptr(), G, rows, 2 * F, H, 2, st)
        call("kvm_sm100_grouped_gemm_bf16", self.h.data_ptr(), self.w2.data_ptr(),
             self.y.data_ptr(), self.loc_off.data_ptr(), G, rows, H, F, 0, st)
        return self.y

    def combine_local(self, T):
        from ._lib import call
        st = torch.cuda.current_stream().cuda_stream
        call("kvm_sm100_moe_combine", self.yback.data_ptr(), self.pos.data_ptr(),
             self.topw.data_ptr(), self.out.data_ptr(), T, self.k, self.H, st)
        return self.out[:T]


class ExpertParallelMoENccl:
    """MoE layer with E/P experts per rank over torch.distributed point-to-point
    messages (NCCL on GPUs, gloo on CPU). The host plans the messages from the
    exchanged counts, which costs one device->host synchronisation per call;
    ExpertParallelMoE below is the synchronisation-free NVLink path. `w13`/`w2`
    may be the full [E, ...] weights (this rank's slice is taken) or already the
    local [E/P, ...] slice."""

    def __init__(self, w_router, w13, w2, *, top_k: int, max_tokens: int, rank: int,
                 world: int, group=None, compute=None):
        E = w_router.shape[0]
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        self.E, self.world, self.rank, self.k = E, world, rank, top_k
        self.epr = E // world
        self.group = group
        e0 = rank * self.epr
        if w13.shape[0] == E:
            w13 = w13[e0:e0 + self.epr].contiguous()
            w2 = w2[e0:e0 + self.epr].contiguous()
        self.w_router, self.w13, self.w2 = w_router, w13, w2
        self.compute = compute or CudaCompute(w_router, w13, w2, top_k, max_tokens, world)
        self.LAUNCHES_PER_CALL = getattr(self.compute, "LAUNCHES", 0)
        dev = w_router.device
        self._send_counts = torch.empty(E, dtype=torch.int32, device=dev)
        self._recv_counts = torch.empty(E, dtype=torch.int32, device=dev)
        self.last_plan: Plan | None = None

    def _exchange(self, src_buf, dst_buf, sends, recvs):
        """Run one batch of messages; rows to/from this rank are local copies."""
        ops = []
        local_src = [(s, n) for (p, s, n) in sends if p == self.rank]
        local_dst = [(d, n) for (p, d, n) in recvs if p == self.rank]
        for (s, n), (d, n2) in zip(local_src, local_dst):
            assert n == n2
            dst_buf[d:d + n].copy_(src_buf[s:s + n])
        for (p, s, n) in sends:
            if p != self.rank:
                ops.append(dist.P2POp(dist.isend, src_buf[s:s + n], self._g(p), self.group))
        for (p, d, n) in recvs:
            if p != self.rank:
                ops.append(dist.P2POp(dist.irecv, dst_buf[d:d + n], self._g(p), self.group))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()

    def _g(self, r: int) -> int:
        return r if self.group is None else dist.get_global_rank(self.group, r)

    def __call__(self, x):
        T = x.shape[0]
        c = self.compute
        xp, offsets = c.dispatch_local(x)
        # per-expert counts of this rank's rows, grouped by destination rank
        torch.sub(offsets[1:], offsets[:-1], out=self._send_counts)
        dist.all_to_all_single(self._recv_counts, self._send_counts, group=self.group)
        both = torch.cat([offsets, self._recv_counts]).cpu()   # the one host sync
        plan = make_plan(self.rank, self.world, self.E, both[: self.E + 1].tolist(),
                         both[self.E + 1:].tolist())
        self.last_plan = plan
        self._exchange(xp, c.recv, plan.send, plan.recv)
        y = c.experts(plan.recv_rows, plan.local_offsets)
        # reverse: what was received from (peer, row) goes back to (peer, row)
        self._exchange(y, c.yback, plan.recv, plan.send)
        return c.combine_local(T)


class ExpertParallelMoE:
    """Expert-parallel MoE layer over NVLink peer memory (one process per GPU).

    Buffers that peers touch (receive rows, expert outputs, count matrix,
    flags) are allocated with kvm_sm100_ipc_alloc and mapped into every rank
    through CUDA IPC handles exchanged over the process group once, at
    construction. A call never synchronises with the host. Weak scaling: each
    rank brings `max_tokens` tokens at most.

    overlap=True (default): the all-to-all rides inside the grouped GEMMs --
    route, permute, prepare (count exchange), local scatter, dispatch fused
    with the gate/up GEMM (peer stores by extra warps; a local expert's tiles
    start once every rank's rows for it have arrived), down GEMM whose
    epilogue stores each result row straight back to the rank that routed the
    token, wait for every rank's outputs, local combine: 9 or 10 launches.
    overlap=False: the serial exchange -- route, permute, count exchange,
    dispatch (peer stores), wait, grouped GEMMs, signal, wait, combine (peer
    loads): 11 or 12 launches. Both are bit-identical to the one-GPU layer.
    """

    @property
    def LAUNCHES_PER_CALL(self) -> int:
        """route 1, permute 2 or 3, then 6 (overlapped: prepare, local
        scatter, dispatch + gate/up, down + push, wait, combine) or 8 (serial:
        count exchange, dispatch, wait, grouped GEMMs 2, signal, wait,
        combine)."""
        from .moe import permute_launches
        return (7 if self.overlap else 9) + permute_launches(self.max_tokens * self.k, self.E)

    def __init__(self, w_router, w13, w2, *, top_k: int, max_tokens: int, rank: int,
                 world: int, group=None, overlap: bool = True):
        import ctypes as C
        from ._lib import EpPeers, call, lib
        E, H = w_router.shape
        if E % world or world > 8:
            raise ValueError(f"{E} experts over {world} ranks (at most 8)")
        self.E, self.H, self.k, self.rank, self.world = E, H, top_k, rank, world
        self.epr = E // world
        e0 = rank * self.epr
        if w13.shape[0] == E:
            w13 = w13[e0:e0 + self.epr].contiguous()
            w2 = w2[e0:e0 + self.epr].contiguous()
        self.w_router, self.w13, self.w2 = w_router, w13, w2
        self.F = w13.shape[1] // 2
        self.group = group
        dev = w_router.device
        T, k = max_tokens, top_k
        self.max_tokens = T
        self.cap = T * k * world
        i32 = torch.int32
        self.logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        self.idx = torch.empty((T, k), dtype=i32, device=dev)
        self.topw = torch.empty((T, k), dtype=torch.float32, device=dev)
        self.offsets = torch.empty(E + 1, dtype=i32, device=dev)
        self.pos = torch.empty(T * k, dtype=i32, device=dev)
        self.src = torch.empty(T * k, dtype=i32, device=dev)
        ws = int(lib().kvm_sm100_moe_permute_workspace(T, k, E))
        self.ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        self.send_base = torch.empty(E, dtype=i32, device=dev)
        self.loc_off = torch.empty(self.epr + 1, dtype=i32, device=dev)
        self.done = torch.zeros(1, dtype=i32, device=dev)
        self.h = torch.empty((self.cap, self.F), dtype=torch.bfloat16, device=dev)
        self.out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        self.overlap = overlap
        self.PHASES = self.PHASES_OVERLAP if overlap else self.PHASES_SERIAL
        wsb = int(lib().kvm_sm100_ep_overlap_workspace(E, self.cap))
        self.ws_ep = torch.empty(max(wsb, 256), dtype=torch.uint8, device=dev)
        # flag words: counts, data, outputs ([world] each), then one per
        # (local expert, source rank)
        sizes = {"recv": self.cap * H * 2, "y": self.cap * H * 2,
                 "cnt": world * E * 4, "flags": (3 * world + self.epr * world) * 4}
        self._own = {}
        for name, nbytes in sizes.items():
            p = C.c_void_p()
            call("kvm_sm100_ipc_alloc", nbytes, C.byref(p))
            self._own[name] = p.value
        handles = {}
        for name, p in self._own.items():
            buf = C.create_string_buffer(64)
            call("kvm_sm100_ipc_get_handle", p, buf)
            handles[name] = buf.raw
        gathered = [None] * world
        if world > 1:
            dist.all_gather_object(gathered, handles, group=group)
        else:
            gathered = [handles]
        self._opened = []
        peers = EpPeers()
        peers.rank, peers.world, peers.E, peers.H, peers.k = rank, world, E, H, k
        for r in range(world):
            for name in sizes:
                if r == rank:
                    ptr = self._own[name]
                else:
                    q = C.c_void_p()
                    call("kvm_sm100_ipc_open_handle", C.create_string_buffer(
                        gathered[r][name], 64), C.byref(q))
                    ptr = q.value
                    self._opened.append(ptr)
                getattr(peers, name)[r] = ptr
        self.peers = peers
        self._peers_ref = C.byref(peers)
        self.epoch = 0
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(group=group)

    # phase marks of a call (kvm_b200.timing.PhaseProbe): one per launch
    PHASES_SERIAL = ["start", "router", "permute", "ep_counts", "ep_dispatch",
                     "ep_wait_data", "gate_up", "down", "ep_signal", "ep_wait_outputs",
                     "ep_combine"]
    PHASES_OVERLAP = ["start", "router", "permute", "ep_prepare", "ep_scatter_local",
                      "ep_dispatch_gate_up", "ep_down_push", "ep_wait_outputs", "combine"]

    def __call__(self, x, probe=None, out=None):
        from ._lib import call
        from .moe import _out_buffer
        mark = probe.mark if probe is not None else (lambda name: None)
        T, H = x.shape
        if H != self.H or T > self.max_tokens or T <= 0:
            raise ValueError(f"x must be [T <= {self.max_tokens}, {self.H}]")
        if x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous():
            raise ValueError("x must be a contiguous bf16 CUDA tensor")
        dst = _out_buffer(out, self.out, T, H)
        self.epoch += 1
        ep, pr = self.epoch, self._peers_ref
        st = torch.cuda.current_stream().cuda_stream
        E, k, F = self.E, self.k, self.F
        mark("start")
        call("kvm_sm100_moe_router_topk", x.data_ptr(), self.w_router.data_ptr(),
             self.logits.data_ptr(), self.idx.data_ptr(), self.topw.data_ptr(),
             T, H, E, k, st)
        mark("router")
        call("kvm_sm100_moe_permute", self.idx.data_ptr(), T, k, E, self.offsets.data_ptr(),
             self.pos.data_ptr(), self.src.data_ptr(), self.ws.data_ptr(), st)
        mark("permute")
        if self.overlap:
            return self._overlapped(x, dst, ep, pr, st, mark)
        call("kvm_sm100_ep_counts", pr, self.offsets.data_ptr(), self.send_base.data_ptr(),
             self.loc_off.data_ptr(), ep, st)
        mark("ep_counts")
        call("kvm_sm100_ep_dispatch", pr, x.data_ptr(), self.idx.data_ptr(),
             self.pos.data_ptr(), self.offsets.data_ptr(), self.send_base.data_ptr(), T,
             self.cap, self.done.data_ptr(), ep, st)
        mark("ep_dispatch")
        call("kvm_sm100_ep_wait", pr, 1, ep, st)
        mark("ep_wait_data")
        recv, y = self._own["recv"], self._own["y"]
        call("kvm_sm100_grouped_gemm_bf16", recv, self.w13.data_ptr(), self.h.data_ptr(),
             self.loc_off.data_ptr(), self.epr, self.cap, 2 * F, H, 2, st)
        mark("gate_up")
        call("kvm_sm100_grouped_gemm_bf16", self.h.data_ptr(), self.w2.data_ptr(), y,
             self.loc_off.data_ptr(), self.epr, self.cap, H, F, 0, st)
        mark("down")
        call("kvm_sm100_ep_signal", pr, 2, ep, st)
        mark("ep_signal")
        call("kvm_sm100_ep_wait", pr, 2, ep, st)
        mark("ep_wait_outputs")
        call("kvm_sm100_ep_combine", pr, self.idx.data_ptr(), self.pos.data_ptr(),
             self.offsets.data_ptr(), self.send_base.data_ptr(), self.topw.data_ptr(),
             dst.data_ptr(), T, self.cap, st)
        mark("ep_combine")
        return dst[:T]

    def _overlapped(self, x, dst, ep, pr, st, mark):
        from ._lib import call
        T = x.shape[0]
        H, F, k = self.H, self.F, self.k
        ws = self.ws_ep.data_ptr()
        call("kvm_sm100_ep_prepare", pr, self.offsets.data_ptr(), self.send_base.data_ptr(),
             self.loc_off.data_ptr(), ws, self.cap, ep, st)
        mark("ep_prepare")
        call("kvm_sm100_ep_scatter_local", pr, x.data_ptr(), self.src.data_ptr(),
             self.offsets.data_ptr(), self.send_base.data_ptr(), T, self.cap, st)
        mark("ep_scatter_local")
        call("kvm_sm100_ep_dispatch_gate_up", pr, x.data_ptr(), self.src.data_ptr(),
             self.offsets.data_ptr(), self.send_base.data_ptr(), self.loc_off.data_ptr(),
             self.w13.data_ptr(), self.h.data_ptr(), F, self.cap, ws, ep, st)
        mark("ep_dispatch_gate_up")
        call("kvm_sm100_ep_down_push", pr, self.h.data_ptr(), self.w2.data_ptr(),
             self.loc_off.data_ptr(), F, self.cap, ws, ep, st)
        mark("ep_down_push")
        call("kvm_sm100_ep_wait", pr, 2, ep, st)
        mark("ep_wait_outputs")
        call("kvm_sm100_moe_combine", self._own["y"], self.pos.data_ptr(),
             self.topw.data_ptr(), dst.data_ptr(), T, k, H, st)
        mark("combine")
        return dst[:T]

    def close(self):
        """Unmap peer buffers and free this rank's (collective: all ranks call it)."""
        from ._lib import call
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        for p in self._opened:
            call("kvm_sm100_ipc_close", p)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)
        for p in self._own.values():
            call("kvm_sm100_ipc_free", p)
        self._own = {}
