"""Torch-facing wrappers over the C ABI (include/kvm_sm100.h).

Torch supplies device memory and the current CUDA stream; every computation
runs in libkvm_sm100.so. Each wrapper checks device, dtype and contiguity and
raises on a bad argument or a non-zero kvm_status; nothing falls back to a
torch or CPU implementation.

Op semantics follow the kernel-dialect ops of the reference
(src/ir/dialect/kernel/dialect.cpp:33-70) as defined for execution in
include/kvm_sm100.h.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import KVM_B_KN, KVM_B_NK, KVM_BF16, KVM_F32, call


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check(t: torch.Tensor, name: str, dtype: torch.dtype, ndim: int | None = None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path exists)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")


def _rowmajor(t: torch.Tensor, name: str) -> int:
    """Row stride of a 2-D tensor whose rows are contiguous."""
    if t.stride(1) != 1:
        raise ValueError(f"{name} must have contiguous rows")
    return t.stride(0)


# ----------------------------------------------------------------- GEMM ---

def matmul(a: torch.Tensor, b: torch.Tensor, *, b_layout: str = "kn",
           c: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """D = A . B (+ C): kernel.matmul / kernel.gemm on the tcgen05 GEMM.

    a: bf16 [M, K]. b: bf16 [K, N] (b_layout="kn", kernel.matmul's layout) or
    [N, K] (b_layout="nk"). c: optional addend [M, N] of out_dtype.
    fp32 accumulation; output bf16 (RNE) or fp32.
    """
    _check(a, "a", torch.bfloat16, 2)
    _check(b, "b", torch.bfloat16, 2)
    M, K = a.shape
    if b_layout == "kn":
        if b.shape[0] != K:
            raise ValueError(f"b {tuple(b.shape)} does not match a {tuple(a.shape)}")
        N, lay = b.shape[1], KVM_B_KN
    elif b_layout == "nk":
        if b.shape[1] != K:
            raise ValueError(f"b {tuple(b.shape)} does not match a {tuple(a.shape)}")
        N, lay = b.shape[0], KVM_B_NK
    else:
        raise ValueError("b_layout must be 'kn' or 'nk'")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("out_dtype must be bf16 or fp32")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    _check(out, "out", out_dtype, 2)
    if c is not None:
        _check(c, "c", out_dtype, 2)
        if c.shape != out.shape or c.stride() != out.stride():
            raise ValueError("c must match out in shape and strides")
    call("kvm_sm100_gemm_bf16", a.data_ptr(), _rowmajor(a, "a"), b.data_ptr(),
         _rowmajor(b, "b"), lay, _ptr(c), out.data_ptr(), _rowmajor(out, "out"),
         KVM_F32 if out_dtype == torch.float32 else KVM_BF16, M, N, K, _stream())
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, **kw) -> torch.Tensor:
    """kernel.gemm: D = A . B + C (src/ir/dialect/kernel/dialect.cpp:35)."""
    return matmul(a, b, c=c, out_dtype=c.dtype, **kw)


def pack_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, layout: str = "nk") -> torch.Tensor:
    """Interleave gate/up weights in 64-row blocks for the SiLU-gate GEMMs.

    layout "nk": inputs [G, F, K] (or [F, K]); "kn": inputs [G, K, F] (or [K, F]).
    Returns [G, 2F, K] (or [2F, K]).
    """
    _check(w_gate, "w_gate", torch.bfloat16)
    _check(w_up, "w_up", torch.bfloat16)
    if w_gate.shape != w_up.shape:
        raise ValueError("gate and up weights must have the same shape")
    squeeze = w_gate.dim() == 2
    wg = w_gate.unsqueeze(0) if squeeze else w_gate
    wu = w_up.unsqueeze(0) if squeeze else w_up
    wg, wu = wg.contiguous(), wu.contiguous()
    G = wg.shape[0]
    if layout == "nk":
        F, K, lay = wg.shape[1], wg.shape[2], KVM_B_NK
    elif layout == "kn":
        K, F, lay = wg.shape[1], wg.shape[2], KVM_B_KN
    else:
        raise ValueError("layout must be 'nk' or 'kn'")
    out = torch.empty((G, 2 * F, K), dtype=torch.bfloat16, device=wg.device)
    call("kvm_sm100_pack_gate_up", wg.data_ptr(), wu.data_ptr(), out.data_ptr(),
         G, F, K, lay, _stream())
    return out[0] if squeeze else out


def transpose(w: torch.Tensor) -> torch.Tensor:
    """[.., R, C] -> [.., C, R] for bf16 matrices (a one-time weight re-layout)."""
    _check(w, "w", torch.bfloat16)
    squeeze = w.dim() == 2
    x = (w.unsqueeze(0) if squeeze else w).contiguous()
    G, R, Cc = x.shape
    out = torch.empty((G, Cc, R), dtype=torch.bfloat16, device=x.device)
    call("kvm_sm100_transpose_bf16", x.data_ptr(), out.data_ptr(), G, R, Cc, _stream())
    return out[0] if squeeze else out


def silu_gate_matmul(a: torch.Tensor, w13: torch.Tensor,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """H = SiLU(A.Wg^T) * (A.Wu^T) with w13 from pack_gate_up(layout any)."""
    _check(a, "a", torch.bfloat16, 2)
    _check(w13, "w13", torch.bfloat16, 2)
    M, K = a.shape
    F = w13.shape[0] // 2
    if w13.shape[1] != K or not w13.is_contiguous():
        raise ValueError("w13 must be contiguous [2F, K]")
    if out is None:
        out = torch.empty((M, F), dtype=torch.bfloat16, device=a.device)
    call("kvm_sm100_gemm_bf16_silu_gate", a.data_ptr(), _rowmajor(a, "a"),
         w13.data_ptr(), out.data_ptr(), _rowmajor(out, "out"), M, F, K, _stream())
    return out


# -------------------------------------------------------------------- FP8 ---

def quantize_e4m3(x: torch.Tensor):
    """128x128 block quantisation: returns (q uint8 [R, C] e4m3 bits, scales fp32
    [ceil(R/128), ceil(C/128)]); s = amax/448, q = e4m3_rn_satfinite(x / s)."""
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("x must be bf16 or fp32")
    _check(x, "x", x.dtype, 2)
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    R, Cc = x.shape
    q = torch.empty((R, Cc), dtype=torch.uint8, device=x.device)
    s = torch.empty(((R + 127) // 128, (Cc + 127) // 128), dtype=torch.float32,
                    device=x.device)
    call("kvm_sm100_quantize_e4m3_block128", x.data_ptr(),
         KVM_F32 if x.dtype == torch.float32 else KVM_BF16, q.data_ptr(), s.data_ptr(),
         R, Cc, _stream())
    return q, s


def transpose_u8(x: torch.Tensor) -> torch.Tensor:
    _check(x, "x", torch.uint8, 2)
    x = x.contiguous()
    out = torch.empty((x.shape[1], x.shape[0]), dtype=torch.uint8, device=x.device)
    call("kvm_sm100_transpose_u8", x.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1],
         _stream())
    return out


def transpose_f32(x: torch.Tensor) -> torch.Tensor:
    _check(x, "x", torch.float32, 2)
    x = x.contiguous()
    out = torch.empty((x.shape[1], x.shape[0]), dtype=torch.float32, device=x.device)
    call("kvm_sm100_transpose_f32", x.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1],
         _stream())
    return out


def matmul_fp8(aq: torch.Tensor, sa: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor,
               out: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None) -> torch.Tensor:
    """D = sum_kb sA*sW * (Aq . Wq^T) over 128-deep blocks, bf16 out.

    aq: uint8 e4m3 [M, K]; sa fp32 [ceil(M/128), K/128]; wq: uint8 e4m3 [N, K];
    sw fp32 [N/128, K/128].
    """
    _check(aq, "aq", torch.uint8, 2)
    _check(wq, "wq", torch.uint8, 2)
    _check(sa, "sa", torch.float32, 2)
    _check(sw, "sw", torch.float32, 2)
    M, K = aq.shape
    N = wq.shape[0]
    if wq.shape[1] != K or sa.shape != ((M + 127) // 128, K // 128) or \
            sw.shape != (N // 128, K // 128):
        raise ValueError("fp8 operand / scale shapes disagree")
    for t, n in ((aq, "aq"), (wq, "wq"), (sa, "sa"), (sw, "sw")):
        if not t.is_contiguous():
            raise ValueError(f"{n} must be contiguous")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=aq.device)
    need = int(_lib.lib().kvm_sm100_gemm_fp8_workspace(M, N, K))
    if need and (workspace is None or workspace.numel() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=aq.device)
    call("kvm_sm100_gemm_fp8_blockscaled", aq.data_ptr(), sa.data_ptr(), wq.data_ptr(),
         sw.data_ptr(), out.data_ptr(), _rowmajor(out, "out"), M, N, K,
         _ptr(workspace) if need else None, need, _stream())
    return out


# -------------------------------------------------------------- attention ---

def attention_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, batch: int,
                      heads_q: int, heads_kv: int, scale: float = 0.0,
                      out: torch.Tensor | None = None,
                      workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Causal GQA attention; q [B*L, HQ*128], k/v [B*L, HKV*128] (row views ok)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check(t, n, torch.bfloat16, 2)
    rows = q.shape[0]
    L = rows // batch
    if out is None:
        out = torch.empty((rows, heads_q * 128), dtype=torch.bfloat16, device=q.device)
    need = int(_lib.lib().kvm_sm100_attention_workspace(batch, L, heads_q, heads_kv))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    call("kvm_sm100_attention_prefill_bf16", q.data_ptr(), _rowmajor(q, "q"), k.data_ptr(),
         _rowmajor(k, "k"), v.data_ptr(), _rowmajor(v, "v"), out.data_ptr(),
         _rowmajor(out, "out"), batch, L, heads_q, heads_kv, 128, float(scale),
         workspace.data_ptr(), workspace.numel(), _stream())
    return out


def rope_(x: torch.Tensor, *, seq_len: int, heads: int, head_dim: int = 128,
          base: float = 10000.0) -> torch.Tensor:
    """In-place rotary embedding of x [B*L, >= heads*head_dim] (a row view is ok)."""
    _check(x, "x", torch.bfloat16, 2)
    call("kvm_sm100_rope_bf16", x.data_ptr(), _rowmajor(x, "x"), x.shape[0], seq_len, heads,
         head_dim, float(base), _stream())
    return x


# ------------------------------------------------------------ elementwise ---

def rmsnorm(x: torch.Tensor, gamma: torch.Tensor | None = None, eps: float = 1e-5,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2) + eps) * gamma over the last dim (bf16 in/out)."""
    _check(x, "x", torch.bfloat16)
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    H = x.shape[-1]
    rows = x.numel() // H
    if gamma is not None:
        _check(gamma, "gamma", torch.bfloat16, 1)
        if gamma.shape[0] != H or not gamma.is_contiguous():
            raise ValueError("gamma must be contiguous [H]")
    if out is None:
        out = torch.empty_like(x)
    call("kvm_sm100_rmsnorm_bf16", x.data_ptr(), _ptr(gamma), out.data_ptr(),
         rows, H, float(eps), _stream())
    return out


def silu_mul(g: torch.Tensor, u: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """h = g * sigmoid(g) * u elementwise (bf16)."""
    _check(g, "g", torch.bfloat16)
    _check(u, "u", torch.bfloat16)
    if g.shape != u.shape or not g.is_contiguous() or not u.is_contiguous():
        raise ValueError("g and u must be contiguous with equal shapes")
    if out is None:
        out = torch.empty_like(g)
    call("kvm_sm100_silu_mul_bf16", g.data_ptr(), u.data_ptr(), out.data_ptr(),
         g.numel(), _stream())
    return out


# -------------------------------------------------------------------- MoE ---

@dataclass
class Routing:
    """Output of moe_route: router logits and the chosen experts per token."""
    logits: torch.Tensor    # fp32 [T, E]
    topk_idx: torch.Tensor  # int32 [T, k]
    topk_w: torch.Tensor    # fp32 [T, k] softmax probabilities (not renormalised)


@dataclass
class Dispatch:
    """Expert-major permutation of the (token, slot) pairs."""
    offsets: torch.Tensor    # int32 [E+1]
    pos: torch.Tensor        # int32 [T*k]: permuted row of pair (t, j)
    src_token: torch.Tensor  # int32 [T*k]: token of each permuted row


def moe_route(x: torch.Tensor, w_router: torch.Tensor, top_k: int = 2) -> Routing:
    """Router GEMM + softmax + top-k (the routing half of comm.moe_dispatch).

    x: bf16 [T, H]; w_router: bf16 [E, H] (one row per expert).
    """
    _check(x, "x", torch.bfloat16, 2)
    _check(w_router, "w_router", torch.bfloat16, 2)
    T, H = x.shape
    E = w_router.shape[0]
    if w_router.shape[1] != H or not x.is_contiguous() or not w_router.is_contiguous():
        raise ValueError("x [T,H] and w_router [E,H] must be contiguous and agree on H")
    logits = torch.empty((T, E), dtype=torch.float32, device=x.device)
    idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    call("kvm_sm100_moe_router_topk", x.data_ptr(), w_router.data_ptr(), logits.data_ptr(),
         idx.data_ptr(), w.data_ptr(), T, H, E, top_k, _stream())
    return Routing(logits, idx, w)


def moe_permute(topk_idx: torch.Tensor, num_experts: int,
                workspace: torch.Tensor | None = None) -> Dispatch:
    """Deterministic (expert, token, slot) ordering of the routed pairs."""
    _check(topk_idx, "topk_idx", torch.int32, 2)
    if not topk_idx.is_contiguous():
        raise ValueError("topk_idx must be contiguous")
    T, k = topk_idx.shape
    dev = topk_idx.device
    ws_bytes = int(_lib.lib().kvm_sm100_moe_permute_workspace(T, k, num_experts))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    pos = torch.empty(T * k, dtype=torch.int32, device=dev)
    src = torch.empty(T * k, dtype=torch.int32, device=dev)
    call("kvm_sm100_moe_permute", topk_idx.data_ptr(), T, k, num_experts,
         offsets.data_ptr(), pos.data_ptr(), src.data_ptr(), workspace.data_ptr(), _stream())
    return Dispatch(offsets, pos, src)


def moe_scatter_rows(x: torch.Tensor, pos: torch.Tensor, top_k: int,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """xp[pos[t*k+j]] = x[t]: the dispatch copy into expert-major order."""
    _check(x, "x", torch.bfloat16, 2)
    _check(pos, "pos", torch.int32, 1)
    T, H = x.shape
    if out is None:
        out = torch.empty((T * top_k, H), dtype=torch.bfloat16, device=x.device)
    call("kvm_sm100_moe_scatter_rows", x.data_ptr(), pos.data_ptr(), out.data_ptr(),
         T, top_k, H, _stream())
    return out


def grouped_matmul(a: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor, *,
                   silu_gate: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-group D[rows of g] = A[rows of g] . w[g]^T; w: [G, N, K].

    With silu_gate=True, w is packed gate/up [G, 2F, K] and D = SiLU(g)*u [rows, F].
    """
    _check(a, "a", torch.bfloat16, 2)
    _check(w, "w", torch.bfloat16, 3)
    _check(offsets, "offsets", torch.int32, 1)
    rows, K = a.shape
    G, N, K2 = w.shape
    if K2 != K or offsets.numel() != G + 1 or not w.is_contiguous() or not a.is_contiguous():
        raise ValueError("grouped_matmul: shapes disagree or tensors not contiguous")
    n_out = N // 2 if silu_gate else N
    if out is None:
        out = torch.empty((rows, n_out), dtype=torch.bfloat16, device=a.device)
    call("kvm_sm100_grouped_gemm_bf16", a.data_ptr(), w.data_ptr(), out.data_ptr(),
         offsets.data_ptr(), G, rows, N, K, 2 if silu_gate else 0, _stream())
    return out


def moe_combine(y: torch.Tensor, pos: torch.Tensor, topk_w: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum_j w[t,j] * y[pos[t*k+j]] (comm.moe_combine)."""
    _check(y, "y", torch.bfloat16, 2)
    _check(pos, "pos", torch.int32, 1)
    _check(topk_w, "topk_w", torch.float32, 2)
    T, k = topk_w.shape
    H = y.shape[1]
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=y.device)
    call("kvm_sm100_moe_combine", y.data_ptr(), pos.data_ptr(), topk_w.data_ptr(),
         out.data_ptr(), T, k, H, _stream())
    return out


# ----------------------------------------------------------- elementwise ---

_EW_TORCH = {torch.bfloat16: "bf16", torch.float32: "f32", torch.float16: "f16",
             torch.int32: "i32"}


def elementwise(instrs, inputs, out_shape, out_dtype: torch.dtype = torch.bfloat16,
                out_reg: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = program(inputs): a fused chain of the kernel dialect's elementwise
    ops (kernel/dialect.cpp:43-55) as one generated sm_100a kernel.

    instrs: (op, a, b, dst) tuples over 16 fp32 registers, op one of
    _lib.EW_OPS ("load" reads input slot `a`); inputs: contiguous CUDA tensors
    (bf16/f32/f16/i32) broadcast numpy-style to out_shape; the result is
    register `out_reg` (default: the last instruction's dst) rounded to
    out_dtype.
    """
    out_shape = tuple(int(d) for d in out_shape)
    for i, t in enumerate(inputs):
        if not t.is_cuda or not t.is_contiguous() or t.dtype not in _EW_TORCH:
            raise ValueError(f"input {i} must be a contiguous CUDA bf16/f32/f16/i32 tensor")
    if out is None:
        out = torch.empty(out_shape, dtype=out_dtype, device=inputs[0].device if inputs
                          else torch.device("cuda"))
    prog = _lib.ew_program(instrs, [_EW_TORCH[t.dtype] for t in inputs],
                           [_lib.broadcast_of(tuple(t.shape), out_shape) for t in inputs],
                           _EW_TORCH[out.dtype],
                           instrs[-1][3] if out_reg is None else out_reg)
    ins = _lib.EwInputs()
    for i, t in enumerate(inputs):
        ins.ptr[i] = t.data_ptr()
    import ctypes
    call("kvm_sm100_elementwise", ctypes.byref(prog), ctypes.byref(ins), out.data_ptr(),
         out.numel(), _stream())
    return out


def device_status() -> int:
    """Synchronise; raise KvmError if a kernel recorded a timeout or bad index."""
    return _lib.device_status(clear=True)


__all__ = [
    "matmul", "gemm", "pack_gate_up", "quantize_e4m3", "matmul_fp8", "transpose_u8",
    "transpose_f32", "attention_prefill", "rope_", "transpose", "silu_gate_matmul", "rmsnorm",
    "silu_mul", "moe_route", "moe_permute", "moe_scatter_rows", "grouped_matmul",
    "moe_combine", "Routing", "Dispatch", "elementwise", "device_status", "KVM_B_KN", "KVM_B_NK",
]
