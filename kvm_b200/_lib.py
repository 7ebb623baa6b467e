"""ctypes binding of libkvm_sm100.so, the C ABI declared in include/kvm_sm100.h.

The library is loaded from the package directory only. There is no fallback:
if the shared object is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libkvm_sm100.so"
HEADER = PKG.parent / "include" / "kvm_sm100.h"

KVM_OK = 0
KVM_ERR_INVALID_ARG = 1
KVM_ERR_UNSUPPORTED = 2
KVM_ERR_CUDA = 3
KVM_ERR_TIMEOUT = 4
KVM_ERR_NCCL = 5

KVM_B_NK = 0
KVM_B_KN = 1
KVM_BF16 = 0
KVM_F32 = 1

_STATUS_NAMES = {
    KVM_ERR_INVALID_ARG: "invalid argument",
    KVM_ERR_UNSUPPORTED: "unsupported",
    KVM_ERR_CUDA: "CUDA error",
    KVM_ERR_TIMEOUT: "device wait timed out",
    KVM_ERR_NCCL: "collective failed",
}


class KvmError(RuntimeError):
    """A kvm_sm100_* call returned a non-zero kvm_status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn}: {_STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


_P = C.c_void_p
_I = C.c_int
_I64 = C.c_int64
_F = C.c_float

# name -> (restype, argtypes); must match include/kvm_sm100.h.
SIGNATURES = {
    "kvm_sm100_version": (_I, []),
    "kvm_sm100_last_error": (C.c_char_p, []),
    "kvm_sm100_device_status": (_I, [C.POINTER(_I), _I]),
    "kvm_sm100_kernel_binary_version": (_I, [C.POINTER(_I)]),
    "kvm_sm100_gemm_bf16": (_I, [_P, _I64, _P, _I64, _I, _P, _P, _I64, _I, _I, _I, _I, _P]),
    "kvm_sm100_gemm_bf16_silu_gate": (_I, [_P, _I64, _P, _P, _I64, _I, _I, _I, _P]),
    "kvm_sm100_pack_gate_up": (_I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "kvm_sm100_transpose_bf16": (_I, [_P, _P, _I, _I, _I, _P]),
    "kvm_sm100_moe_router_topk": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "kvm_sm100_moe_permute_workspace": (_I64, [_I, _I, _I]),
    "kvm_sm100_moe_permute": (_I, [_P, _I, _I, _I, _P, _P, _P, _P, _P]),
    "kvm_sm100_moe_permute_noalloc": (_I, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "kvm_sm100_moe_permute_noalloc_status": (_I, [C.POINTER(_I), _I]),
    "kvm_sm100_moe_scatter_rows": (_I, [_P, _P, _P, _I, _I, _I, _P]),
    "kvm_sm100_grouped_gemm_bf16": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "kvm_sm100_moe_combine": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "kvm_sm100_ipc_alloc": (_I, [_I64, C.POINTER(C.c_void_p)]),
    "kvm_sm100_ipc_free": (_I, [_P]),
    "kvm_sm100_ipc_get_handle": (_I, [_P, _P]),
    "kvm_sm100_ipc_open_handle": (_I, [_P, C.POINTER(C.c_void_p)]),
    "kvm_sm100_ipc_close": (_I, [_P]),
    "kvm_sm100_ep_counts": (_I, [_P, _P, _P, _P, C.c_uint32, _P]),
    "kvm_sm100_ep_dispatch": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _P, C.c_uint32, _P]),
    "kvm_sm100_ep_wait": (_I, [_P, _I, C.c_uint32, _P]),
    "kvm_sm100_ep_signal": (_I, [_P, _I, C.c_uint32, _P]),
    "kvm_sm100_ep_combine": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _P]),
    "kvm_sm100_ep_overlap_workspace": (_I64, [_I, _I64]),
    "kvm_sm100_ep_prepare": (_I, [_P, _P, _P, _P, _P, _I64, C.c_uint32, _P]),
    "kvm_sm100_ep_scatter_local": (_I, [_P, _P, _P, _P, _P, _I, _I64, _P]),
    "kvm_sm100_ep_dispatch_gate_up": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I64, _P,
                                           C.c_uint32, _P]),
    "kvm_sm100_ep_down_push": (_I, [_P, _P, _P, _P, _I, _I64, _P, C.c_uint32, _P]),
    "kvm_sm100_gemm_fp8_workspace": (_I64, [_I, _I, _I]),
    "kvm_sm100_gemm_fp8_blockscaled": (_I, [_P, _P, _P, _P, _P, _I64, _I, _I, _I, _P, _I64,
                                            _P]),
    "kvm_sm100_quantize_e4m3_block128": (_I, [_P, _I, _P, _P, _I, _I, _P]),
    "kvm_sm100_transpose_u8": (_I, [_P, _P, _I, _I, _P]),
    "kvm_sm100_transpose_f32": (_I, [_P, _P, _I, _I, _P]),
    "kvm_sm100_attention_workspace": (_I64, [_I, _I, _I, _I]),
    "kvm_sm100_attention_prefill_bf16": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I,
                                              _I, _I, _I, _F, _P, _I64, _P]),
    "kvm_sm100_rope_bf16": (_I, [_P, _I64, _I, _I, _I, _I, _F, _P]),
    "kvm_sm100_elementwise": (_I, [_P, _P, _P, _I64, _P]),
    "kvm_sm100_elementwise_prepare": (_I, [_P, _P, _P, _I64]),
    "kvm_sm100_gemv_bf16": (_I, [_P, _I64, _P, _P, _I, _I, _I, _P]),
    "kvm_sm100_moe_topk": (_I, [_P, _I, _I, _I, _I, _P, _P, _P]),
    "kvm_sm100_fill_normal": (_I, [_P, _I, _I64, C.c_uint64, _F, _F, _P]),
    "kvm_sm100_rmsnorm_bf16": (_I, [_P, _P, _P, _I, _I, _F, _P]),
    "kvm_sm100_silu_mul_bf16": (_I, [_P, _P, _P, _I64, _P]),
    "kvm_sm100_comm_unique_id": (_I, [_P]),
    "kvm_sm100_comm_init": (_I, [_I, _I, _P, C.POINTER(C.c_void_p)]),
    "kvm_sm100_comm_split": (_I, [_P, _P, _I, C.POINTER(C.c_void_p)]),
    "kvm_sm100_comm_rank": (_I, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "kvm_sm100_comm_destroy": (_I, [_P]),
    "kvm_sm100_all_reduce": (_I, [_P, _P, _P, _I64, _I, _I, _P]),
    "kvm_sm100_all_gather": (_I, [_P, _P, _P, _I64, _I, _P]),
    "kvm_sm100_broadcast": (_I, [_P, _P, _P, _I64, _I, _I, _P]),
    "kvm_sm100_send": (_I, [_P, _P, _I64, _I, _I, _P]),
    "kvm_sm100_recv": (_I, [_P, _P, _I64, _I, _I, _P]),
    "kvm_sm100_all_to_all": (_I, [_P, _P, _P, _I64, _I, _P]),
    "kvm_sm100_kvcache_write": (_I, [_P, _P, _P, _I64, _P, _I64, _P, _P, _P, _P, _I, _I, _P]),
    "kvm_sm100_kvcache_read": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _P]),
    "kvm_sm100_attention_decode_workspace": (_I64, [_I, _I, _I, _I, _I]),
    "kvm_sm100_attention_decode_paged": (_I, [_P, _I64, _P, _P, _P, _I64, _P, _P, _P, _P,
                                              _I, _I, _I, _I, _F, _P, _I64, _P]),
}

KVM_EP_MAX_RANKS = 8


class EpPeers(C.Structure):
    """Mirror of struct kvm_ep_peers (include/kvm_sm100.h)."""
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("E", C.c_int32),
                ("H", C.c_int32), ("k", C.c_int32), ("pad_", C.c_int32),
                ("recv", C.c_void_p * KVM_EP_MAX_RANKS), ("y", C.c_void_p * KVM_EP_MAX_RANKS),
                ("cnt", C.c_void_p * KVM_EP_MAX_RANKS),
                ("flags", C.c_void_p * KVM_EP_MAX_RANKS)]


class KvLayout(C.Structure):
    """Mirror of struct kvm_kv_layout (include/kvm_sm100.h)."""
    _fields_ = [("page_stride", C.c_int64), ("layer_stride", C.c_int64),
                ("kv_stride", C.c_int64), ("token_stride", C.c_int64),
                ("block_size", C.c_int32), ("layer", C.c_int32), ("width", C.c_int32),
                ("num_pages", C.c_int32)]


KVM_EW_MAX_INPUTS, KVM_EW_MAX_INSTR, KVM_EW_MAX_REGS = 8, 32, 16
# enum kvm_ew_dtype / kvm_ew_op (include/kvm_sm100.h)
EW_DTYPES = {"bf16": 0, "f32": 1, "f16": 2, "i32": 3}
EW_OPS = ["load", "add", "sub", "mul", "div", "max", "min", "neg", "exp", "log", "sqrt",
          "rsqrt", "abs", "rcp", "cmp.eq", "cmp.ne", "cmp.lt", "cmp.le", "cmp.gt",
          "cmp.ge", "round.bf16", "round.f16", "trunc.i32"]


class EwProgram(C.Structure):
    """Mirror of struct kvm_ew_program (include/kvm_sm100.h)."""
    _fields_ = [("n_inputs", C.c_int32), ("n_instr", C.c_int32), ("out_reg", C.c_int32),
                ("out_dtype", C.c_int32), ("in_dtype", C.c_int32 * KVM_EW_MAX_INPUTS),
                ("in_size", C.c_int64 * KVM_EW_MAX_INPUTS),
                ("in_div", C.c_int64 * KVM_EW_MAX_INPUTS),
                ("op", C.c_uint8 * KVM_EW_MAX_INSTR), ("a", C.c_uint8 * KVM_EW_MAX_INSTR),
                ("b", C.c_uint8 * KVM_EW_MAX_INSTR), ("dst", C.c_uint8 * KVM_EW_MAX_INSTR)]


class EwInputs(C.Structure):
    """Mirror of struct kvm_ew_inputs (include/kvm_sm100.h)."""
    _fields_ = [("ptr", C.c_void_p * KVM_EW_MAX_INPUTS)]


def broadcast_of(in_shape, out_shape) -> tuple[int, int]:
    """(in_size, in_div) of an input of `in_shape` broadcast numpy-style to
    `out_shape`: its non-1 dimensions, right-aligned, must be one contiguous
    run of the output's dimensions."""
    r = len(out_shape)
    if len(in_shape) > r:
        raise ValueError("elementwise operand has more dimensions than the result")
    s = [1] * (r - len(in_shape)) + list(in_shape)
    run = [d for d in range(r) if s[d] != 1]
    for d in run:
        if s[d] != out_shape[d]:
            raise ValueError("elementwise operand does not broadcast")
    if run and run != list(range(run[0], run[-1] + 1)):
        raise ValueError("unsupported broadcast pattern")
    if not run:
        return 1, 1
    size = 1
    for d in run:
        size *= out_shape[d]
    div = 1
    for d in range(run[-1] + 1, r):
        div *= out_shape[d]
    return size, div


def ew_program(instrs, in_dtypes, in_bcast, out_dtype: str, out_reg: int) -> EwProgram:
    """An EwProgram from (op, a, b, dst) tuples (op a name of EW_OPS; for
    "load", `a` is the input slot), input dtype names and (size, div) pairs."""
    p = EwProgram()
    p.n_inputs, p.n_instr = len(in_dtypes), len(instrs)
    p.out_reg, p.out_dtype = out_reg, EW_DTYPES[out_dtype]
    for i, (dt, (size, div)) in enumerate(zip(in_dtypes, in_bcast)):
        p.in_dtype[i], p.in_size[i], p.in_div[i] = EW_DTYPES[dt], size, div
    for s, (op, a, b, dst) in enumerate(instrs):
        p.op[s], p.a[s], p.b[s], p.dst[s] = EW_OPS.index(op), a, b, dst
    return p


_lib: C.CDLL | None = None


def header_symbols() -> list[str]:
    """Every function name declared in include/kvm_sm100.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(kvm_sm100_\w+)\s*\(", text)))


def lib() -> C.CDLL:
    """Load (once) and return the C ABI library, with typed signatures."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m kvm_b200.build`"
                " (there is no CPU fallback)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def call(name: str, *args) -> None:
    """Call kvm_sm100_<name>; raise KvmError on a non-zero status."""
    L = lib()
    rc = getattr(L, name)(*args)
    if rc != KVM_OK:
        msg = L.kvm_sm100_last_error()
        raise KvmError(name, rc, msg.decode() if msg else "")


def device_status(clear: bool = True) -> int:
    """Synchronise and return the device status word (raises on error bits)."""
    v = C.c_int(0)
    call("kvm_sm100_device_status", C.byref(v), int(clear))
    return v.value
