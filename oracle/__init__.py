"""CPU oracle for the KVM execution backend -- TEST INFRASTRUCTURE ONLY.

numpy front end over oracle/_build/liboracle.so (oracle/oracle.c, built by
``make -C oracle``). Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg use this module, as the checker. Parity is UNPINNED: the
reference has no numeric execution path or golden vectors; the C file states
which reference op definitions each function restates.

bf16 arrays are carried as numpy uint16 (raw bit patterns).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_lib: C.CDLL | None = None


def build() -> Path:
    """Compile oracle.c (gcc, OpenMP) into _build/liboracle.so."""
    r = subprocess.run(["make", "-s", "-C", str(HERE)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.c_float
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_f32_to_bf16.argtypes = [F]
        L.orc_bf16_to_f32.restype = F
        L.orc_bf16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_bf16_array.argtypes = [P, P, I64]
        L.orc_gemm_bf16.argtypes = [P, I64, P, I64, I, P, P, I64, I, I, I, I]
        L.orc_gemm_silu_gate.argtypes = [P, P, P, P, I, I, I]
        L.orc_pack_gate_up.argtypes = [P, P, P, I, I, I]
        L.orc_rmsnorm_bf16.argtypes = [P, P, P, I, I, F]
        L.orc_silu_mul_bf16.argtypes = [P, P, P, I64]
        L.orc_moe_topk.argtypes = [P, I, I, I, P, P]
        L.orc_moe_permute.restype = I
        L.orc_moe_permute.argtypes = [P, I, I, I, P, P, P]
        L.orc_moe_scatter_rows.argtypes = [P, P, P, I, I, I]
        L.orc_grouped_gemm_bf16.argtypes = [P, P, P, P, I, I, I, I]
        L.orc_moe_combine.argtypes = [P, P, P, P, I, I, I]
        L.orc_moe_layer.argtypes = [P, P, P, P, P, I, I, I, I, I, P, P, P]
        L.orc_num_threads.restype = I
        L.orc_f32_to_e4m3_array.argtypes = [P, P, I64]
        L.orc_e4m3_to_f32.restype = F
        L.orc_e4m3_to_f32.argtypes = [C.c_uint8]
        L.orc_quantize_e4m3_block128.argtypes = [P, I, I, P, P]
        L.orc_gemm_fp8_blockscaled.argtypes = [P, P, P, P, P, I, I, I]
        L.orc_rope_bf16.argtypes = [P, I64, I, I, I, I, F]
        L.orc_attention_bf16.argtypes = [P, I64, P, I64, P, I64, P, I64, I, I, I, I, I, F]
        L.orc_kvcache_write.argtypes = [P, I64, I64, I64, I64, I, I, I, P, I64, P, I64,
                                        P, P, P, P, I]
        L.orc_kvcache_read.argtypes = [P, I64, I64, I64, I64, I, I, I, P, P, P, P, P, I]
        L.orc_attention_decode.argtypes = [P, I64, P, I64, I64, I64, I64, I, I, P, I64,
                                           P, P, P, P, I, I, I, I, F]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def _c(a: np.ndarray, dtype) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype != dtype:
        raise TypeError(f"expected {dtype}, got {a.dtype}")
    return a


# ------------------------------------------------------------- numerics ---

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (RNE); returns uint16 bit patterns."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_bf16_array(_p(x), _p(out), x.size)
    return out


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    return (h.astype(np.uint32) << 16).view(np.float32)


def elementwise(instrs, inputs, bcast, out_dtype: str, out_reg: int, n: int) -> np.ndarray:
    """The elementwise program of kvm_sm100_elementwise, element by element in
    fp32 numpy: the kernel dialect's arithmetic, compare and cast ops
    (src/ir/dialect/kernel/dialect.cpp:43-55) as task.alu.* / task.sfu.*
    (src/ir/dialect/task/dialect.cpp:36-51), each rounded to fp32 on its own.

    instrs: (op, a, b, dst) tuples; inputs: (array, dtype name) with bf16 and
    f16 as raw uint16 bits; bcast: (size, div) per input -- output element i
    reads input[(i // div) % size]. Returns bf16/f16 as uint16 bits, f32 or
    int32 (saturating toward zero, NaN -> 0)."""
    i = np.arange(n, dtype=np.int64)
    regs = [np.zeros(n, np.float32) for _ in range(16)]
    f32 = np.float32
    with np.errstate(all="ignore"):
        for op, a, b, dst in instrs:
            if op == "load":
                arr, dt = inputs[a]
                size, div = bcast[a]
                flat = np.ascontiguousarray(arr).reshape(-1)
                if dt == "bf16":
                    vals = bf16_to_f32(flat)
                elif dt == "f16":
                    vals = flat.view(np.float16).astype(f32)
                else:
                    vals = flat.astype(f32)
                v = vals[(i // div) % size]
            else:
                x, y = regs[a], regs[b]
                v = {
                    "add": lambda: x + y, "sub": lambda: x - y, "mul": lambda: x * y,
                    "div": lambda: x / y, "max": lambda: np.fmax(x, y),
                    "min": lambda: np.fmin(x, y), "neg": lambda: -x,
                    "exp": lambda: np.exp(x), "log": lambda: np.log(x),
                    "sqrt": lambda: np.sqrt(x), "rsqrt": lambda: f32(1) / np.sqrt(x),
                    "abs": lambda: np.abs(x), "rcp": lambda: f32(1) / x,
                    "cmp.eq": lambda: (x == y).astype(f32), "cmp.ne": lambda: (x != y).astype(f32),
                    "cmp.lt": lambda: (x < y).astype(f32), "cmp.le": lambda: (x <= y).astype(f32),
                    "cmp.gt": lambda: (x > y).astype(f32), "cmp.ge": lambda: (x >= y).astype(f32),
                    "round.bf16": lambda: bf16_to_f32(f32_to_bf16(x)),
                    "round.f16": lambda: x.astype(np.float16).astype(f32),
                    "trunc.i32": lambda: np.trunc(x),
                }[op]()
            regs[dst] = np.asarray(v, dtype=f32)
        r = regs[out_reg]
        if out_dtype == "bf16":
            return f32_to_bf16(r)
        if out_dtype == "f16":
            return r.astype(np.float16).view(np.uint16)
        if out_dtype == "i32":
            t = np.nan_to_num(np.trunc(r.astype(np.float64)), nan=0.0)
            return np.clip(t, -2.0 ** 31, 2.0 ** 31 - 1).astype(np.int32)
        return r


def normal_bf16(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    """Seeded N(0, std^2) values rounded to bf16 (uint16 bits)."""
    return f32_to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


# ------------------------------------------------------------------ ops ---

def gemm(a: np.ndarray, b: np.ndarray, *, b_layout: str = "kn",
         c: np.ndarray | None = None, out_f32: bool = False) -> np.ndarray:
    a = _c(a, np.uint16)
    b = _c(b, np.uint16)
    M, K = a.shape
    if b_layout == "kn":
        N, bkn = b.shape[1], 1
    else:
        N, bkn = b.shape[0], 0
    out = np.empty((M, N), dtype=np.float32 if out_f32 else np.uint16)
    if c is not None:
        c = _c(c, out.dtype)
    lib().orc_gemm_bf16(_p(a), K, _p(b), b.shape[1], bkn, _p(c), _p(out), N,
                        int(out_f32), M, N, K)
    return out


def gemm_silu_gate(a: np.ndarray, wg: np.ndarray, wu: np.ndarray) -> np.ndarray:
    a, wg, wu = _c(a, np.uint16), _c(wg, np.uint16), _c(wu, np.uint16)
    M, K = a.shape
    F = wg.shape[0]
    out = np.empty((M, F), dtype=np.uint16)
    lib().orc_gemm_silu_gate(_p(a), _p(wg), _p(wu), _p(out), M, F, K)
    return out


def pack_gate_up(wg: np.ndarray, wu: np.ndarray) -> np.ndarray:
    """[G, F, K] gate/up -> [G, 2F, K] interleaved in 64-row blocks."""
    wg, wu = _c(wg, np.uint16), _c(wu, np.uint16)
    G, F, K = wg.shape
    out = np.empty((G, 2 * F, K), dtype=np.uint16)
    lib().orc_pack_gate_up(_p(wg), _p(wu), _p(out), G, F, K)
    return out


def rmsnorm(x: np.ndarray, gamma: np.ndarray | None, eps: float) -> np.ndarray:
    x = _c(x, np.uint16)
    H = x.shape[-1]
    out = np.empty_like(x)
    g = None if gamma is None else _c(gamma, np.uint16)
    lib().orc_rmsnorm_bf16(_p(x), _p(g), _p(out), x.size // H, H, eps)
    return out


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g, u = _c(g, np.uint16), _c(u, np.uint16)
    out = np.empty_like(g)
    lib().orc_silu_mul_bf16(_p(g), _p(u), _p(out), g.size)
    return out


def moe_topk(logits: np.ndarray, k: int):
    logits = _c(logits, np.float32)
    T, E = logits.shape
    idx = np.empty((T, k), dtype=np.int32)
    w = np.empty((T, k), dtype=np.float32)
    lib().orc_moe_topk(_p(logits), T, E, k, _p(idx), _p(w))
    return idx, w


def moe_permute(idx: np.ndarray, E: int):
    idx = _c(idx, np.int32)
    T, k = idx.shape
    off = np.empty(E + 1, dtype=np.int32)
    pos = np.empty(T * k, dtype=np.int32)
    src = np.empty(T * k, dtype=np.int32)
    rc = lib().orc_moe_permute(_p(idx), T, k, E, _p(off), _p(pos), _p(src))
    if rc != 0:
        raise ValueError("expert index out of range")
    return off, pos, src


def moe_scatter_rows(x: np.ndarray, pos: np.ndarray, k: int) -> np.ndarray:
    x, pos = _c(x, np.uint16), _c(pos, np.int32)
    T, H = x.shape
    out = np.zeros((T * k, H), dtype=np.uint16)
    lib().orc_moe_scatter_rows(_p(x), _p(pos), _p(out), T, k, H)
    return out


def grouped_gemm(a: np.ndarray, w: np.ndarray, offsets: np.ndarray,
                 silu_gate: bool = False) -> np.ndarray:
    a, w, offsets = _c(a, np.uint16), _c(w, np.uint16), _c(offsets, np.int32)
    rows, K = a.shape
    G, N, _ = w.shape
    out = np.zeros((rows, N // 2 if silu_gate else N), dtype=np.uint16)
    lib().orc_grouped_gemm_bf16(_p(a), _p(w), _p(out), _p(offsets), G, N, K, int(silu_gate))
    return out


def moe_combine(y: np.ndarray, pos: np.ndarray, w: np.ndarray) -> np.ndarray:
    y, pos, w = _c(y, np.uint16), _c(pos, np.int32), _c(w, np.float32)
    T, k = w.shape
    H = y.shape[1]
    out = np.empty((T, H), dtype=np.uint16)
    lib().orc_moe_combine(_p(y), _p(pos), _p(w), _p(out), T, k, H)
    return out


def moe_layer_given_routing(x, w13, w2, idx, tw):
    """The MoE layer after routing, for a given top-k (idx [T,k] int32, tw
    [T,k] fp32): permute, scatter, grouped SiLU-gate GEMM, grouped down GEMM,
    combine -- the same steps orc_moe_layer takes after its own top-k."""
    E = w13.shape[0]
    k = idx.shape[1]
    off, pos, _ = moe_permute(idx, E)
    xp = moe_scatter_rows(x, pos, k)
    h = grouped_gemm(xp, w13, off, silu_gate=True)
    y = grouped_gemm(h, w2, off)
    return moe_combine(y, pos, tw)


def topk_gap(logits: np.ndarray, k: int) -> np.ndarray:
    """Per row, the fp32 gap between the k-th and (k+1)-th largest logit: a
    row whose top-k can flip under fp32 reassociation has a gap near 0."""
    s = -np.sort(-np.asarray(logits, dtype=np.float32), axis=1)
    if s.shape[1] <= k:
        return np.full(s.shape[0], np.inf, dtype=np.float32)
    return s[:, k - 1] - s[:, k]


def moe_layer(x, w_router, w13, w2, k: int):
    """Whole MoE layer; returns (out, logits, topk_idx, topk_w)."""
    x, wr = _c(x, np.uint16), _c(w_router, np.uint16)
    w13, w2 = _c(w13, np.uint16), _c(w2, np.uint16)
    T, H = x.shape
    E = wr.shape[0]
    F = w13.shape[1] // 2
    out = np.empty((T, H), dtype=np.uint16)
    logits = np.empty((T, E), dtype=np.float32)
    idx = np.empty((T, k), dtype=np.int32)
    tw = np.empty((T, k), dtype=np.float32)
    lib().orc_moe_layer(_p(x), _p(wr), _p(w13), _p(w2), _p(out), T, H, E, F, k,
                        _p(logits), _p(idx), _p(tw))
    return out, logits, idx, tw


# ------------------------------------------------------------------ FP8 ---

def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    lib().orc_f32_to_e4m3_array(_p(x), _p(out), x.size)
    return out


def e4m3_to_f32(q: np.ndarray) -> np.ndarray:
    lut = np.array([lib().orc_e4m3_to_f32(v) for v in range(256)], dtype=np.float32)
    return lut[np.asarray(q, dtype=np.uint8)]


def quantize_e4m3_block128(x: np.ndarray):
    x = _c(np.asarray(x, dtype=np.float32), np.float32)
    R, Cc = x.shape
    q = np.empty((R, Cc), dtype=np.uint8)
    s = np.empty(((R + 127) // 128, (Cc + 127) // 128), dtype=np.float32)
    lib().orc_quantize_e4m3_block128(_p(x), R, Cc, _p(q), _p(s))
    return q, s


def gemm_fp8_blockscaled(aq, sa, wq, sw) -> np.ndarray:
    aq, wq = _c(aq, np.uint8), _c(wq, np.uint8)
    sa, sw = _c(sa, np.float32), _c(sw, np.float32)
    M, K = aq.shape
    N = wq.shape[0]
    out = np.empty((M, N), dtype=np.uint16)
    lib().orc_gemm_fp8_blockscaled(_p(aq), _p(sa), _p(wq), _p(sw), _p(out), M, N, K)
    return out


def rope(x: np.ndarray, L: int, heads: int, hd: int = 128, base: float = 10000.0):
    """Rotary embedding of a [rows, heads*hd] bf16 matrix (returns a copy)."""
    x = np.array(_c(x, np.uint16), copy=True)
    lib().orc_rope_bf16(_p(x), x.shape[1], x.shape[0], L, heads, hd, base)
    return x


def attention(q, k, v, B: int, HQ: int, HKV: int, hd: int = 128, scale: float = 0.0):
    q, k, v = _c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16)
    L = q.shape[0] // B
    if scale <= 0:
        scale = 1.0 / np.sqrt(hd)
    out = np.empty((q.shape[0], HQ * hd), dtype=np.uint16)
    lib().orc_attention_bf16(_p(q), q.shape[1], _p(k), k.shape[1], _p(v), v.shape[1],
                             _p(out), out.shape[1], B, L, HQ, HKV, hd, float(scale))
    return out


# ------------------------------------------------------- paged KV cache ---

def kv_strides(layout: str, pages: int, layers: int, block_size: int, width: int):
    """Element strides (page, layer, kv, token) of a paged KV pool holding K
    and V for `layers` layers: page_first = [page][layer][kv][slot][width],
    layer_first = [layer][page][kv][slot][width]."""
    tok = width
    kv = block_size * width
    if layout == "page_first":
        layer = 2 * kv
        page = layers * layer
    elif layout == "layer_first":
        page = 2 * kv
        layer = pages * page
    else:
        raise ValueError(layout)
    return page, layer, kv, tok


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def kvcache_write(cache: np.ndarray, strides, block_size: int, layer: int, k, v,
                  q_off, q_pos, bt, bt_off) -> np.ndarray:
    """Copy of the flat bf16 pool `cache` with the new tokens' K/V rows written."""
    cache = np.array(_c(cache, np.uint16), copy=True)
    k, v = _c(k, np.uint16), _c(v, np.uint16)
    q_off, q_pos, bt, bt_off = _i32(q_off), _i32(q_pos), _i32(bt), _i32(bt_off)
    lib().orc_kvcache_write(_p(cache), *strides, block_size, layer, k.shape[1], _p(k),
                            k.shape[1], _p(v), v.shape[1], _p(q_off), _p(q_pos), _p(bt),
                            _p(bt_off), len(q_off) - 1)
    return cache


def kvcache_read(cache: np.ndarray, strides, block_size: int, layer: int, width: int,
                 kv_off, bt, bt_off):
    """(k, v) [sum kv_len, width]: each sequence's cached tokens in order."""
    cache = _c(cache, np.uint16)
    kv_off, bt, bt_off = _i32(kv_off), _i32(bt), _i32(bt_off)
    rows = int(kv_off[-1])
    k = np.empty((rows, width), dtype=np.uint16)
    v = np.empty((rows, width), dtype=np.uint16)
    lib().orc_kvcache_read(_p(cache), *strides, block_size, layer, width, _p(k), _p(v),
                           _p(kv_off), _p(bt), _p(bt_off), len(kv_off) - 1)
    return k, v


def attention_decode(q, cache, strides, block_size: int, layer: int, q_off, q_pos, bt,
                     bt_off, HQ: int, HKV: int, hd: int = 128, scale: float = 0.0):
    """Causal attention of the new query rows over the paged cache."""
    q, cache = _c(q, np.uint16), _c(cache, np.uint16)
    q_off, q_pos, bt, bt_off = _i32(q_off), _i32(q_pos), _i32(bt), _i32(bt_off)
    if scale <= 0:
        scale = 1.0 / np.sqrt(hd)
    out = np.empty((q.shape[0], HQ * hd), dtype=np.uint16)
    lib().orc_attention_decode(_p(q), q.shape[1], _p(cache), *strides, block_size, layer,
                               _p(out), out.shape[1], _p(q_off), _p(q_pos), _p(bt),
                               _p(bt_off), len(q_off) - 1, HQ, HKV, hd, float(scale))
    return out


def cuda_host_e4m3(x: np.ndarray) -> np.ndarray:
    """CUDA's host-side saturating e4m3 conversion (the known answer)."""
    so = HERE / "_build" / "libfp8pin.so"
    if not so.exists():
        build()
    L = C.CDLL(str(so))
    L.pin_f32_to_e4m3_array.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8)
    L.pin_f32_to_e4m3_array(_p(x), _p(out), x.size)
    return out


def num_threads() -> int:
    return int(lib().orc_num_threads())
