"""Paged KV cache and decode attention on the sm_100a kernels.

A pool holds K and V for `layers` layers in pages of `block_size` token
slots; a slot is one token's K (or V) row of width HKV * 128 bf16. KVMeta's
two layouts (src/ir/graph_config.h:20-39):
    page_first   [page][layer][kv][slot][width]
    layer_first  [layer][page][kv][slot][width]
Sequences own pages through a block table (AttnMetaImpl's kv block_table,
src/ir/dialect/kernel/values.h:83-117), flattened as `block_table` with
`bt_offsets` [S+1]. kvcache.write / kvcache.read / attn.decode are the ops of
src/ir/dialect/kernel/dialect.cpp:39,69-70.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import call
from .ops import _check, _rowmajor, _stream


def kv_strides(layout: str, pages: int, layers: int, block_size: int, width: int):
    """Element strides (page, layer, kv, token) of a pool in `layout`."""
    kv = block_size * width
    if layout == "page_first":
        layer = 2 * kv
        page = layers * layer
    elif layout == "layer_first":
        page = 2 * kv
        layer = pages * page
    else:
        raise ValueError(f"unknown KV layout {layout!r}")
    return page, layer, kv, width


class PagedKVCache:
    """A device pool of KV pages (bf16, zero-initialised)."""

    def __init__(self, *, pages: int, layers: int, block_size: int, heads_kv: int,
                 layout: str = "page_first", device=None):
        self.pages, self.layers, self.block_size = pages, layers, block_size
        self.heads_kv, self.width, self.layout = heads_kv, heads_kv * 128, layout
        self.strides = kv_strides(layout, pages, layers, block_size, self.width)
        n = pages * layers * 2 * block_size * self.width
        self.pool = torch.zeros(n, dtype=torch.bfloat16, device=device)

    def layout_struct(self, layer: int) -> _lib.KvLayout:
        if not 0 <= layer < self.layers:
            raise ValueError("layer out of range")
        ps, ls, ks, ts = self.strides
        return _lib.KvLayout(ps, ls, ks, ts, self.block_size, layer, self.width, self.pages)

    def write(self, layer: int, k: torch.Tensor, v: torch.Tensor, q_offsets: torch.Tensor,
              q_positions: torch.Tensor, block_table: torch.Tensor,
              bt_offsets: torch.Tensor) -> None:
        """kvcache.write: rows of k/v [rows, width] to their page slots."""
        _check(k, "k", torch.bfloat16, 2)
        _check(v, "v", torch.bfloat16, 2)
        for t, n in ((q_offsets, "q_offsets"), (q_positions, "q_positions"),
                     (block_table, "block_table"), (bt_offsets, "bt_offsets")):
            _check(t, n, torch.int32, 1)
        L = self.layout_struct(layer)
        call("kvm_sm100_kvcache_write", self.pool.data_ptr(), C.byref(L), k.data_ptr(),
             _rowmajor(k, "k"), v.data_ptr(), _rowmajor(v, "v"), q_offsets.data_ptr(),
             q_positions.data_ptr(), block_table.data_ptr(), bt_offsets.data_ptr(),
             q_offsets.numel() - 1, k.shape[0], _stream())

    def read(self, layer: int, kv_offsets: torch.Tensor, block_table: torch.Tensor,
             bt_offsets: torch.Tensor, rows: int):
        """kvcache.read: (k, v) [rows, width], each sequence's tokens in order."""
        L = self.layout_struct(layer)
        k = torch.empty((rows, self.width), dtype=torch.bfloat16, device=self.pool.device)
        v = torch.empty_like(k)
        call("kvm_sm100_kvcache_read", self.pool.data_ptr(), C.byref(L), k.data_ptr(),
             v.data_ptr(), kv_offsets.data_ptr(), block_table.data_ptr(),
             bt_offsets.data_ptr(), kv_offsets.numel() - 1, rows, _stream())
        return k, v

    def decode(self, layer: int, q: torch.Tensor, q_offsets: torch.Tensor,
               q_positions: torch.Tensor, block_table: torch.Tensor,
               bt_offsets: torch.Tensor, *, heads_q: int, max_q_rows: int, max_keys: int,
               scale: float = 0.0, out: torch.Tensor | None = None,
               workspace: torch.Tensor | None = None) -> torch.Tensor:
        """attn.decode: causal attention of the new rows q [rows, HQ*128] over
        the cached positions up to their own."""
        _check(q, "q", torch.bfloat16, 2)
        L = self.layout_struct(layer)
        S = q_offsets.numel() - 1
        if out is None:
            out = torch.empty((q.shape[0], heads_q * 128), dtype=torch.bfloat16,
                              device=q.device)
        need = int(_lib.lib().kvm_sm100_attention_decode_workspace(
            S, heads_q, self.heads_kv, max_q_rows, max_keys))
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
        call("kvm_sm100_attention_decode_paged", q.data_ptr(), _rowmajor(q, "q"),
             self.pool.data_ptr(), C.byref(L), out.data_ptr(), _rowmajor(out, "out"),
             q_offsets.data_ptr(), q_positions.data_ptr(), block_table.data_ptr(),
             bt_offsets.data_ptr(), S, heads_q, max_q_rows, max_keys, float(scale),
             workspace.data_ptr(), workspace.numel(), _stream())
        return out
