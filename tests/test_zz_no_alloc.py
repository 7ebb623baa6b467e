"""The allocation-free permute entry point (kvm_sm100_moe_permute_noalloc).

Callers that cannot allocate GPU memory while routing -- a host program that
owns all device buffers through its own pool, or a serving loop that must not
call cudaMalloc/cudaFree because they synchronise the device -- use this entry
point; its scratch is a fixed static device array instead of a workspace.

The GPU tests call it through the C ABI several times in a row (each call sees
the previous call's leftovers in the shared array) and compare every output
with the workspace-based kvm_sm100_moe_permute, bit for bit (permutation work
is integer work). The sizes cover the fused path (count matrix up to 16 K
cells), the separate scan pass (16 K to 64 K cells) and the exact 65536-cell
limit. Further tests check that a call allocates nothing and that an
out-of-range expert index reaches the entry point's own status word. The file
is collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from kvm_b200 import _lib

MAX_CELLS = 65536


def _cells(T, k, E):
    return -(-T * k // 256) * E


def _buffers(T, k, E, dev):
    off = torch.full((E + 1,), -7, dtype=torch.int32, device=dev)
    pos = torch.full((T * k,), -7, dtype=torch.int32, device=dev)
    src = torch.full((T * k,), -7, dtype=torch.int32, device=dev)
    return off, pos, src


def _call_noalloc(idx, E, off, pos, src):
    T, k = idx.shape
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("kvm_sm100_moe_permute_noalloc", idx.data_ptr(), T, k, E,
              off.data_ptr(), pos.data_ptr(), src.data_ptr(), st)


def _permute(idx: torch.Tensor, E: int, noalloc: bool):
    T, k = idx.shape
    off, pos, src = _buffers(T, k, E, idx.device)
    if noalloc:
        _call_noalloc(idx, E, off, pos, src)
    else:
        st = torch.cuda.current_stream().cuda_stream
        nbytes = int(_lib.lib().kvm_sm100_moe_permute_workspace(T, k, E))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=idx.device)
        _lib.call("kvm_sm100_moe_permute", idx.data_ptr(), T, k, E, off.data_ptr(),
                  pos.data_ptr(), src.data_ptr(), ws.data_ptr(), st)
    torch.cuda.synchronize()
    return off.cpu().numpy(), pos.cpu().numpy(), src.cpu().numpy()


def _noalloc_status(clear=True):
    v = C.c_int(0)
    rc = _lib.lib().kvm_sm100_moe_permute_noalloc_status(C.byref(v), int(clear))
    return rc, v.value


@pytest.mark.gpu
def test_noalloc_permute_matches_workspace_permute(cuda):
    rng = np.random.default_rng(123)
    _noalloc_status(clear=True)
    # Calls in a row, largest first, so later calls run on a scratch array
    # still holding an earlier call's counts and bases.
    cases = [(32768, 2, 256),   # exactly MAX_CELLS: separate scan pass
             (40000, 2, 64),    # 20032 cells: separate scan pass
             (8192, 2, 64),     # 4096 cells: scan fused into the rank pass
             (1000, 3, 40)]     # 480 cells, ragged last chunk
    assert _cells(*cases[0]) == MAX_CELLS
    for T, k, E in cases:
        idx = torch.from_numpy(rng.integers(0, E, (T, k)).astype(np.int32)).to(cuda)
        want = _permute(idx, E, noalloc=False)
        got = _permute(idx, E, noalloc=True)
        for a, b in zip(got, want):
            assert np.array_equal(a, b), (T, k, E)
    _lib.device_status()
    assert _noalloc_status() == (_lib.KVM_OK, 0)


@pytest.mark.gpu
def test_noalloc_permute_allocates_nothing(cuda):
    T, k, E = 8192, 2, 64
    rng = np.random.default_rng(7)
    idx = torch.from_numpy(rng.integers(0, E, (T, k)).astype(np.int32)).to(cuda)
    off, pos, src = _buffers(T, k, E, cuda)
    _call_noalloc(idx, E, off, pos, src)     # warm-up: the one-time set-up
    torch.cuda.synchronize()
    torch_before = torch.cuda.memory_allocated(cuda)
    free_before, _ = torch.cuda.mem_get_info(cuda)
    for _ in range(3):
        _call_noalloc(idx, E, off, pos, src)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(cuda)
    assert torch.cuda.memory_allocated(cuda) == torch_before
    assert free_after == free_before
    assert _noalloc_status() == (_lib.KVM_OK, 0)


@pytest.mark.gpu
def test_noalloc_permute_reports_out_of_range_expert(cuda):
    T, k, E = 300, 2, 16
    rng = np.random.default_rng(11)
    idx_np = rng.integers(0, E, (T, k)).astype(np.int32)
    idx_np[5, 1] = E          # one past the last expert
    idx_np[200, 0] = -1
    idx = torch.from_numpy(idx_np).to(cuda)
    assert _noalloc_status() == (_lib.KVM_OK, 0)
    off, pos, src = _permute(idx, E, noalloc=True)
    rc, word = _noalloc_status(clear=True)
    assert rc == _lib.KVM_ERR_INVALID_ARG and word != 0
    assert _noalloc_status() == (_lib.KVM_OK, 0)     # cleared
    assert pos[5 * k + 1] == -1 and pos[200 * k + 0] == -1
    assert off[E] == T * k - 2
    want = _permute(idx, E, noalloc=False)
    with pytest.raises(_lib.KvmError):                # the workspace path's word
        _lib.device_status()
    assert np.array_equal(off, want[0]) and np.array_equal(pos, want[1])
    assert np.array_equal(src[:off[E]], want[2][:off[E]])


def test_noalloc_permute_rejects_sizes_beyond_the_static_scratch():
    L = _lib.lib()
    # ceil(T*k/256) * E = 1024 * 128 > MAX_CELLS: rejected before any GPU work.
    assert L.kvm_sm100_moe_permute_noalloc(None, 131072, 2, 128, None, None, None,
                                           None) == _lib.KVM_ERR_INVALID_ARG
    assert b"exceeds the static scratch" in L.kvm_sm100_last_error()
    # 257 * 256 = 65792 cells: one chunk past the limit.
    assert _cells(32769, 2, 256) > MAX_CELLS
    assert L.kvm_sm100_moe_permute_noalloc(None, 32769, 2, 256, None, None, None,
                                           None) == _lib.KVM_ERR_INVALID_ARG
    assert b"exceeds the static scratch" in L.kvm_sm100_last_error()
    # Exactly 65536 cells passes the size check (and then stops at the NULL
    # pointers, still before any GPU work).
    assert L.kvm_sm100_moe_permute_noalloc(None, 32768, 2, 256, None, None, None,
                                           None) == _lib.KVM_ERR_INVALID_ARG
    assert b"NULL pointer" in L.kvm_sm100_last_error()
