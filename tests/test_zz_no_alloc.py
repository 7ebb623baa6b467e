"""The allocation-free permute entry point (kvm_sm100_moe_permute_noalloc).

Callers that cannot allocate GPU memory while routing -- a host program that
owns all device buffers through its own pool, or a serving loop that must not
call cudaMalloc/cudaFree because they synchronise the device -- use this entry
point; its scratch is a fixed static device array instead of a workspace.

The GPU test calls it through the C ABI twice in a row (the second call sees
the first call's leftovers in the shared array) and compares every output
with the workspace-based kvm_sm100_moe_permute, bit for bit (permutation work
is integer work). It sits in its own file, collected last.
"""
import numpy as np
import pytest
import torch

from kvm_b200 import _lib

MAX_CELLS = 65536


def _permute(idx: torch.Tensor, E: int, noalloc: bool):
    T, k = idx.shape
    dev = idx.device
    off = torch.full((E + 1,), -7, dtype=torch.int32, device=dev)
    pos = torch.full((T * k,), -7, dtype=torch.int32, device=dev)
    src = torch.full((T * k,), -7, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    if noalloc:
        _lib.call("kvm_sm100_moe_permute_noalloc", idx.data_ptr(), T, k, E,
                  off.data_ptr(), pos.data_ptr(), src.data_ptr(), st)
    else:
        nbytes = int(_lib.lib().kvm_sm100_moe_permute_workspace(T, k, E))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _lib.call("kvm_sm100_moe_permute", idx.data_ptr(), T, k, E, off.data_ptr(),
                  pos.data_ptr(), src.data_ptr(), ws.data_ptr(), st)
    torch.cuda.synchronize()
    return off.cpu().numpy(), pos.cpu().numpy(), src.cpu().numpy()


@pytest.mark.gpu
def test_noalloc_permute_matches_workspace_permute(cuda):
    rng = np.random.default_rng(123)
    # Two calls in a row; the first is the larger, so the second runs on a
    # scratch array still holding the first call's counts and bases.
    for T, k, E in [(8192, 2, 64), (1000, 3, 40)]:
        idx = torch.from_numpy(rng.integers(0, E, (T, k)).astype(np.int32)).to(cuda)
        want = _permute(idx, E, noalloc=False)
        got = _permute(idx, E, noalloc=True)
        for a, b in zip(got, want):
            assert np.array_equal(a, b)
    _lib.device_status()


def test_noalloc_permute_rejects_sizes_beyond_the_static_scratch():
    # ceil(T*k/256) * E = 1024 * 128 > MAX_CELLS: rejected before any GPU work.
    rc = _lib.lib().kvm_sm100_moe_permute_noalloc(None, 131072, 2, 128, None, None,
                                                  None, None)
    assert rc == _lib.KVM_ERR_INVALID_ARG
    assert b"exceeds the static scratch" in _lib.lib().kvm_sm100_last_error()
