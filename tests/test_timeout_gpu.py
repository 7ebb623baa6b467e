"""Failure detection without a GPU fault: a device-side wait on a flag that
nothing sets runs out after its bound (2 s), the kernel returns, the host
reads KVM_ERR_TIMEOUT from the status word, and the context stays usable."""
import ctypes as C
import time

import numpy as np
import pytest
import torch

from kvm_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_unset_flag_times_out_and_context_survives(cuda):
    L = _lib.lib()
    bufs = []
    for nbytes in (16 * 128 * 2, 16 * 128 * 2, 4 * 8, 3 * 4):   # recv, y, cnt, flags
        p = C.c_void_p()
        _lib.call("kvm_sm100_ipc_alloc", nbytes, C.byref(p))
        bufs.append(p.value)
    peers = _lib.EpPeers()
    peers.rank, peers.world, peers.E, peers.H, peers.k = 0, 1, 8, 128, 1
    peers.recv[0], peers.y[0], peers.cnt[0], peers.flags[0] = bufs
    _lib.device_status()                      # start from a clean status word
    t0 = time.time()
    # epoch 7 was never signalled: the wait gives up after its bound
    _lib.call("kvm_sm100_ep_wait", C.byref(peers), 1, 7, None)
    with pytest.raises(_lib.KvmError) as ei:
        _lib.device_status()
    assert ei.value.code == _lib.KVM_ERR_TIMEOUT
    assert 1.5 < time.time() - t0 < 30
    # the status word was cleared and the context still runs work correctly
    assert _lib.device_status() == 0
    a = torch.randn((256, 256), device=cuda).to(torch.bfloat16)
    b = torch.randn((256, 256), device=cuda).to(torch.bfloat16)
    d = ops.matmul(a, b)
    ref = (a.float() @ b.float())
    assert torch.allclose(d.float(), ref, rtol=2e-2, atol=2e-1)
    for p in bufs:
        _lib.call("kvm_sm100_ipc_free", p)
