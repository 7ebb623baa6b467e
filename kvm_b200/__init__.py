"""kvm_b200: B200 (sm_100a) execution backend for KVM kernel/task-dialect graphs.

The compute lives in libkvm_sm100.so (C ABI: include/kvm_sm100.h); this
package is the host-side mirror of the reference's op surface over that ABI.
"""
from . import ops  # noqa: F401
from ._lib import KvmError, lib  # noqa: F401

__all__ = ["ops", "lib", "KvmError"]
