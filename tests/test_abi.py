"""The C-ABI library loads, exports every symbol include/kvm_sm100.h declares,
and rejects bad arguments before touching a GPU (runs on CPU)."""
import ctypes as C
from pathlib import Path

import pytest

from kvm_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    declared = _lib.header_symbols()
    assert declared, "no kvm_sm100_* declarations found in the header"
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_signatures_cover_header():
    assert sorted(_lib.SIGNATURES) == _lib.header_symbols()


def test_abi_version():
    assert _lib.lib().kvm_sm100_version() == 1


def test_invalid_shapes_rejected_without_gpu():
    L = _lib.lib()
    null = None
    rc = L.kvm_sm100_gemm_bf16(null, 0, null, 0, 0, null, null, 0, 0, 0, 0, 0, null)
    assert rc == _lib.KVM_ERR_INVALID_ARG
    assert b"positive" in L.kvm_sm100_last_error()
    # E = 300 experts: beyond the router's 256 (the permute takes up to 1024)
    rc = L.kvm_sm100_moe_router_topk(null, null, null, null, null, 16, 64, 300, 2, null)
    assert rc == _lib.KVM_ERR_UNSUPPORTED
    # E = 96 passes the expert bound and stops at the NULL pointers
    rc = L.kvm_sm100_moe_router_topk(null, null, null, null, null, 16, 64, 96, 2, null)
    assert rc == _lib.KVM_ERR_INVALID_ARG
    rc = L.kvm_sm100_moe_permute(null, 4, 9, 64, null, null, null, null, null)
    assert rc == _lib.KVM_ERR_INVALID_ARG
    rc = L.kvm_sm100_rmsnorm_bf16(null, null, null, 4, 12, C.c_float(1e-5), null)
    assert rc == _lib.KVM_ERR_INVALID_ARG
    rc = L.kvm_sm100_pack_gate_up(null, null, null, 1, 100, 64, 0, null)
    assert rc == _lib.KVM_ERR_INVALID_ARG


def test_call_raises_kvm_error():
    with pytest.raises(_lib.KvmError) as ei:
        _lib.call("kvm_sm100_silu_mul_bf16", None, None, None, 7, None)
    assert ei.value.code == _lib.KVM_ERR_INVALID_ARG


def test_permute_workspace_size():
    L = _lib.lib()
    # 8192 tokens x top-2 = 64 chunks of 256 pairs; counts + bases of 64 experts.
    assert L.kvm_sm100_moe_permute_workspace(8192, 2, 64) == 2 * 64 * 64 * 4


def test_permute_launch_count():
    """The permutation folds its scan into the rank kernel (2 launches) while
    the per-block count matrix has at most 16 K cells, else 3."""
    from kvm_b200.moe import permute_launches
    assert permute_launches(8192 * 2, 64) == 2          # 64 x 64 cells
    assert permute_launches(256 * 256, 64) == 2         # exactly 16 K cells
    assert permute_launches(256 * 256 + 1, 64) == 3
    assert permute_launches(40000 * 2, 64) == 3


def test_product_code_never_imports_the_oracle():
    offenders = []
    for p in (ROOT / "kvm_b200").rglob("*"):
        if p.suffix in (".py", ".cu", ".cuh", ".h", ".cpp") and p.is_file():
            text = p.read_text(errors="ignore")
            if "import oracle" in text or "from oracle" in text or "liboracle" in text:
                offenders.append(str(p))
    assert not offenders, offenders


def test_kernels_built_for_sm100a_only():
    """Every translation unit and the link step get exactly one -gencode,
    sm_100a cubins with no PTX to JIT elsewhere (the GPU test below reads the
    binary version the device actually runs)."""
    from kvm_b200 import build as kbuild
    assert kbuild.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    flags = " ".join(kbuild.NVCC_FLAGS)
    assert "-gencode" not in flags and "-arch" not in flags


@pytest.mark.gpu
def test_device_runs_the_sm100_cubins(cuda):
    v = C.c_int(0)
    _lib.call("kvm_sm100_kernel_binary_version", C.byref(v))
    assert v.value == 100


def test_fp8_workspace_plan():
    """The FP8 GEMM's workspace query (host-side plan, no GPU needed, 148 SMs
    assumed without a device): the swapped form (M <= 64) splits K blocks
    stream-K and needs two fp32 partial tiles per CTA when tiles are cut; the
    128-row form with tiles enough for every SM takes whole tiles and needs
    none; tiles fewer than SMs are split (partials again)."""
    L = _lib.lib()
    part = 2 * 128 * 128 * 4
    assert L.kvm_sm100_gemm_fp8_workspace(16, 28672, 8192) == 148 * part
    assert L.kvm_sm100_gemm_fp8_workspace(128, 28672, 8192) == 0
    assert L.kvm_sm100_gemm_fp8_workspace(1024, 28672, 8192) == 0
    assert L.kvm_sm100_gemm_fp8_workspace(128, 1024, 2048) > 0   # 8 tiles on 148 SMs
    assert L.kvm_sm100_gemm_fp8_workspace(16, 128, 128) == 0      # one block: nothing to cut
    assert L.kvm_sm100_gemm_fp8_workspace(16, 100, 128) == 0      # N % 128 != 0: invalid
