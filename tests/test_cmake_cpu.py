"""The CMake build of the C++ host side (kvm_b200/host/CMakeLists.txt), on CPU:
configure against the reference tree the host build used, build the front
end, the sm_100a Device target, kvm_run and the reference's own tests (linked
against the in-tree libkvm_sm100.so), then run them through ctest."""
import os
import shutil
import subprocess

import pytest

from kvm_b200.host import build_host

HOST_SRC = build_host.HERE


def _reference():
    d = os.environ.get("KVM_REFERENCE_DIR")
    if d and os.path.exists(os.path.join(d, "src", "ir", "graph.cpp")):
        return d
    r = build_host.recorded_ref_dir()
    return str(r) if r else None


def test_cmake_builds_and_runs_the_host_side(tmp_path):
    ref = _reference()
    if ref is None:
        pytest.skip("no reference tree (set KVM_REFERENCE_DIR or run the host build)")
    if shutil.which("cmake") is None:
        pytest.skip("cmake unavailable")
    lib = build_host.PKG / "libkvm_sm100.so"
    if not lib.exists():
        pytest.skip("libkvm_sm100.so not built")
    gen = ["-G", "Ninja"] if shutil.which("ninja") else []
    b = tmp_path / "build"
    r = subprocess.run(["cmake", "-S", str(HOST_SRC), "-B", str(b), *gen,
                        f"-DKVM_REFERENCE_DIR={ref}", f"-DKVM_SM100_LIB={lib}"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    r = subprocess.run(["cmake", "--build", str(b), "-j", str(os.cpu_count() or 4)],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    r = subprocess.run(["ctest", "--output-on-failure"], cwd=b, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "100% tests passed" in r.stdout
    assert (b / "kvm_run").exists()
