"""Build the C++ host side: the KVM front end + the sm_100a Device target +
the executor + kvm_run, and the reference's own tests against the sm_100a
target.

    python -m kvm_b200.host.build_host [--ref DIR]

The front end (parser, serializer, graph, kernel/task/tile dialects, the
kernel->task transform) is compiled from the reference's own sources where
they lie (--ref DIR, else $KVM_REFERENCE_DIR; there is no default); nothing is
copied. The tree used is recorded in kvm_b200/_build/host/reference_dir.txt
so that later steps (the CMake build check) find the same one.
Two build-time shims are needed because of this machine's toolchain:
  * glog is not installed: kvm_b200/host/shim/glog/logging.h supplies CHECK;
  * GCC rejects `struct ::kvm::ir::MarkMember<...>` (a global qualifier before
    a class-key, accepted by Clang) in the KVM_MARK_MEMBER macro
    (src/ir/any_of.h:76): each translation unit is preprocessed and that one
    token sequence is rewritten to `struct kvm::ir::MarkMember<...>` in the
    preprocessed output before it is compiled.
The reference's src/device/device.cpp is replaced by kvm_b200/host/
sm100_device.cpp (the sm_100a Device target). Outputs go to
kvm_b200/_build/host/ only. Without the reference sources the build is
skipped and previously built binaries are kept.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
OUT = PKG / "_build" / "host"

FRONTEND = [
    "src/ir/graph.cpp",
    "src/ir/serialization/serializer.cpp",
    "src/ir/serialization/parser.cpp",
    "src/ir/dialect/kernel/values.cpp",
    "src/ir/dialect/kernel/ops.cpp",
    "src/ir/dialect/kernel/dialect.cpp",
    "src/ir/dialect/task/ops.cpp",
    "src/ir/dialect/task/dialect.cpp",
    "src/ir/dialect/tile/ops.cpp",
    "src/ir/dialect/tile/verify.cpp",
    "src/ir/dialect/tile/dialect.cpp",
    "src/transform/kernel_to_task/kernel_to_task.cpp",
]
OURS = ["sm100_device.cpp", "executor.cpp", "task_to_tile.cpp", "kvm_run.cpp"]
REF_TESTS = ["value", "graph", "attr", "serialize", "parse", "kernel_dialect",
             "task_dialect", "tile_dialect", "decomp"]

CXX = os.environ.get("CXX", "g++")
FLAGS = ["-std=c++20", "-O2", "-fPIC", "-Wall", "-Wno-unused-parameter"]
BAD = b"struct ::kvm::ir::MarkMember"
GOOD = b"struct kvm::ir::MarkMember"


def ref_dir(arg: str | None) -> Path | None:
    """The reference tree: the argument, else $KVM_REFERENCE_DIR, else None."""
    d = arg or os.environ.get("KVM_REFERENCE_DIR")
    return Path(d) if d else None


def recorded_ref_dir() -> Path | None:
    """The reference tree the last successful build used, if any."""
    f = OUT / "reference_dir.txt"
    if f.exists():
        d = Path(f.read_text().strip())
        if (d / "src" / "ir" / "graph.cpp").exists():
            return d
    return None


def includes(ref: Path) -> list[str]:
    return [f"-I{ref / 'src'}", f"-I{ref / 'src' / 'ir'}", f"-I{ref / 'tests'}",
            f"-I{HERE / 'shim'}", f"-I{HERE}", f"-I{ROOT / 'include'}",
            "-I/usr/local/cuda/include"]


def compile_one(src: Path, obj: Path, ref: Path) -> Path:
    inc = includes(ref)
    key = hashlib.sha256()
    key.update(src.read_bytes())
    key.update(" ".join(FLAGS + inc).encode())
    for h in list(HERE.glob("*.h")) + [ROOT / "include" / "kvm_sm100.h"]:
        key.update(h.read_bytes())
    stamp = obj.with_suffix(".sha")
    if obj.exists() and stamp.exists() and stamp.read_text() == key.hexdigest():
        return obj
    pre = subprocess.run([CXX, *FLAGS, *inc, "-E", str(src)], capture_output=True)
    if pre.returncode != 0:
        raise RuntimeError(f"preprocess failed: {src}\n{pre.stderr.decode()}")
    ii = obj.with_suffix(".ii")
    ii.write_bytes(pre.stdout.replace(BAD, GOOD))
    r = subprocess.run([CXX, *FLAGS, "-c", str(ii), "-o", str(obj)],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stderr}")
    ii.unlink()
    stamp.write_text(key.hexdigest())
    return obj


def link(out: Path, objs: list[Path], extra: list[str] = ()) -> None:
    r = subprocess.run([CXX, "-o", str(out), *map(str, objs), *extra],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed: {out}\n{r.stderr}")


def cuda_libdirs() -> list[str]:
    dirs = []
    try:
        import nvidia.cuda_runtime as cr  # torch's bundled runtime
        dirs.append(str(Path(cr.__path__[0]) / "lib"))
    except Exception:
        pass
    dirs.append("/usr/local/cuda/lib64")
    return dirs


def build(ref_arg: str | None = None, verbose: bool = False) -> bool:
    ref = ref_dir(ref_arg)
    if ref is None or not (ref / "src" / "ir" / "graph.cpp").exists():
        if verbose:
            print("host build skipped: no reference sources "
                  f"({'set KVM_REFERENCE_DIR or pass --ref' if ref is None else ref})")
        return False
    OUT.mkdir(parents=True, exist_ok=True)
    jobs = [(ref / s, OUT / (s.replace("/", "_")[:-4] + ".o")) for s in FRONTEND]
    jobs += [(HERE / s, OUT / ("kvm_" + s[:-4] + ".o")) for s in OURS]
    jobs += [(ref / "tests" / f"test_{t}.cpp", OUT / f"reftest_{t}.o") for t in REF_TESTS]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda j: compile_one(j[0], j[1], ref), jobs))
    front = [OUT / (s.replace("/", "_")[:-4] + ".o") for s in FRONTEND]
    device = OUT / "kvm_sm100_device.o"
    for t in REF_TESTS:
        link(OUT / f"test_{t}", [OUT / f"reftest_{t}.o", *front, device])
    lib = PKG / "libkvm_sm100.so"
    rpaths = [f"-Wl,-rpath,{PKG}", "-Wl,-rpath,$ORIGIN/../.."]
    libdirs = cuda_libdirs()
    extra = [f"-L{PKG}", "-lkvm_sm100", *[f"-L{d}" for d in libdirs], "-lcudart",
             *rpaths, *[f"-Wl,-rpath,{d}" for d in libdirs]]
    if not lib.exists():
        raise RuntimeError("build libkvm_sm100.so first (python -m kvm_b200.build)")
    link(OUT / "kvm_run", [OUT / "kvm_kvm_run.o", OUT / "kvm_executor.o",
                           OUT / "kvm_task_to_tile.o", device, *front], extra)
    (OUT / "reference_dir.txt").write_text(str(ref.resolve()) + "\n")
    if verbose:
        print(f"built host binaries in {OUT}")
    return True


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--ref", default=None)
    a = ap.parse_args(argv)
    build(a.ref, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
