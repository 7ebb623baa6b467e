"""Build libkvm_sm100.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m kvm_b200.build [--force]

Every ``kvm_b200/csrc/*.cu`` is compiled for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) into ``kvm_b200/_build/*.o``
and linked into ``kvm_b200/libkvm_sm100.so``. A translation unit is rebuilt
when its source or any header it can include changed. nvcc cross-compiles, so
this runs on a machine without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_build"
LIB = PKG / "libkvm_sm100.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wall", "--expt-relaxed-constexpr",
    f"-I{ROOT / 'include'}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required")
    return cand


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) +
                  list((ROOT / "include").glob("*.h")))


def _digest(src: Path) -> str:
    h = hashlib.sha256()
    for p in [src] + _headers():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    return h.hexdigest()


def _compile(src: Path, force: bool) -> Path:
    obj = OUT_DIR / (src.stem + ".o")
    stamp = OUT_DIR / (src.stem + ".sha")
    dig = _digest(src)
    if not force and obj.exists() and stamp.exists() and stamp.read_text() == dig:
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    stamp.write_text(dig)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), sources))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", "-Xcompiler", "-fPIC",
               *[str(o) for o in objs], "-o", str(tmp)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    build(force=args.force, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
