"""Build libcrosscache.so in-tree: C host side (gcc), C++ adaptors (g++) and
the sm_100a kernels (nvcc), linked into one shared library next to this file.

    python -m demo_b200.build          # incremental
    python -m demo_b200.build --force  # rebuild everything
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libcrosscache.so"

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

C_SOURCES = [
    "infra/log.c",
    "infra/mempool.c",
    "infra/kvmap.c",
    "infra/threadpool.c",
    "cache/cache.c",
    "cache/disk.c",
]
CXX_SOURCES = [
    "device/device.cpp",
    "device/mem_adaptor.cpp",
]
CU_SOURCES = [
    "device/kv_copy.cu",
    "device/cuda_adaptor.cu",
    "device/block_hash.cu",
    "device/kv_copy_noalloc.cu",
]
HEADERS = sorted(str(p) for p in list(INCLUDE.glob("*.h")) + list(CSRC.rglob("*.h")))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    deps = [src] + [Path(h) for h in HEADERS]
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every source for sm_100a and link libcrosscache.so; returns its path."""
    BUILD.mkdir(exist_ok=True)
    inc = [f"-I{INCLUDE}", f"-I{CSRC}", f"-I{CSRC / 'device'}"]
    objs: list[Path] = []
    for rel in C_SOURCES:
        src = CSRC / rel
        obj = BUILD / (rel.replace("/", "_") + ".o")
        if force or _stale(obj, src):
            _run(["gcc", "-std=gnu11", "-O2", "-g", "-fPIC", "-Wall", "-Wextra",
                  "-Wno-unused-parameter", "-pthread", *inc, "-c", str(src), "-o", str(obj)], verbose)
        objs.append(obj)
    for rel in CXX_SOURCES:
        src = CSRC / rel
        obj = BUILD / (rel.replace("/", "_") + ".o")
        if force or _stale(obj, src):
            _run(["g++", "-std=c++17", "-O2", "-g", "-fPIC", "-Wall", "-Wextra",
                  "-Wno-unused-parameter", "-pthread", "-I/usr/local/cuda/include", *inc,
                  "-c", str(src), "-o", str(obj)], verbose)
        objs.append(obj)
    for rel in CU_SOURCES:
        src = CSRC / rel
        obj = BUILD / (rel.replace("/", "_") + ".o")
        if force or _stale(obj, src):
            cmd = [NVCC, *ARCH, "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-Wall",
                   *inc, "-c", str(src), "-o", str(obj)]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd, verbose or ptxas_info)
        objs.append(obj)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        # --exclude-libs: keep the statically linked CUDA runtime's symbols
        # private, so they never interpose another runtime in the process
        _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs),
              "-Xlinker", "-soname,libcrosscache.so", "-Xlinker", "--exclude-libs,ALL", "-lpthread"], verbose)
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", "-v", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/spill report")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))


if __name__ == "__main__":
    main()
