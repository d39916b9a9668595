"""Builds libunified_fpn_b200.so (all CUDA kernels + engine + C ABI) for sm_100a.

Incremental: an object is rebuilt when its source or any header under csrc/ or
include/ is newer.  Output goes next to the Python package so the library
travels with the source tree:

    -unifiedfpn_b200/unified_fpn/libunified_fpn_b200.so

Usage: python build.py [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
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
LIB = PKG / "unified_fpn" / "libunified_fpn_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]
SOURCES = ["tc_kernels.cu", "simt_kernels.cu", "backward.cu", "engine.cu", "capi.cpp", "noalloc.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers_mtime() -> float:
    m = 0.0
    for d in (CSRC, INCLUDE):
        for p in d.rglob("*"):
            if p.suffix in (".h", ".cuh", ".hpp"):
                m = max(m, p.stat().st_mtime)
    return m


def _compile(src: Path, obj: Path) -> tuple[Path, str]:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd[1:1] = ["-x", "cu"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, jobs: int = 4, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    todo = []
    objs = []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
            for obj, err in ex.map(lambda t: _compile(*t), todo):
                if verbose and err.strip():
                    print(err, file=sys.stderr)
    if force or todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=4)
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.jobs, verbose=True))
