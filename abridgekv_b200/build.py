"""Build libabkv.so (sm_100a) in-tree with nvcc.

Usage: python -m abridgekv_b200.build [--verbose] [--ptxas-info]

Every CUDA source under csrc/ is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) with -lineinfo; host C++ sources are
compiled by nvcc's host compiler.  Objects go to _build/ and the shared library
to abridgekv_b200/libabkv.so, which travels with the repository snapshot.
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
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libabkv.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}"]
CUDA_FLAGS = ARCH + ["-lineinfo", "--expt-relaxed-constexpr"] + COMMON


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: libabkv.so needs the CUDA 12.9 toolchain")
    return cand


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _digest(paths: list[Path], flags: list[str]) -> str:
    h = hashlib.sha256()
    for p in paths + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h")):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(flags).encode())
    return h.hexdigest()


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    nvcc = _nvcc()
    srcs = _sources()
    flags = CUDA_FLAGS + (["-Xptxas", "-v"] if ptxas_info else [])
    stamp = BUILD / "libabkv.stamp"
    digest = _digest(srcs, flags)
    if LIB.exists() and stamp.exists() and stamp.read_text() == digest and not force and not ptxas_info:
        return LIB
    BUILD.mkdir(exist_ok=True)

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = BUILD / (src.stem + src.suffix.replace(".", "_") + ".o")
        if src.suffix == ".cu":
            cmd = [nvcc] + flags + ["-c", str(src), "-o", str(obj)]
        else:  # host-only C++ (the planner): plain g++
            cmd = [shutil.which("g++") or "g++", "-O3", "-std=c++17", "-fPIC", "-Wall", f"-I{INCLUDE}",
                   f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return obj, (r.stdout + r.stderr)

    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(compile_one, srcs))
    for (obj, log), src in zip(results, srcs):
        if verbose or ptxas_info:
            if log.strip():
                print(f"--- {src.name}\n{log}", file=sys.stderr)
    objs = [str(o) for o, _ in results]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", str(tmp)] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    stamp.write_text(digest)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info, force=a.force))


if __name__ == "__main__":
    main()
