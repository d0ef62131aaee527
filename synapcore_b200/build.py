"""Build libsckv.so (CUDA kernels for sm_100a + host C++), in-tree.

    python -m synapcore_b200.build [--force] [--verbose]

The shared library lands in synapcore_b200/_lib/libsckv.so next to the
sources so it travels with the checkout; nothing is installed elsewhere.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libsckv.so"
OBJ_DIR = LIB_DIR / "obj"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "--extended-lambda",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libsckv.so")
    return cand


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    if src.stat().st_mtime > t:
        return True
    return any(h.stat().st_mtime > t for h in _headers())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every source for sm_100a and link libsckv.so. Returns its path."""
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    changed = force or not LIB_PATH.exists()
    for src in sources():
        obj = OBJ_DIR / (src.name + ".o")
        objs.append(obj)
        if not force and not _stale(obj, src):
            continue
        changed = True
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if ptxas_verbose and src.suffix == ".cu":
            cmd += ["-Xptxas", "-v"]
        if src.suffix == ".cpp":
            # host-only C++: no device code, so no target architecture to warn about
            cmd = [nvcc, "-O3", "-std=c++17", "-Wno-deprecated-gpu-targets", "-Xcompiler", "-fPIC",
                   "-Xcompiler", "-fvisibility=hidden",
                   "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        if verbose or ptxas_verbose:
            sys.stdout.write(res.stdout + res.stderr)
    if changed:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas))


if __name__ == "__main__":
    main()
