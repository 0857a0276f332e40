"""Build librolaq_b200.so in-tree with nvcc for sm_100a.

    python -m mla_kv_quant_b200.build [--verbose]

The shared library lands in ``mla_kv_quant_b200/_lib/`` next to the package, so it
travels with a copy of the repository.  Objects are rebuilt when a source or header
is newer than the library.
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
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "librolaq_b200.so"
SOURCES = ["abi.cu", "writer.cu", "codec.cu", "decode.cu", "decode_tc.cu", "proj.cu", "window.cu", "peer.cu"]
HEADERS = ["common.cuh", "kernels.cuh", "merge.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA 12.8+ toolkit is required to build librolaq_b200.so")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [ROOT / "include" / "rolaq_b200.h"]
    objs = []
    flags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", *ARCH]
    if verbose:
        flags += ["-Xptxas", "-v"]
    for src in SOURCES:
        obj = OUT_DIR / (Path(src).stem + ".o")
        objs.append(obj)
        if force or verbose or _stale(obj, [CSRC / src, *headers]):
            cmd = [nvcc(), *flags, "-c", str(CSRC / src), "-o", str(obj)]
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-ldl", "-lrt",
               "-lpthread"]
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose", action="store_true", help="pass -Xptxas -v (registers, spills)")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    print(build(verbose=args.verbose, force=args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
