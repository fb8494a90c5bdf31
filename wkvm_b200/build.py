"""Builds libwkvm_b200.so in-tree with nvcc for sm_100a.

The library is a plain C-ABI shared object (no torch types in its
signatures); Python loads it with ctypes. Run ``python -m wkvm_b200.build``
or call :func:`build`.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libwkvm_b200.so"
SOURCES = ["recurrent.cu", "slots.cu", "selftest.cu", "chunk.cu", "gdn_chunk.cu", "gdn_wy.cu",
           "gdn_static.cu", "timemix.cu", "shift_mix.cu", "tma.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu under csrc/ into one shared library (sm_100a)."""
    if not force and not _stale():
        return LIB
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    flags = [
        "-O3", "-std=c++17", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC",
        "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}",
    ]
    if verbose:
        flags += ["-Xptxas", "-v"]
    objs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [_nvcc(), *flags, "-c", str(src), "-o", str(obj)]
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([_nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
