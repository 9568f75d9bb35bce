"""Build libfgb200.so (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

The library is one translation unit (csrc/fgb200.cu includes every
component). The result lands next to this file so it travels with the
source tree; nothing is installed into site-packages. A stamp beside it
holds the SHA-256 of every source and of the compiler flags it was built
from; the library is rebuilt whenever that digest changes (file times are
not trusted: a copied tree can carry a library newer than its sources).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_NAME = "libfgb200.so"
LIB_PATH = PKG_DIR / LIB_NAME
STAMP_PATH = PKG_DIR / (LIB_NAME + ".stamp")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC",
    "-shared",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the fgb200 CUDA library cannot be built")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def source_digest() -> str:
    """SHA-256 over the compiler flags and every source file (path + bytes)."""
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS).encode())
    for p in sources():
        h.update(p.relative_to(PKG_DIR.parent).as_posix().encode())
        h.update(b"\0")
        h.update(p.read_bytes())
    return h.hexdigest()


def needs_rebuild() -> bool:
    if not LIB_PATH.exists() or not STAMP_PATH.exists():
        return True
    return STAMP_PATH.read_text().strip() != source_digest()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/fgb200.cu into fluidgpu_b200/libfgb200.so (sm_100a)."""
    if not force and not needs_rebuild():
        return LIB_PATH
    digest = source_digest()
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp), str(CSRC / "fgb200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose and proc.stderr:
        print(proc.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    STAMP_PATH.write_text(digest + "\n")
    return LIB_PATH


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(out)
