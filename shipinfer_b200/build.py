"""Build ``libshipk.so`` in-tree with nvcc for sm_100a (B200).

``python -m shipinfer_b200.build`` compiles ``shipinfer_b200/csrc/*.cu`` into
``shipinfer_b200/_lib/libshipk.so``. The library is built in the source tree on purpose: it
travels with the tree to the machine that runs it, and the loader refuses to work without it.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libshipk.so"
SOURCES = ["abi.cu", "letterbox.cu", "crop.cu", "crop_nv12.cu", "nms.cu", "decode.cu", "mask.cu", "selfcheck.cu"]
HEADERS = ["common.cuh", "kernels.h"]
PUBLIC_HEADER = PKG.parent / "include" / "shipk.h"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    # Device float arithmetic is contracted only where a kernel asks for it with __fmaf_rn:
    # the reference formulations depend on which multiply-adds fuse.
    "--fmad=false",
    "-Xcompiler",
    "-fPIC,-ffp-contract=off,-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
    "-cudart",
    "shared",
    "-Xlinker",
    "-rpath,/usr/local/cuda/lib64",
]


def _stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PUBLIC_HEADER, Path(__file__)]
    return any(d.stat().st_mtime > built for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it; return its path."""
    if not force and not _stale():
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, *FLAGS, "-shared", "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
