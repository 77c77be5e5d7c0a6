"""Build recipe of the sm_100a shared library ``libgofish_b200.so``.

The library is built in-tree next to this file with nvcc directly (no JIT, no
torch extension machinery), so it travels with the source tree.  The
floating-point flags are part of the parity contract: no implicit FMA
contraction, IEEE division and square root, no flush-to-zero.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
LIBRARY = PACKAGE_DIR / "libgofish_b200.so"
SOURCES = [CSRC / "gf_tracer.cu", CSRC / "gf_sort_static.cu", CSRC / "gf_field.cu", CSRC / "gf_mip.cu",
           CSRC / "gf_shape.cu", CSRC / "gf_sites.cu", CSRC / "gf_mesh.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [PACKAGE_DIR.parent / "include" / "gofish_b200.h"]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-fmad=false",
    "-prec-div=true",
    "-prec-sqrt=true",
    "-ftz=false",
    "-Xcompiler", "-fPIC",
    "-shared",
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def needs_build() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources."""
    if not force and not needs_build():
        return LIBRARY
    cmd = [nvcc(), *NVCC_FLAGS, *map(str, SOURCES), "-o", str(LIBRARY)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIBRARY


if __name__ == "__main__":
    build(force=True, verbose=True)
