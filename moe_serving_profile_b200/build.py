"""Build the sm_100a shared library ``libb200moe.so`` next to this file.

nvcc compiles every kernel for ``sm_100a`` only (no PTX fallback, no other
architecture). The library links the CUDA runtime statically and exports the
C ABI declared in ``include/b200moe.h``. Run ``python -m
moe_serving_profile_b200.build`` or call :func:`build`.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libb200moe.so"
SOURCES = ["api.cu", "router.cu", "permute.cu", "gemm.cu", "decode.cu", "combine.cu", "a2a.cu", "a2a_p2p.cu", "p2p.cu", "w8a8.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(cuda) / "bin" / "nvcc")


def _stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh"))
    deps.append(INCLUDE / "b200moe.h")
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it; return its path."""
    if not force and not _stale():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [
            nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
            "-Xptxas", "-v" if verbose else "-O3",
            "-I", str(INCLUDE), "-I", str(CSRC),
            "-c", str(CSRC / src), "-o", str(obj),
        ]
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart_static", "-lrt",
                    "-lpthread", "-ldl"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
