"""Build the C-ABI shared library ``eraserdit_b200/liberaserdit_b200.so``.

nvcc cross-compiles for sm_100a only; no GPU is needed to build.  The library
links the CUDA runtime statically and resolves the driver's tensor-map encoder
at run time, so it loads next to any PyTorch build in the same process.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PACKAGE = CSRC.parent
REPO = PACKAGE.parent
LIBRARY = PACKAGE / "liberaserdit_b200.so"
SOURCES = ["host_common.cu", "prologue.cu", "attention_bf16.cu", "attention_fp8.cu",
           "attention_fp8_static.cu", "tokens.cu", "peer.cu", "quant.cu", "linear.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the CUDA library cannot be built")


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [
        REPO / "include" / "eraserdit_b200.h", Path(__file__)]
    if (not force and LIBRARY.exists()
            and LIBRARY.stat().st_mtime >= max(d.stat().st_mtime for d in deps)):
        return LIBRARY
    build_dir = REPO / "_build"
    build_dir.mkdir(exist_ok=True)
    objects = []
    for src in srcs:
        obj = build_dir / (src.stem + ".o")
        cmd = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
               "-I", str(REPO / "include"), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIBRARY.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *objects,
                    "-o", str(tmp)], check=True)
    tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
