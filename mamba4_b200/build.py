"""Build the in-tree CUDA shared library `libmamba4_b200.so` for sm_100a.

One nvcc invocation per translation unit, linked into a single shared
library next to this file (it travels with the source tree; nothing is
installed). The CUDA runtime is linked statically so the library depends
only on the driver.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
LIB = HERE / "libmamba4_b200.so"
SOURCES = ["abi.cu", "memread.cu", "scan.cu", "glue.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")
    return path


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = list(SRC.glob("*.cu")) + list(SRC.glob("*.cuh")) + [HERE.parent / "include" / "mamba4_b200.h"]
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu for sm_100a and link libmamba4_b200.so (in-tree)."""
    if not force and not stale():
        return LIB
    obj_dir = HERE / "_build"
    obj_dir.mkdir(exist_ok=True)
    objects, procs = [], []
    # The translation units compile in parallel (one nvcc process each).
    for name in SOURCES:
        obj = obj_dir / (Path(name).stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(SRC / name), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd)))
        objects.append(str(obj))
    failed = [cmd for cmd, proc in procs if proc.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objects], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
