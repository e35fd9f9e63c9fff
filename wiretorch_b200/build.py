"""Compile the engine's CUDA sources into ``wiretorch_b200/_lib/libwiretorch_b200.so``.

    python -m wiretorch_b200.build

sm_100a only (``-gencode arch=compute_100a,code=sm_100a``). The membrane and adjoint
arithmetic is built with ``-fmad=false`` so that every float32 operation rounds on its
own, as the reference's PyTorch expressions do. The library is built in the source
tree, so it travels with the repository to the GPU machine.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).parent
ROOT = HERE.parent
SOURCES = sorted((HERE / "csrc").glob("*.cu"))
HEADERS = sorted((HERE / "csrc").glob("*.cuh")) + [ROOT / "include" / "wiretorch_b200.h"]
OUT_DIR = HERE / "_lib"
LIB = OUT_DIR / "libwiretorch_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC",
         f"-I{ROOT / 'include'}", f"-I{HERE / 'csrc'}"]  # fmt: skip


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build")
    return found


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every source (in parallel) and link the shared library."""
    if not force and not stale():
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    objs, procs = [], []
    for src in SOURCES:
        obj = OUT_DIR / (src.stem + ".o")
        objs.append(obj)
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stdout.write(out.decode())
        if p.returncode:
            failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed on {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)],
                   check=True)  # fmt: skip
    os.replace(tmp, LIB)
    for obj in objs:
        obj.unlink()
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
