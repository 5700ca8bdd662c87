"""Builds libgrx.so (the CUDA kernels and the C ABI of include/grx.h) in
place, for sm_100a only.

    python -m gorelaxor_b200.build          # or gorelaxor_b200.build.build()

Every kernel file is compiled with --fmad=false: the kernels reproduce the
reference's float arithmetic operation by operation and fuse a multiply
and an add only where they call __fmaf_rn (see csrc/common.cuh).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libgrx.so"
OBJ = HERE / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC,-O2,-Wall", "-I", str(HERE.parent / "include")]


def _sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _compile(src: Path, extra: list[str]) -> Path:
    obj = OBJ / (src.name + ".o")
    deps = [src] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "grx.h"]
    if obj.exists() and obj.stat().st_mtime > max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> Path:
    """Compiles every source that changed and links libgrx.so."""
    OBJ.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), _sources()))
    if not OUT.exists() or OUT.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(OUT), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
