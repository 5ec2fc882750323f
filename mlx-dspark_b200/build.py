"""Build libdspark.so (the C-ABI CUDA library) in-tree for sm_100a.

``python mlx-dspark_b200/build.py`` compiles every ``csrc/*.cu`` with nvcc (in parallel) and
links ``mlx-dspark_b200/libdspark.so``. Objects go to ``mlx-dspark_b200/_build/`` and are
reused when a source (and no header) is unchanged.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libdspark.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-I", str(CSRC), "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the dspark CUDA library cannot be built")


def _newest_header() -> float:
    hs = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _newest_header()):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if os.environ.get("DSPARK_PTXAS_V"):
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if os.environ.get("DSPARK_PTXAS_V") and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 4))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
           "-lcuda" if False else "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
