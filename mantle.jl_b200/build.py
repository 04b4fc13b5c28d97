"""Build libmantle_cuda.so in-tree for sm_100a.

    python mantle.jl_b200/build.py            # incremental
    python mantle.jl_b200/build.py --force    # rebuild everything

Every translation unit is compiled by nvcc with
`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`, then linked into one
shared library with the CUDA runtime linked statically, so the library does not
depend on which libcudart another package in the process loaded.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OUT = HERE / "mantle_cuda" / "libmantle_cuda.so"
OBJ = HERE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")) + list(CSRC.glob("kernels/*.cu")))


def headers() -> list[Path]:
    return sorted(list(CSRC.rglob("*.hpp")) + list(CSRC.rglob("*.cuh")) + [ROOT / "include" / "mantle_cuda.h"])


# Flags for single translation units. showcase.cu and mesh_raster.cu: no FMA
# contraction, so their float arithmetic is the sequence of IEEE operations the
# C oracle performs.
PER_FILE = {"showcase.cu": ["-fmad=false"], "mesh_raster.cu": ["-fmad=false"]}


def compile_one(src: Path, force: bool) -> Path:
    obj = OBJ / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [nvcc(), *ARCH, *COMMON, *PER_FILE.get(src.name, []), "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), *COMMON, "-x", "c++", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not OUT.exists() or OUT.stat().st_mtime < newest:
        # --no-undefined: a symbol missing from the library fails the build, not the first load
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-Xlinker", "--no-undefined", "-o", str(OUT),
               *map(str, objs), "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    try:
        build(force=args.force, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
