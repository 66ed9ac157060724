"""Build libgs3d.so (all CUDA sources under ../csrc) for sm_100a, in-tree.

Every translation unit except bwd_raster.cu (FILE_FLAGS) is compiled with ``-fmad=false``:
floating-point contraction is written explicitly (``fmaf``) where wanted, so results are
reproducible by the CPU oracle.
Objects are rebuilt only when their source or a header is newer. Usage:

    python -m gs3d.build            (from threedgaussiansplatting.jl_b200/)
    python threedgaussiansplatting.jl_b200/gs3d/build.py
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR.parent / "csrc"
INCLUDE = PKG_DIR.parent.parent / "include"
BUILD_DIR = PKG_DIR.parent / "_build"
LIB_PATH = PKG_DIR / "libgs3d.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-fmad=false", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-O2", "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


# Per-file exceptions to the numerics flags. bwd_raster.cu (the backward blend: float-atomic
# gradient sums, compared within a tolerance) allows floating-point contraction; its decision
# of which (pixel, Gaussian) pairs to take does not depend on it (see the file).
FILE_FLAGS = {"bwd_raster.cu": {"-fmad=false": "-fmad=true"}}


def _flags(src: Path) -> list[str]:
    sub = FILE_FLAGS.get(src.name, {})
    return [sub.get(f, f) for f in NVCC_FLAGS]


def _compile(src: Path, obj: Path, verbose_ptxas: bool) -> str:
    cmd = [nvcc(), *ARCH_FLAGS, *_flags(src), "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    todo = []
    objs = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            todo.append((src, obj))
    logs = {}
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, verbose_ptxas): s for s, o in todo}
            for fut in cf.as_completed(futs):
                logs[futs[fut].name] = fut.result()
    if todo or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    if verbose_ptxas:
        for name, log in sorted(logs.items()):
            print(f"== {name}\n{log}")
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
    print(LIB_PATH)
