"""Build recipe of the CPU oracle (TEST INFRASTRUCTURE ONLY).

* ``build_oracle()`` compiles this directory's C++ restatement of ThreeDGaussianSplatting.jl
  into ``oracle/_lib/libgs3d_oracle.so`` with ``-ffp-contract=off`` (no fused multiply-add
  unless written ``fmaf``), the numerics contract the CUDA build follows.
* ``build_ref()`` compiles the reference's only native component,
  ``deps/cub_sort_pairs/cub_sort_pairs_wrapper.cu``, from where it lies in the reference
  checkout, with the flags of the reference's ``deps/build.jl:11-29`` (nvcc -std=c++17
  -shared -Xcompiler -fPIC) for sm_100a, into ``oracle/_ref/cub_sort_pairs_wrapper.so``. It
  is used as the sort-parity oracle and the reference sort timing on the GPU box. Nothing
  is copied: when the reference checkout is absent this step is skipped and any
  previously built ``_ref`` library is kept.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
LIB_DIR = ORACLE_DIR / "_lib"
REF_DIR = ORACLE_DIR / "_ref"
ORACLE_LIB = LIB_DIR / "libgs3d_oracle.so"
REF_LIB = REF_DIR / "cub_sort_pairs_wrapper.so"
# the reference checkout: $GS3D_REFERENCE_ROOT, else the directory `reference` beside the repository
REFERENCE_ROOT = Path(os.environ.get("GS3D_REFERENCE_ROOT", ORACLE_DIR.parent.parent / "reference"))
REF_SRC_REL = Path("deps/cub_sort_pairs/cub_sort_pairs_wrapper.cu")


def build_oracle(force: bool = False) -> Path:
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sorted(ORACLE_DIR.glob("*.cpp"))
    deps = srcs + sorted(ORACLE_DIR.glob("*.h")) + [ORACLE_DIR.parent / "include" / "gs3d.h"]
    if not force and ORACLE_LIB.exists() and ORACLE_LIB.stat().st_mtime >= max(p.stat().st_mtime for p in deps):
        return ORACLE_LIB
    tmp = ORACLE_LIB.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           "-pthread", "-o", str(tmp), *map(str, srcs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{' '.join(cmd)}\n{res.stderr}")
    os.replace(tmp, ORACLE_LIB)
    return ORACLE_LIB


def build_ref(force: bool = False) -> Path | None:
    src = REFERENCE_ROOT / REF_SRC_REL
    if not src.exists():
        return REF_LIB if REF_LIB.exists() else None
    if not force and REF_LIB.exists() and REF_LIB.stat().st_mtime >= src.stat().st_mtime:
        return REF_LIB
    REF_DIR.mkdir(exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    tmp = REF_LIB.with_suffix(".so.tmp")
    cmd = [nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared",
           "-Xcompiler", "-fPIC", "-o", str(tmp), str(src)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference sort build failed:\n{' '.join(cmd)}\n{res.stderr}")
    os.replace(tmp, REF_LIB)
    return REF_LIB


if __name__ == "__main__":
    print(build_oracle(force=True))
    print(build_ref(force=True))
