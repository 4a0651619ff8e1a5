"""Build the native libraries of locali_b200 in-tree.

* ``locali_b200/liblmoe.so``        - sm_100a routed-MoE kernels (nvcc)
* ``locali_b200/liblocali_core.so`` - slot-residency planner (g++)

Run ``python -m locali_b200.csrc.build`` (or ``__graft_entry__.build()``).
Outputs are rebuilt only when a source is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Wno-deprecated-gpu-targets"]

LMOE_SOURCES = ["lmoe_route.cu", "lmoe_gemv.cu", "lmoe_stream.cu", "lmoe_vec.cu", "lmoe_prefill.cu", "lmoe_ep.cu", "lmoe_api.cu"]
LMOE_DEPS = LMOE_SOURCES + ["lmoe_common.cuh", "lmoe_kernels.cuh"]
LMOE_LIB = PKG / "liblmoe.so"
CORE_LIB = PKG / "liblocali_core.so"


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build liblmoe.so")
    return cand


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (exit {proc.returncode})")


def build_lmoe(force: bool = False, verbose: bool = False) -> Path:
    deps = [CSRC / s for s in LMOE_DEPS] + [INCLUDE / "lmoe.h"]
    if not force and not _stale(LMOE_LIB, deps):
        return LMOE_LIB
    nvcc = _nvcc()
    objdir = CSRC / "_build"
    objdir.mkdir(exist_ok=True)
    headers = [CSRC / s for s in LMOE_DEPS if s.endswith(".cuh")] + [INCLUDE / "lmoe.h", Path(__file__)]
    objs = []
    for src in LMOE_SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        if force or verbose or _stale(obj, [CSRC / src, *headers]):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(CSRC / src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd)
        objs.append(str(obj))
    tmp = LMOE_LIB.with_suffix(".so.tmp")
    _run([nvcc, *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart"])
    os.replace(tmp, LMOE_LIB)
    return LMOE_LIB


def build_core(force: bool = False) -> Path:
    src = CSRC / "locali_core.cpp"
    deps = [src, INCLUDE / "locali_core.h"]
    if not force and not _stale(CORE_LIB, deps):
        return CORE_LIB
    cxx = shutil.which("g++") or "c++"
    tmp = CORE_LIB.with_suffix(".so.tmp")
    _run([cxx, "-O3", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC", str(src), "-o", str(tmp)])
    os.replace(tmp, CORE_LIB)
    return CORE_LIB


def build_all(force: bool = False) -> None:
    build_core(force)
    build_lmoe(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(f"built {LMOE_LIB} and {CORE_LIB}")
