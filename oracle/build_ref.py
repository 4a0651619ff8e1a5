"""Compile pieces of the reference from its own sources into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  Two reference components build from a few source
files without the reference's build system:

* ``liblocali_core_ref.so`` - the reference slot planner, ``native/locali_core.c``
  compiled with gcc exactly as its Makefile does (``native/Makefile:2``:
  ``-O3 -std=c11 -Wall -Wextra -Werror``, ``-shared -fPIC``).
* ``libref_dsv4.so`` - the reference's CUDA fused 2-bit gate/up + clamped
  SwiGLU kernel body (``dsv4_kernels.py:100-173``), read out of the Python
  source with ``ast`` (the module itself imports mlx and is never executed),
  wrapped in a ``__global__`` signature with the input names and template
  parameters that ``mx.fast.cuda_kernel`` gives it (``dsv4_kernels.py:197-214``,
  ``:276-299``), and compiled for sm_100a for a fixed set of shapes.

Outputs go to ``oracle/_ref/`` only (git-ignored; they travel to the GPU box
with the snapshot).  Nothing is copied into the repository.
"""

from __future__ import annotations

import ast
import os
import shutil
import subprocess
from pathlib import Path

REFERENCE_ROOT = Path(os.environ.get("LOCALI_REFERENCE", "/root/reference"))
OUT = Path(__file__).resolve().parent / "_ref"
CORE_REF = OUT / "liblocali_core_ref.so"
DSV4_REF = OUT / "libref_dsv4.so"

# (K, N, GS, TOP_K, ROUTES, LIMIT) instantiations of the reference kernel
REF_SHAPES = [
    (256, 128, 128, 2, 2, 10),     # reference test geometry (tests/test_dsv4_kernels.py:43-75)
    (1024, 512, 64, 6, 6, 10),     # C0 widths, 2-bit
    (1024, 512, 128, 6, 6, 10),
    (4096, 2048, 64, 6, 6, 10),    # C1 decode
    (4096, 2048, 128, 6, 6, 10),
]


def reference_present() -> bool:
    return (REFERENCE_ROOT / "native" / "locali_core.c").is_file()


def build_core_ref() -> Path | None:
    src = REFERENCE_ROOT / "native" / "locali_core.c"
    if not src.is_file():
        return None
    OUT.mkdir(exist_ok=True)
    cc = shutil.which("gcc") or shutil.which("cc")
    subprocess.run([cc, "-O3", "-std=c11", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC", str(src), "-o",
                    str(CORE_REF)], check=True)
    return CORE_REF


def _cuda_body() -> str:
    src = (REFERENCE_ROOT / "dsv4_kernels.py").read_text()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "_CUDA_SOURCE" for t in node.targets):
            return ast.literal_eval(node.value)
    raise RuntimeError("reference _CUDA_SOURCE not found")


def _wrapper(body: str) -> str:
    inst = []
    for K, N, GS, TK, R, L in REF_SHAPES:
        for tname, suffix in (("__nv_bfloat16", 0), ("__half", 1)):
            inst.append(
                f"  if (K=={K} && N=={N} && GS=={GS} && top_k=={TK} && routes=={R} && limit=={L} && f16=={suffix}) {{\n"
                f"    ref_affine2_swiglu<{tname},{K}u,{N}u,{GS}u,{TK}u,{R}u,{L}><<<dim3(1, {R}*({N}/8), 1), dim3(32, 2, 1), 0, st>>>(\n"
                f"      (const {tname}*)input, indices, wu, (const {tname}*)su, (const {tname}*)bu, wg,\n"
                f"      (const {tname}*)sg, (const {tname}*)bg, ({tname}*)output);\n"
                f"    return (int)cudaGetLastError();\n  }}\n")
    return (
        "#include <cuda_bf16.h>\n#include <cuda_fp16.h>\n#include <cstdint>\n"
        "template <typename T, unsigned K, unsigned N, unsigned GS, unsigned TOP_K, unsigned ROUTES, int LIMIT>\n"
        "__global__ void ref_affine2_swiglu(const T* input, const uint32_t* indices, const uint32_t* weight_up,\n"
        "    const T* scales_up, const T* biases_up, const uint32_t* weight_gate, const T* scales_gate,\n"
        "    const T* biases_gate, T* output) {\n" + body + "\n}\n"
        "extern \"C\" int ref_affine2_swiglu_launch(int K, int N, int GS, int top_k, int routes, int limit, int f16,\n"
        "    const void* input, const uint32_t* indices, const uint32_t* wu, const void* su, const void* bu,\n"
        "    const uint32_t* wg, const void* sg, const void* bg, void* output, void* stream) {\n"
        "  cudaStream_t st = (cudaStream_t)stream;\n" + "".join(inst) + "  return -2;\n}\n"
    )


def build_dsv4_ref() -> Path | None:
    if not (REFERENCE_ROOT / "dsv4_kernels.py").is_file():
        return None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    OUT.mkdir(exist_ok=True)
    cu = OUT / "ref_dsv4_fused.cu"
    cu.write_text(_wrapper(_cuda_body()))
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                    "-shared", str(cu), "-o", str(DSV4_REF)], check=True,
                   stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    return DSV4_REF


def build_all() -> list[Path]:
    out = []
    for fn in (build_core_ref, build_dsv4_ref):
        p = fn()
        if p is not None:
            out.append(p)
    return out


if __name__ == "__main__":
    for p in build_all():
        print("built", p)
