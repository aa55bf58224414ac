"""Builds the native library ``lib/libv7_threading.so`` in-tree.

The library holds the sm_100a kernels (``csrc/*.cu``), the batched C-ABI
(``include/v7g.h``) and the reference-compatible ms_abi export surface
(``include/v7_threading.h``).  Kernels are compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); the CUDA runtime is linked
statically so the file has no dependency beyond the driver.  The exported
symbol set is fixed by a linker version script: the 99 names the reference's
loader resolves (src/v7_lib.h:585-739) plus the ``v7g_*`` entries.

Run ``python -m v7multiplikator_b200.build`` (or ``build()`` from Python).
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libv7_threading.so"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: the reference rounds every product that it does not fuse
# explicitly, and the kernels spell each intended fused multiply-add as one
# (fp.cuh, arith.cuh); the compiler must not contract anything else.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills"] + ARCH
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-parameter", f"-I{CUDA_HOME / 'include'}"]

KERNEL_SOURCES = ["runtime.cu", "norm.cu", "norm_q8.cu", "rope.cu", "rope_only.cu", "rope_tables.cu", "swiglu.cu", "add.cu",
                  "gemv.cu", "noalloc.cu", "selftest.cu"]
# Units whose kernels the reference runs with MXCSR FTZ+DAZ and that use the
# packed-pair intrinsics, whose denormal mode follows -ftz (csrc/arith.cuh).
# Explicit-PTX arithmetic elsewhere carries its own .ftz or not.
FTZ_SOURCES = {"norm_q8.cu", "swiglu.cu", "gemv.cu", "selftest.cu"}
HOST_SOURCES = ["abi.cpp", "rope_freqs.cpp"]
HEADERS = ["fp.cuh", "arith.cuh", "reduce.cuh", "q8.cuh", "q8_fast.cuh", "internal.h", "launch.cuh", "pipeline.cuh", "rowpipe.cuh"]


def exported_names() -> list[str]:
    """Every symbol the library exports: the hot-path, runtime and stub names
    of include/v7_threading*.h and the v7g_* entries of include/v7g.h."""
    inc = ROOT / "include"
    names: list[str] = []
    drop_in = (inc / "v7_threading.h").read_text()
    names += re.findall(r"V7_ABI\s+[\w\s\*]*?\b(\w+)\s*\(", drop_in)
    names += re.findall(r"extern int (\w+);", drop_in)
    stubs = (inc / "v7_threading_stubs.h").read_text()
    void_part = stubs[stubs.index("#define V7G_STUBS_VOID"):stubs.index("#define V7G_STUBS_RET")]
    ret_part = stubs[stubs.index("#define V7G_STUBS_RET"):stubs.index("#define V7G_DECLARE_VOID")]
    names += re.findall(r"^\s*X\((\w+),", void_part, flags=re.M)
    names += re.findall(r"^\s*X\([^,]+,\s*(\w+),", ret_part, flags=re.M)
    names += re.findall(r"\b(v7g_\w+)\s*\(", (inc / "v7g.h").read_text())
    seen: list[str] = []
    for n in names:
        if n not in seen and not n.startswith("__"):
            seen.append(n)
    return seen


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + sorted((ROOT / "include").glob("*.h"))
    objs: list[Path] = []
    for src in KERNEL_SOURCES:
        obj = BUILD / (src + ".o")
        if force or _stale(obj, [CSRC / src] + headers):
            ftz = ["-ftz=true", "-DV7G_FTZ_TU"] if src in FTZ_SOURCES else ["-ftz=false"]
            _run([NVCC, *NVCC_FLAGS, *ftz, "-c", str(CSRC / src), "-o", str(obj)])
        objs.append(obj)
    for src in HOST_SOURCES:
        obj = BUILD / (src + ".o")
        if force or _stale(obj, [CSRC / src] + headers):
            _run(["g++", *CXX_FLAGS, "-c", str(CSRC / src), "-o", str(obj)])
        objs.append(obj)
    vmap = BUILD / "exports.map"
    names = exported_names()
    vmap.write_text("{\n  global:\n" + "".join(f"    {n};\n" for n in names) + "  local: *;\n};\n")
    if force or _stale(LIB, objs + [vmap]):
        tmp = LIB.with_suffix(".so.tmp")
        _run([NVCC, "-shared", *ARCH, "-o", str(tmp), *map(str, objs),
              "-Xlinker", f"--version-script={vmap}", "-Xlinker", "-soname=libv7_threading.so",
              "-Xlinker", "-z,defs", "-lpthread", "-ldl", "-lrt"])
        shutil.move(str(tmp), str(LIB))
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
