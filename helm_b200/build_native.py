"""Builds libhelm_b200.so (the C-ABI library) from helm_b200/csrc/*.cu.

The library is compiled for sm_100a only and written in-tree to
helm_b200/lib/libhelm_b200.so, so that it travels with the source tree to the
GPU host.  Run ``python -m helm_b200.build_native`` or call :func:`build`.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libhelm_b200.so"
SOURCES = ["common.cu", "paged_attn.cu", "int8_linear.cu", "kv_append.cu", "kv_prefill.cu", "gather_merge.cu", "norm.cu",
           "page_copy.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3",
    "-cudart", "shared",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the helm_b200 CUDA library cannot be built")
    return cand


def _stale(sources, target: pathlib.Path) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    deps = list(sources) + list(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "helm_b200.h",
                                                         pathlib.Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> pathlib.Path:
    """Compile every kernel source into one shared library (sm_100a)."""
    srcs = [CSRC / s for s in SOURCES]
    if not force and not _stale(srcs, LIB):
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    objdir = PKG / "lib" / "obj"
    objdir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs = []
    for src in srcs:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0 or verbose or ptxas_verbose:
            sys.stderr.write(res.stdout + res.stderr)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}")
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "shared",
           "-Xlinker", "-rpath,/usr/local/cuda/lib64", *objs, "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc link of libhelm_b200.so failed")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build(force=force, verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv))
