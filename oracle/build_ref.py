"""Compiles the reference's own CPU GEMV (helm/kernels/fp16_gemv.cpp) into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The source is compiled where it lies in the
reference checkout (never copied into this repository); the resulting Python
extension module oracle/_ref/helm_fp16_gemv_ref*.so is git-ignored but travels
with the tree, so the GPU host can time the reference kernel as the CPU
baseline of the INT8 linear without the reference checkout.

Flags follow the reference's own JIT build (helm/kernels/__init__.py:40-46:
-O3 -ffast-math -fopenmp) except -march=native, replaced by the explicit
-mavx2 -mf16c -mfma the kernel needs, so that the module runs on any AVX2 host.
The compiler is /usr/bin/g++ (the image's default g++ lacks libgomp.spec).
"""
from __future__ import annotations

import os
import pathlib
import subprocess
import sys
import sysconfig

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"
# Root of the HELM checkout whose fp16_gemv.cpp is compiled; required to (re)build the module.
_ROOT_ENV = os.environ.get("HELM_REFERENCE_ROOT")
REF_ROOT = pathlib.Path(_ROOT_ENV) if _ROOT_ENV else None
REF_SRC = REF_ROOT / "helm" / "kernels" / "fp16_gemv.cpp" if REF_ROOT else None
MODULE = "helm_fp16_gemv_ref"


def module_path() -> pathlib.Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return OUT / (MODULE + suffix)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path | None:
    """Builds the module when the reference source is present; returns its path or None."""
    target = module_path()
    if target.exists() and not force:
        return target
    if REF_SRC is None or not REF_SRC.exists():
        if target.exists():
            return target
        why = ("HELM_REFERENCE_ROOT is not set" if REF_SRC is None
               else f"{REF_SRC} not found")
        print(f"[oracle] reference GEMV not built: {why}", file=sys.stderr)
        return None
    import torch.utils.cpp_extension as ce
    OUT.mkdir(exist_ok=True)
    cxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
    inc = []
    for p in ce.include_paths():
        inc += ["-I", p]
    inc += ["-I", sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths()
    cmd = [cxx, "-O3", "-mavx2", "-mf16c", "-mfma", "-ffast-math", "-fopenmp", "-shared", "-fPIC",
           "-std=c++17", f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-D_GLIBCXX_USE_CXX11_ABI=1", *inc, str(REF_SRC), "-o", str(target)]
    for d in libdirs:
        cmd += ["-L", d, f"-Wl,-rpath,{d}"]
    cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-fopenmp"]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stderr[-4000:])
        raise RuntimeError("building the reference fp16 GEMV failed")
    return target


def load():
    """Imports the built reference module (torch must be importable)."""
    import importlib.util
    import torch  # noqa: F401  (loads libtorch for the extension)
    path = module_path()
    if not path.exists():
        raise RuntimeError(f"reference GEMV module not built: {path}")
    spec = importlib.util.spec_from_file_location(MODULE, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
