"""Build recipe for the reference's own DeepSeek-V4 CUDA kernels, as a test-only oracle.

    python oracle/build_ref.py [--force]

Compiles exfold/deepseek_v4/csrc/exfold_kernels.cu from the reference checkout at
/root/reference (or $EXFOLD_REFERENCE), where it lies, with the flags of the reference's own
build script (exfold/deepseek_v4/csrc/build.py:17: -O3 --use_fast_math -lineinfo, plus the
flags torch.utils.cpp_extension adds to every CUDA source) for sm_100a, and links it with
oracle/ref_dsv4_binding.cpp into the Python module oracle/_ref/exfold_ref_dsv4.so.  Outputs go to
oracle/_ref/ only (git-ignored; the built module travels with the tree to a GPU machine, where
the reference checkout is absent).  Without the reference checkout nothing is built.

The module is a checker for tests/test_gpu_reference_dsv4.py.  Nothing in the product loads it.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
MODULE = OUT_DIR / "exfold_ref_dsv4.so"
BINDING = HERE / "ref_dsv4_binding.cpp"
REFERENCE = Path(os.environ.get("EXFOLD_REFERENCE", "/root/reference"))
KERNELS = REFERENCE / "exfold" / "deepseek_v4" / "csrc" / "exfold_kernels.cu"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
REFERENCE_CUDA_FLAGS = ["-O3", "--use_fast_math", "-lineinfo"]  # build.py:17


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def available() -> bool:
    return KERNELS.is_file()


def build(force: bool = False, verbose: bool = False) -> Path | None:
    """Build the module if the reference checkout is present; returns its path (or None)."""
    if not available():
        return MODULE if MODULE.is_file() else None
    deps = [KERNELS, BINDING, Path(__file__)]
    if (not force and MODULE.is_file()
            and MODULE.stat().st_mtime >= max(d.stat().st_mtime for d in deps)):
        return MODULE
    import torch
    from torch.utils import cpp_extension as ext

    OUT_DIR.mkdir(parents=True, exist_ok=True)
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"
    defs = ["-DTORCH_EXTENSION_NAME=exfold_ref_dsv4", "-DTORCH_API_INCLUDE_EXTENSION_H", abi]
    incs = [f"-I{p}" for p in ext.include_paths(device_type="cuda")]
    incs.append(f"-I{sysconfig.get_paths()['include']}")
    kobj = OUT_DIR / "exfold_kernels.o"
    bobj = OUT_DIR / "ref_dsv4_binding.o"
    cmds = [
        [_nvcc(), *ARCH, *REFERENCE_CUDA_FLAGS, *ext.COMMON_NVCC_FLAGS, "-std=c++17",
         "-Xcompiler", "-fPIC", *defs, *incs, "-c", str(KERNELS), "-o", str(kobj)],
        ["g++", "-O3", "-std=c++17", "-fPIC", *defs, *incs, "-c", str(BINDING), "-o", str(bobj)],
    ]
    libs = [f"-L{p}" for p in ext.library_paths(device_type="cuda")]
    rpath = [f"-Wl,-rpath,{p}" for p in ext.library_paths(device_type="cuda")]
    cmds.append(["g++", "-shared", "-o", str(MODULE), str(kobj), str(bobj), *libs, *rpath,
                 "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
                 "-ltorch_python", "-lcudart"])
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"reference build failed:\n{' '.join(cmd)}\n{res.stdout}\n"
                               f"{res.stderr}")
    kobj.unlink()
    bobj.unlink()
    return MODULE


def load():
    """Import the built module (torch first, for its symbols); None if it was not built."""
    if not MODULE.is_file():
        return None
    import importlib.util

    import torch  # noqa: F401

    spec = importlib.util.spec_from_file_location("exfold_ref_dsv4", MODULE)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    path = build(force=a.force, verbose=True)
    print(path if path else "reference checkout not found: nothing built", file=sys.stdout)
