"""In-tree build of the engine.

* ``libspmm_b200.so``  - the CUDA kernels and the C ABI of include/spmm_b200.h,
  compiled by nvcc for sm_100a only.
* ``custom_ops_lib<EXT_SUFFIX>`` - the torch-facing pybind module with the
  reference's operator names (extension/custom_op.cpp:1413-1492), a thin
  C++ layer that validates tensors and calls the C ABI.

Both land next to this file so they travel with the repository snapshot.
Objects go to ``_build/`` (git-ignored).  Rebuilds are incremental on file
modification times.  ``python build.py [--force]``.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
INCLUDE = ROOT / "include"
LIB = PKG / "libspmm_b200.so"
EXT = PKG / f"custom_ops_lib{sysconfig.get_config_var('EXT_SUFFIX') or '.so'}"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              f"-I{INCLUDE}"]

CU_SOURCES = ["status.cu", "gather.cu", "gather_mma.cu", "window.cu", "window_warp.cu", "window_tc.cu", "rows.cu", "cube.cu", "preprocess.cu", "noalloc.cu", "l2plan.cu", "capi.cu"]
HEADERS = ["common.cuh", "engine.h"]


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_lib(force=False, verbose=False) -> Path:
    OBJ.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / "spmm_b200.h"]
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = OBJ / (s.stem + ".o")
        if force or _newer(o, [s, *headers]):
            _run([NVCC, *ARCH, *NVCC_FLAGS, "-c", s, "-o", o], verbose)
        objs.append(o)
    if force or _newer(LIB, objs):
        tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC", *objs, "-o", tmp],
             verbose)
        os.replace(tmp, LIB)
    return LIB


def build_ext(force=False, verbose=False) -> Path:
    src = PKG / "host" / "custom_ops_lib.cpp"
    if not (force or _newer(EXT, [src, LIB, INCLUDE / "spmm_b200.h"])):
        return EXT
    import torch
    from torch.utils import cpp_extension

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=custom_ops_lib",
           "-DTORCH_API_INCLUDE_EXTENSION_H", f"-I{INCLUDE}", f"-isystem{CUDA_HOME / 'include'}"]
    for inc in cpp_extension.include_paths():
        cmd += ["-isystem", inc]
    cmd += ["-isystem", sysconfig.get_paths()["include"]]
    tmp = EXT.with_suffix(f".tmp{os.getpid()}.so")
    cmd += [src, "-o", tmp, f"-L{PKG}", "-lspmm_b200", "-Wl,-rpath,$ORIGIN"]
    for lib in cpp_extension.library_paths():
        cmd += [f"-L{lib}", f"-Wl,-rpath,{lib}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    _run(cmd, verbose)
    os.replace(tmp, EXT)
    return EXT


def build(force=False, verbose=False):
    build_lib(force, verbose)
    build_ext(force, verbose)
    return LIB, EXT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
