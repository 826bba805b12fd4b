"""Build recipe for ``oracle/_ref``: the reference's own CPU preprocessing.

TEST INFRASTRUCTURE ONLY.  The product never imports, links or runs anything
built here; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may use it, and only as a checker or as the timed CPU
baseline.

What is built: the reference's ``extension/custom_op.cpp`` compiled
unmodified, straight from the read-only reference tree, with g++ against the
CPU build of torch.  No reference source is copied into this repository.

* ``custom_op.cpp`` includes ``../common/pytorch_npu_helper.hpp``, which needs
  torch_npu and the CANN runtime.  Its include guard ``PYTORCH_NPU_HELPER_HPP_``
  is predefined so the body is skipped, and ``oracle/ref_shim.h`` is
  force-included to stand in for the one macro the file uses from it
  (``EXEC_NPU_CMD``, pytorch_npu_helper.hpp:516-581) with an error.
* The resulting pybind module (``ref_custom_ops_lib``) exports the reference's
  ``preprocess``, ``csr_to_bcsr``, ``csr_to_ascend_cube`` and
  ``block_level_split`` (custom_op.cpp:1413-1492), which run on CPU tensors.
  Its NPU operators raise if called.

The recipe needs the reference source tree.  Its location comes from the
environment variable ``ASCEND_SPMM_REFERENCE``, else from the
``reference_path`` entry of the repository's ``BASELINE.json`` (the record of
where the reference checkout of this build lives).  When neither names an
existing tree (e.g. on a GPU box) the build is skipped and an already-built
``oracle/_ref`` is used as is.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
MODULE = "ref_custom_ops_lib"


def reference_root() -> Path | None:
    """The reference source tree, or None when no location is recorded."""
    env = os.environ.get("ASCEND_SPMM_REFERENCE")
    if env:
        return Path(env)
    try:
        import json

        recorded = json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
    except (OSError, ValueError):
        recorded = None
    return Path(recorded) if recorded else None


def built_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return OUT_DIR / f"{MODULE}{suffix}"


def build(force: bool = False, verbose: bool = False) -> Path | None:
    """Compile the reference preprocessing into ``oracle/_ref``.

    Returns the path of the built module, or None when neither the reference
    tree nor a previous build is available.
    """
    out = built_path()
    root = reference_root()
    src = root / "extension" / "custom_op.cpp" if root is not None else None
    if src is None or not src.is_file():
        return out if out.is_file() else None
    if out.is_file() and not force and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    import torch
    from torch.utils import cpp_extension

    OUT_DIR.mkdir(parents=True, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        "g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        f"-DTORCH_EXTENSION_NAME={MODULE}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        "-DPYTORCH_NPU_HELPER_HPP_",
        "-include", str(HERE / "ref_shim.h"),
    ]
    for inc in cpp_extension.include_paths():
        cmd += ["-isystem", inc]
    cmd += ["-isystem", sysconfig.get_paths()["include"]]
    cmd += [str(src), "-o", str(out)]
    for lib in cpp_extension.library_paths():
        cmd += [f"-L{lib}", f"-Wl,-rpath,{lib}"]
    cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


def load():
    """Import the built reference module (building it first if possible)."""
    path = build()
    if path is None or not path.is_file():
        return None
    import importlib.util

    import torch  # noqa: F401  (loads libtorch before the extension)

    spec = importlib.util.spec_from_file_location(MODULE, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True)
    print(p if p else "reference tree not found; nothing built")
