"""CPU checks of the drop-in boundary: the C-ABI library loads and exports
every entry point include/spmm_b200.h declares; the torch-facing module
imports and exposes the reference's operator names.  No compute (no GPU)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "ascend-spmm_b200"


def declared_functions():
    text = (ROOT / "include" / "spmm_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spmm_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import build

    build.build_lib()
    return ctypes.CDLL(str(build.LIB))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("spmm_csr_launch", "spmm_ascend_cube_launch", "spmm_csr_workspace_bytes",
              "spmm_device_status", "spmm_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_workspace_queries(lib):
    assert lib.spmm_abi_version() == 1
    lib.spmm_csr_workspace_bytes.restype = ctypes.c_size_t
    lib.spmm_csr_workspace_bytes.argtypes = [ctypes.c_int64] * 3 + [ctypes.c_int]
    # two fp32 partial rows of N=128 per unit, then one int64 per unit
    # boundary.  163840 nonzeros: units of 64 (small matrices), 2560 units
    assert lib.spmm_csr_workspace_bytes(16384, 128, 163840, 0) == 2560 * 2 * 128 * 4 + 2561 * 8
    # 2^22 nonzeros: units of 256, 16384 units
    assert lib.spmm_csr_workspace_bytes(1 << 18, 128, 1 << 22, 0) == 16384 * 2 * 128 * 4 + 16385 * 8


def test_argument_errors_need_no_gpu(lib):
    """Contract violations are rejected on the host with the reference's text."""
    lib.spmm_csr_launch.restype = ctypes.c_int
    lib.spmm_last_error.restype = ctypes.c_char_p
    V = ctypes.c_void_p
    i64 = ctypes.c_int64
    lib.spmm_csr_launch.argtypes = [V, V, V, V, V, i64, V, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int,
                                    V, ctypes.c_size_t, V]
    rc = lib.spmm_csr_launch(None, None, None, None, None, 0, None, 4, 4, 24, 0, 0, 0, None, 0, None)
    assert rc == 1
    assert b"feature width divisible by 16, but got 24" in lib.spmm_last_error()
    rc = lib.spmm_csr_launch(None, None, None, None, None, 0, None, 4, 4, 1040, 0, 0, 0, None, 0, None)
    assert rc == 1 and b"0 < feature width <= 1024 for FP16" in lib.spmm_last_error()


def test_torch_module_exposes_reference_names():
    import build

    build.build()
    import spmm_npu

    for name in ("block_level_split", "csr_to_ascend_cube", "csr_to_bcsr", "pack_node_tensor", "preprocess",
                 "restore_node_tensor", "spmm_ascend_cube", "spmm_ascend_cube_aic_without_pipeline",
                 "spmm_ascend_cube_aiv_mb", "spmm_csr", "spmm_csr_aiv_mb_batch", "spmm_cube"):
        assert name in spmm_npu.__all__


def test_operators_reject_cpu_tensors():
    import torch

    import spmm_npu

    x = torch.zeros(2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="must be CUDA tensor"):
        spmm_npu.spmm_csr(x, x[:0], torch.zeros(0, dtype=torch.float16), torch.zeros(4, 16, dtype=torch.float16), x)


def test_l2_plan_reserved_only_for_large_problems_with_wide_rows(lib, monkeypatch):
    # default (auto): 1 KB rows and at least 2^26 nonzeros; nothing else pays
    # for the plan's workspace
    monkeypatch.delenv("SPMM_B200_L2PLAN", raising=False)
    lib.spmm_csr_l2_plan_offset.restype = ctypes.c_size_t
    lib.spmm_csr_l2_plan_offset.argtypes = [ctypes.c_int64] * 3 + [ctypes.c_int]
    lib.spmm_csr_workspace_bytes.restype = ctypes.c_size_t
    lib.spmm_csr_workspace_bytes.argtypes = [ctypes.c_int64] * 3 + [ctypes.c_int]
    none = ctypes.c_size_t(-1).value
    for N, nnz, dt in ((512, 1 << 20, 0), (128, 1 << 27, 0), (256, 1 << 20, 1), (128, 1 << 27, 1)):
        assert lib.spmm_csr_l2_plan_offset(1 << 16, N, nnz, dt) == none
    for N, nnz, dt in ((1024, 1 << 27, 0), (256, 1 << 26, 1)):
        off = lib.spmm_csr_l2_plan_offset(1 << 16, N, nnz, dt)
        total = lib.spmm_csr_workspace_bytes(1 << 16, N, nnz, dt)
        assert off != none and off % 256 == 0 and total - off > (1 << 26)
    monkeypatch.setenv("SPMM_B200_L2PLAN", "off")
    assert lib.spmm_csr_l2_plan_offset(1 << 16, 1024, 1 << 27, 0) == none
    monkeypatch.setenv("SPMM_B200_L2PLAN", "on")
    assert lib.spmm_csr_l2_plan_offset(1 << 16, 512, 1 << 10, 0) != none
    assert lib.spmm_csr_l2_plan_offset(1 << 16, 256, 1 << 10, 0) == none   # 512-byte rows: never
