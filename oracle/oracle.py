"""CPU oracle for the SpMM hot path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as the checker or the timed CPU
baseline.  The product (``ascend-spmm_b200/``) never imports it and has no CPU
fallback.

Contents
--------
* ``csr_to_bcsr``, ``csr_to_ascend_cube``, ``block_level_split``,
  ``preprocess``: ctypes front-ends over ``spmm_oracle.c``, a plain-C
  restatement of the reference's CPU layout code
  (extension/custom_op.cpp:429-1412, extension/boundary_bucket_sort.h,
  extension/packed_column_reindex.h).  They return the reference's dict keys
  with the reference's dtypes: index arrays follow the input index dtype,
  values follow the input value dtype, ``permutation``/``inv_permutation`` and
  audit counters are int64 and costs float64 (custom_op.cpp:1037-1109).
* ``csr_to_spmm_cube``: the producer of ``spmm_cube``'s window encoding
  (the reference has the consumer only) in ToBCSR's merge order.
* ``spmm_csr_f64`` / ``spmm_mixed_f64`` / ``spmm_cube_f64``: the SpMM semantics of the reference
  kernels (op_kernel/spmm_csr.cpp:383-423; op_kernel/spmm_ascend_cube.cpp:52-165,
  265-288, 782-875; op_kernel/spmm_cube.cpp:51-147) evaluated in float64 on the (already fp16/fp32-rounded)
  inputs - the same construction as the reference's unused
  ``cpu_reference`` (tests/aic_aiv_ablation/common.py:173-177).
* ``neutronsparse_parts_np``: the NeutronSparse partition of the reference's
  Table 6 helpers (tests/task_mapping/common.py:170-229) in NumPy.
* ``cpu_reference``: that reference function restated (torch.sparse.mm in
  fp32), used as the timed CPU baseline of the reference's own CPU path.
* ``make_start``: tests/task_mapping/common.py:119-127 restated.

Parity pin: ``tests/test_oracle_pin.py`` checks every layout function against
the reference's compiled code (``oracle/_ref``) when it is available, and
``tests/test_oracle_golden.py`` against committed fixtures in all cases.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle_spmm.so"
SRC_PATH = HERE / "spmm_oracle.c"


def build(force: bool = False) -> Path:
    """Compile ``spmm_oracle.c`` with gcc (no fast-math: the cost model is
    evaluated in IEEE double exactly as the reference does)."""
    if LIB_PATH.is_file() and not force and LIB_PATH.stat().st_mtime >= SRC_PATH.stat().st_mtime:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
    subprocess.run(
        ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off",
         str(SRC_PATH), "-o", str(tmp), "-lm"],
        check=True,
    )
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


_I64P = ctypes.POINTER(ctypes.c_int64)
_U8P = ctypes.POINTER(ctypes.c_uint8)


class _Layout(ctypes.Structure):
    _fields_ = [
        ("crow_window_ptr", _I64P), ("n_crow", ctypes.c_int64),
        ("unique_col_ids", _I64P), ("n_uniq", ctypes.c_int64),
        ("value", _U8P), ("n_value", ctypes.c_int64),
        ("vrow_window_ptr", _I64P), ("n_vrow", ctypes.c_int64),
        ("vcol_indices", _I64P), ("n_vcol", ctypes.c_int64),
        ("vvalue", _U8P), ("n_vvalue", ctypes.c_int64),
    ]


class _Pre(ctypes.Structure):
    _fields_ = [
        ("fwd", _Layout), ("tr", _Layout),
        ("renumbered_unique_col_ids", _I64P), ("n_ren_uniq", ctypes.c_int64),
        ("renumbered_vcol_indices", _I64P), ("n_ren_vcol", ctypes.c_int64),
        ("permutation", _I64P), ("n_perm", ctypes.c_int64),
        ("inv_permutation", _I64P), ("n_inv", ctypes.c_int64),
        ("packed_rows", ctypes.c_int64),
        ("packed_layout_supported", ctypes.c_int64),
        ("marginal_window", ctypes.c_int64),
        ("marginal_aic_blocks", ctypes.c_int64),
        ("marginal_total_blocks", ctypes.c_int64),
        ("shared_windows", ctypes.c_int64),
        ("estimated_aic_cost", ctypes.c_double),
        ("estimated_aiv_cost", ctypes.c_double),
        ("estimated_max_cost", ctypes.c_double),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        _lib.orc_last_error.restype = ctypes.c_char_p
        common = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _I64P, _I64P,
                  ctypes.c_void_p, ctypes.c_int64]
        _lib.orc_csr_to_bcsr.argtypes = common + [ctypes.c_int64, ctypes.POINTER(_Layout)]
        _lib.orc_csr_to_ascend_cube.argtypes = common + [ctypes.c_int64, ctypes.POINTER(_Layout)]
        _lib.orc_block_level_split.argtypes = common + [ctypes.c_double, ctypes.c_int64,
                                                        ctypes.POINTER(_Layout)]
        _lib.orc_preprocess.argtypes = common + [ctypes.c_int64, ctypes.c_int,
                                                 ctypes.POINTER(_Pre)]
        _lib.orc_free_layout.argtypes = [ctypes.POINTER(_Layout)]
        _lib.orc_free_preprocess.argtypes = [ctypes.POINTER(_Pre)]
        dp = ctypes.POINTER(ctypes.c_double)
        _lib.orc_spmm_csr_f64.argtypes = [ctypes.c_int64, ctypes.c_int64, _I64P, _I64P, dp, dp, dp]
        _lib.orc_spmm_window_f64.argtypes = [ctypes.c_int64, ctypes.c_int64, _I64P, _I64P, dp, dp, dp]
        _lib.orc_spmm_cube_f64.argtypes = [ctypes.c_int64, ctypes.c_int64, _I64P, _I64P, dp, dp, dp]
        _lib.orc_csr_to_spmm_cube.argtypes = common + [ctypes.c_int64, ctypes.POINTER(_Layout)]
    return _lib


# --------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------

def _np(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().contiguous().numpy()
    return np.ascontiguousarray(x)


def _i64(x) -> np.ndarray:
    return np.ascontiguousarray(_np(x).astype(np.int64, copy=False))


def _ptr(a: np.ndarray, ty=_I64P):
    return a.ctypes.data_as(ty)


def _index_dtype(crow) -> torch.dtype:
    if isinstance(crow, torch.Tensor):
        return crow.dtype
    return torch.from_numpy(np.asarray(crow)[:0]).dtype


def _values(values):
    """Return (raw uint8 view, element size, torch dtype) of the values."""
    if isinstance(values, torch.Tensor):
        t = values.detach().cpu().contiguous()
    else:
        t = torch.from_numpy(np.ascontiguousarray(values))
    raw = t.view(torch.uint8).numpy() if t.numel() else np.zeros(0, np.uint8)
    return np.ascontiguousarray(raw), t.element_size(), t.dtype


def _take_i64(p, n, dtype) -> torch.Tensor:
    if n == 0:
        return torch.empty(0, dtype=dtype)
    a = np.ctypeslib.as_array(p, shape=(n,)).copy()
    return torch.from_numpy(a).to(dtype)


def _take_val(p, n, esz, dtype) -> torch.Tensor:
    if n == 0:
        return torch.empty(0, dtype=dtype)
    a = np.ctypeslib.as_array(p, shape=(n * esz,)).copy()
    return torch.from_numpy(a).view(dtype)


def _check(rc):
    if rc != 0:
        raise ValueError(lib().orc_last_error().decode())


def _layout_dict(o: _Layout, idx, esz, vdt, with_v=True) -> dict:
    d = {
        "crow_window_ptr": _take_i64(o.crow_window_ptr, o.n_crow, idx),
        "unique_col_ids": _take_i64(o.unique_col_ids, o.n_uniq, idx),
        "value": _take_val(o.value, o.n_value, esz, vdt),
    }
    if with_v:
        d.update({
            "vrow_window_ptr": _take_i64(o.vrow_window_ptr, o.n_vrow, idx),
            "vcol_indices": _take_i64(o.vcol_indices, o.n_vcol, idx),
            "vvalue": _take_val(o.vvalue, o.n_vvalue, esz, vdt),
        })
    return d


def _prep(crow_ptr, col_indices, values):
    crow = _i64(crow_ptr)
    col = _i64(col_indices)
    raw, esz, vdt = _values(values)
    return crow, col, raw, esz, vdt, _index_dtype(crow_ptr)


# --------------------------------------------------------------------------
# layout functions (reference API, custom_op.cpp:1413-1492)
# --------------------------------------------------------------------------

def csr_to_bcsr(crow_ptr, col_indices, values, nrows, ncols, window_size=16) -> dict:
    crow, col, raw, esz, vdt, idx = _prep(crow_ptr, col_indices, values)
    o = _Layout()
    _check(lib().orc_csr_to_bcsr(nrows, ncols, col.size, _ptr(crow), _ptr(col),
                                 raw.ctypes.data, esz, window_size, ctypes.byref(o)))
    try:
        return _layout_dict(o, idx, esz, vdt, with_v=False)
    finally:
        lib().orc_free_layout(ctypes.byref(o))


def csr_to_ascend_cube(crow_ptr, col_indices, values, nrows, ncols, window_size=16) -> dict:
    crow, col, raw, esz, vdt, idx = _prep(crow_ptr, col_indices, values)
    o = _Layout()
    _check(lib().orc_csr_to_ascend_cube(nrows, ncols, col.size, _ptr(crow), _ptr(col),
                                        raw.ctypes.data, esz, window_size, ctypes.byref(o)))
    try:
        return _layout_dict(o, idx, esz, vdt, with_v=False)
    finally:
        lib().orc_free_layout(ctypes.byref(o))


def block_level_split(crow_ptr, col_indices, values, nrows, ncols, a, window_size=16) -> dict:
    crow, col, raw, esz, vdt, idx = _prep(crow_ptr, col_indices, values)
    o = _Layout()
    _check(lib().orc_block_level_split(nrows, ncols, col.size, _ptr(crow), _ptr(col),
                                       raw.ctypes.data, esz, float(a), window_size,
                                       ctypes.byref(o)))
    try:
        return _layout_dict(o, idx, esz, vdt)
    finally:
        lib().orc_free_layout(ctypes.byref(o))


def csr_to_spmm_cube(crow_ptr, col_indices, values, nrows, ncols, window_size=16) -> dict:
    """Producer of the ``spmm_cube`` input (keys ``rowptr``, ``col``, ``value``):
    per 16-row window the entries in (column, row) order, ``col`` holding
    ``(column << 4) | row``.  The reference ships only the consumer
    (op_kernel/spmm_cube.cpp:51-147); the order is ToBCSR's merge order
    (custom_op.cpp:611-671)."""
    crow, col, raw, esz, vdt, idx = _prep(crow_ptr, col_indices, values)
    o = _Layout()
    _check(lib().orc_csr_to_spmm_cube(nrows, ncols, col.size, _ptr(crow), _ptr(col),
                                      raw.ctypes.data, esz, window_size, ctypes.byref(o)))
    try:
        d = _layout_dict(o, idx, esz, vdt, with_v=False)
        return {"rowptr": d["crow_window_ptr"], "col": d["unique_col_ids"], "value": d["value"]}
    finally:
        lib().orc_free_layout(ctypes.byref(o))


def preprocess(crow_ptr, col_indices, values, nrows, ncols, window_size=16,
               graph_layout=False) -> dict:
    crow, col, raw, esz, vdt, idx = _prep(crow_ptr, col_indices, values)
    o = _Pre()
    _check(lib().orc_preprocess(nrows, ncols, col.size, _ptr(crow), _ptr(col),
                                raw.ctypes.data, esz, window_size, int(bool(graph_layout)),
                                ctypes.byref(o)))
    try:
        d = _layout_dict(o.fwd, idx, esz, vdt)
        d["renumbered_unique_col_ids"] = _take_i64(o.renumbered_unique_col_ids, o.n_ren_uniq, idx)
        d["renumbered_vcol_indices"] = _take_i64(o.renumbered_vcol_indices, o.n_ren_vcol, idx)
        tr = _layout_dict(o.tr, idx, esz, vdt)
        for k, v in tr.items():
            d["transpose_" + k] = v
        d["permutation"] = _take_i64(o.permutation, o.n_perm, torch.int64)
        d["inv_permutation"] = _take_i64(o.inv_permutation, o.n_inv, torch.int64)
        for k in ("packed_rows", "packed_layout_supported", "marginal_window",
                  "marginal_aic_blocks", "marginal_total_blocks", "shared_windows"):
            d[k] = torch.tensor([getattr(o, k)], dtype=torch.int64)
        for k in ("estimated_aic_cost", "estimated_aiv_cost", "estimated_max_cost"):
            d[k] = torch.tensor([getattr(o, k)], dtype=torch.float64)
        return d
    finally:
        lib().orc_free_preprocess(ctypes.byref(o))


# --------------------------------------------------------------------------
# SpMM semantics
# --------------------------------------------------------------------------

def _f64(x) -> np.ndarray:
    return np.ascontiguousarray(_np(x).astype(np.float64))


def spmm_csr_f64(rowptr, col, value, dense) -> np.ndarray:
    """y = A @ B in float64 (op_kernel/spmm_csr.cpp:383-423 semantics)."""
    crow, c = _i64(rowptr), _i64(col)
    v, B = _f64(value), _f64(dense)
    nrows, n = crow.size - 1, B.shape[1]
    y = np.zeros((nrows, n), np.float64)
    dp = ctypes.POINTER(ctypes.c_double)
    lib().orc_spmm_csr_f64(nrows, n, _ptr(crow), _ptr(c), _ptr(v, dp), _ptr(B, dp), _ptr(y, dp))
    return y


def spmm_mixed_f64(Crowptr, Ccol_ids, Cvalue, Vrowptr, Vcol_ids, Vvalue, dense) -> np.ndarray:
    """Output of ``spmm_ascend_cube`` in float64.

    Rows = max(16 * #windows, #V rows) (custom_op.cpp:146); window slot s adds
    its (16 x 1)-block products to rows [16s, 16s + 16)
    (op_kernel/spmm_ascend_cube.cpp:52-165, 265-288) and the CSR part adds to
    its own rows (op_kernel/spmm_ascend_cube.cpp:782-875); both contributions
    are summed.
    """
    cptr, ccol, cval = _i64(Crowptr), _i64(Ccol_ids), _f64(Cvalue)
    vptr, vcol, vval = _i64(Vrowptr), _i64(Vcol_ids), _f64(Vvalue)
    B = _f64(dense)
    nwin, vrows, n = cptr.size - 1, vptr.size - 1, B.shape[1]
    rows = max(16 * nwin, vrows)
    y = np.zeros((rows, n), np.float64)
    dp = ctypes.POINTER(ctypes.c_double)
    lib().orc_spmm_window_f64(nwin, n, _ptr(cptr), _ptr(ccol), _ptr(cval, dp), _ptr(B, dp),
                              _ptr(y, dp))
    if vrows > 0:
        yv = np.zeros((vrows, n), np.float64)
        lib().orc_spmm_csr_f64(vrows, n, _ptr(vptr), _ptr(vcol), _ptr(vval, dp), _ptr(B, dp),
                               _ptr(yv, dp))
        y[:vrows] += yv
    return y


def spmm_cube_f64(rowptr, col, value, dense) -> np.ndarray:
    """Output of ``spmm_cube`` in float64 ([16 * #windows, N]): runs of equal
    column inside a window form one (16 x 1) block, the last entry of a row in
    a run wins (op_kernel/spmm_cube.cpp:51-147)."""
    rp, c, v, B = _i64(rowptr), _i64(col), _f64(value), _f64(dense)
    nwin, n = rp.size - 1, B.shape[1]
    y = np.zeros((16 * nwin, n), np.float64)
    dp = ctypes.POINTER(ctypes.c_double)
    lib().orc_spmm_cube_f64(nwin, n, _ptr(rp), _ptr(c), _ptr(v, dp), _ptr(B, dp), _ptr(y, dp))
    return y


def spmm_ascend_cube_tiles_f64(crow_window_ptr, unique_col_ids, value, dense) -> np.ndarray:
    """SpMM over the 16 x 16 tiles of ``csr_to_ascend_cube`` in float64
    ([16 * #windows, N]): y[16 w + r] = sum over the window's tiles t and
    k < 16 of value[256 t + 16 r + k] * B[unique_col_ids[16 t + k]]
    (tile layout of custom_op.cpp:429-592; padding entries are literal
    zeros of column 0)."""
    tp, c, v, B = _i64(crow_window_ptr), _i64(unique_col_ids), _f64(value), _f64(dense)
    nwin, n = tp.size - 1, B.shape[1]
    y = np.zeros((16 * nwin, n), np.float64)
    for w in range(nwin):
        for t in range(int(tp[w]), int(tp[w + 1])):
            tile = v[256 * t: 256 * t + 256].reshape(16, 16)        # [row, k]
            y[16 * w: 16 * w + 16] += tile @ B[c[16 * t: 16 * t + 16]]
    return y


def neutronsparse_parts_np(crow, col, rows, cols, assume_symmetric=False, threshold=None):
    """tests/task_mapping/common.py:170-229 restated in NumPy (the
    reference's own formulation): returns (window mask, window row counts,
    CSR row counts, dense-row count, dense-column count)."""
    indptr = _i64(crow)
    columns = _i64(col)
    row_degree = np.diff(indptr).astype(np.int64)
    if assume_symmetric and rows == cols:
        column_degree = row_degree.copy()
    else:
        column_degree = np.bincount(columns, minlength=cols).astype(np.int64)
    edge_dense_column = (column_degree > threshold)[columns]
    row_dense_degree = np.zeros(rows, dtype=np.int64)
    nonempty = row_degree > 0
    if nonempty.any():
        row_dense_degree[nonempty] = np.add.reduceat(edge_dense_column, indptr[:-1][nonempty], dtype=np.int64)
    dense_row = row_dense_degree > threshold
    mask = np.logical_and(edge_dense_column, np.repeat(dense_row, row_degree))
    cube_counts = np.where(dense_row, row_dense_degree, 0)
    return mask, cube_counts, row_degree - cube_counts, int(dense_row.sum()), int((column_degree > threshold).sum())


def cpu_reference(rows, cols, crow, col, values, dense) -> torch.Tensor:
    """tests/aic_aiv_ablation/common.py:173-177 restated: torch.sparse.mm in fp32."""
    matrix = torch.sparse_csr_tensor(crow, col, values.float(), size=(rows, cols),
                                     check_invariants=False)
    return torch.sparse.mm(matrix, dense.float())


def make_start(pointer: torch.Tensor, cores: int) -> torch.Tensor:
    """tests/task_mapping/common.py:119-127 restated."""
    total = int(pointer[-1]) if pointer.numel() else 0
    if total <= 0:
        return torch.zeros(cores, dtype=torch.int32)
    chunk = (total + cores - 1) // cores
    targets = torch.arange(cores, dtype=torch.int64) * chunk
    return (torch.searchsorted(pointer.to(torch.int64), targets, right=True) - 1
            ).clamp_min(0).to(torch.int32)


def tolerance(dtype: torch.dtype) -> tuple[float, float]:
    """(atol, rtol) of tests/task_mapping/correctness.py:140-143."""
    return (2e-2, 2e-2) if dtype == torch.float16 else (1e-4, 1e-4)


__all__ = [
    "build", "csr_to_bcsr", "csr_to_ascend_cube", "block_level_split", "preprocess",
    "csr_to_spmm_cube", "spmm_csr_f64", "spmm_mixed_f64", "spmm_cube_f64", "spmm_ascend_cube_tiles_f64", "neutronsparse_parts_np", "cpu_reference", "make_start", "tolerance",
]
