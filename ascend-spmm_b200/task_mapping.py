"""Task-mapping methods of the reference's Table 6 comparison, on the GPU.

The reference compares four ways of splitting a CSR matrix between its
matrix cores (window layout) and vector cores (CSR rows), all consumed by
``spmm_ascend_cube`` (tests/task_mapping/common.py:19-28, 286-331):

* ``ours``          - ``preprocess`` (the cost-model task mapping);
* ``block-split``   - ``block_level_split`` with ratio (222/190) * 0.5;
* ``naive``         - the first nnz/3 nonzeros to the window part
                      (common.py:264-283);
* ``neutronsparse`` - dense columns (degree above a threshold) inside dense
                      rows to the window part (common.py:146-229, threshold
                      rule of NeutronSparseLite's SplitStrategy, :146-158).

Here every method produces the same dict of CUDA tensors and every step runs
on the device: the layout builders are this engine's GPU kernels, and the two
extra partitioners are written with device tensor operations (degree counts,
prefix sums, masks and compaction) instead of the reference's NumPy.  The
on-disk CSR payload format of the reference's tests (``.pt`` with ``shape``,
``crow_indices``, ``col_indices``; tests/data/prepare_data.py:24-43) is read
by ``load_payload`` with the reference's validation messages
(common.py:33-63) and written by ``convert_matrix``.
"""

from __future__ import annotations

import hashlib
import math
from pathlib import Path
from typing import Dict, Optional, Tuple

import torch

import spmm_npu

AIC_CORES = 20
AIV_CORES = 40
WINDOW_SIZE = 16
METHODS = ("ours", "naive", "neutronsparse", "block-split")
METHOD_LABELS = {
    "ours": "Ascend-SpMM task mapping",
    "naive": "Naive load balancing",
    "neutronsparse": "NeutronSparse load balancing",
    "block-split": "Block-Level split",
}
DEFAULT_BLOCK_RATIO = (222.0 / 190.0) * 0.5
DEFAULT_NAIVE_FRACTION = 1.0 / 3.0


# --------------------------------------------------------------------------
# CSR payload files
# --------------------------------------------------------------------------

def load_payload(path: Path):
    """Read a CSR structure file; returns (name, rows, cols, crow, col) with
    int64 index tensors (common.py:33-63, same checks and messages)."""
    path = Path(path)
    try:
        payload = torch.load(path, map_location="cpu", weights_only=True)
    except TypeError:
        payload = torch.load(path, map_location="cpu")
    required = {"shape", "crow_indices", "col_indices"}
    missing = sorted(required.difference(payload))
    if missing:
        raise ValueError(f"missing payload fields: {', '.join(missing)}")
    rows, cols = map(int, payload["shape"])
    crow = payload["crow_indices"].to(torch.int64).contiguous()
    col = payload["col_indices"].to(torch.int64).contiguous()
    if rows <= 0 or cols <= 0:
        raise ValueError(f"invalid matrix shape: {(rows, cols)}")
    if crow.ndim != 1 or crow.numel() != rows + 1:
        raise ValueError("crow_indices must contain rows + 1 entries")
    if col.ndim != 1 or int(crow[0]) != 0 or int(crow[-1]) != col.numel():
        raise ValueError("invalid CSR pointer or column array")
    if bool((crow[1:] < crow[:-1]).any().item()):
        raise ValueError("crow_indices must be nondecreasing")
    if not col.numel():
        raise ValueError("empty matrices are not supported")
    if int(col.min()) < 0 or int(col.max()) >= cols:
        raise ValueError("col_indices contains an out-of-range index")
    if max(rows, cols, col.numel()) > torch.iinfo(torch.int32).max:
        raise ValueError("matrix exceeds the 32-bit NPU index contract")
    if "nnz" in payload and int(payload["nnz"]) != col.numel():
        raise ValueError("payload nnz does not match col_indices")
    fallback = path.stem[:-4] if path.stem.endswith("_csr") else path.stem
    name = str(payload.get("name") or fallback)
    return name, rows, cols, crow, col


def save_payload(destination: Path, name: str, rows: int, cols: int, crow, col) -> None:
    """Write a CSR structure file in the reference's payload format."""
    destination = Path(destination)
    destination.parent.mkdir(parents=True, exist_ok=True)
    torch.save({"name": name, "shape": (int(rows), int(cols)), "nnz": int(col.numel()),
                "crow_indices": crow.detach().cpu().to(torch.int64).contiguous(),
                "col_indices": col.detach().cpu().to(torch.int64).contiguous()}, destination)


def convert_matrix(source: Path, destination: Path):
    """Matrix Market file -> payload: duplicates summed, explicit zeros
    dropped, rows sorted (tests/data/prepare_data.py:24-43).  Returns
    (rows, cols, nnz)."""
    import numpy as np
    from scipy import sparse
    from scipy.io import mmread

    matrix = mmread(str(source))
    if not sparse.issparse(matrix):
        matrix = sparse.coo_matrix(np.asarray(matrix))
    csr = matrix.tocsr(copy=False)
    csr.sum_duplicates()
    csr.eliminate_zeros()
    csr.sort_indices()
    rows, cols = csr.shape
    save_payload(destination, Path(source).stem, rows, cols,
                 torch.from_numpy(csr.indptr.astype(np.int64)), torch.from_numpy(csr.indices.astype(np.int64)))
    return rows, cols, csr.nnz


def discover_datasets(dataset_dir: Path, name: str = "", index: Optional[int] = None, start: int = 0,
                      stop: Optional[int] = None, limit: Optional[int] = None):
    """Sorted ``*.pt`` files under dataset_dir with the reference's filters
    (common.py:66-100)."""
    dataset_dir = Path(dataset_dir)
    paths = sorted(dataset_dir.rglob("*.pt"), key=lambda item: item.relative_to(dataset_dir).as_posix())
    if name:
        paths = [p for p in paths if name == p.parent.name or name in p.stem]
    if index is not None:
        if index < 0 or index >= len(paths):
            raise ValueError(f"--index {index} is outside the discovered range [0, {len(paths)})")
        return [paths[index]]
    if start < 0:
        raise ValueError("--start must be non-negative")
    if stop is not None and stop < start:
        raise ValueError("--stop must be greater than or equal to --start")
    paths = paths[start:stop]
    if limit is not None:
        if limit <= 0:
            raise ValueError("--limit must be positive")
        paths = paths[:limit]
    if not paths:
        raise ValueError(f"no .pt datasets selected under {dataset_dir}")
    return paths


def stable_seed(base_seed: int, relative_path: str) -> int:
    """Per-dataset seed (common.py:114-116)."""
    digest = hashlib.sha256(relative_path.encode("utf-8")).digest()
    return (base_seed + int.from_bytes(digest[:8], "little")) % (2**63 - 1)


def make_values(nnz: int, dtype: torch.dtype, seed: int) -> torch.Tensor:
    """U[-1, 1] values (common.py:133-135)."""
    generator = torch.Generator().manual_seed(seed)
    return (torch.rand(nnz, generator=generator) * 2 - 1).to(dtype).contiguous()


def make_dense(cols: int, dim: int, dtype: torch.dtype, seed: int) -> torch.Tensor:
    """U[-1, 1] dense operand (common.py:138-143)."""
    generator = torch.Generator().manual_seed(seed)
    return (torch.rand((cols, dim), generator=generator) * 2 - 1).to(dtype).contiguous()


def make_start(pointer: torch.Tensor, cores: int) -> torch.Tensor:
    """Per-core first row (common.py:119-127); the engine accepts and
    ignores these arrays, they are built for API compatibility."""
    total = int(pointer[-1]) if pointer.numel() else 0
    if total <= 0:
        return torch.zeros(cores, dtype=torch.int32, device=pointer.device)
    chunk = (total + cores - 1) // cores
    targets = torch.arange(cores, dtype=torch.int64, device=pointer.device) * chunk
    return (torch.searchsorted(pointer.to(torch.int64), targets, right=True) - 1).clamp_min(0).to(torch.int32)


# --------------------------------------------------------------------------
# partitioners
# --------------------------------------------------------------------------

def compute_neutronsparse_threshold(rows: int, cols: int, nnz: int) -> int:
    """Dense-degree threshold of NeutronSparseLite's SplitStrategy
    (common.py:146-158, same constants and branch order)."""
    if rows == 0:
        return 32
    average_degree = nnz / rows
    sparsity = nnz / (rows * cols) if rows * cols else 0.0
    if sparsity < 0.0002:
        alpha = 1.8 if rows > 1_000_000 else 1.0
    elif sparsity > 0.01:
        alpha = 0.25
    else:
        alpha = 0.55
    return max(4, int(average_degree * alpha))


def _ptr_from_counts(counts: torch.Tensor) -> torch.Tensor:
    ptr = torch.zeros(counts.numel() + 1, dtype=torch.int64, device=counts.device)
    torch.cumsum(counts.to(torch.int64), 0, out=ptr[1:])
    return ptr


def neutronsparse_parts(crow, col, values, rows: int, cols: int, assume_symmetric: bool = False):
    """Dense columns (column degree > threshold) inside dense rows (more than
    threshold dense-column entries) go to the window part, everything else to
    the CSR part (common.py:170-229).  Returns ((crow, col, values) window
    part, (crow, col, values) CSR part, metadata); both parts keep the
    original row count and CSR order."""
    crow64 = crow.to(torch.int64)
    nnz = col.numel()
    row_degree = crow64[1:] - crow64[:-1]
    if assume_symmetric and rows == cols:
        column_degree = row_degree.clone()
    else:
        column_degree = torch.bincount(col.to(torch.int64), minlength=cols)
    threshold = compute_neutronsparse_threshold(rows, cols, nnz)
    dense_column = column_degree > threshold
    edge_dense_column = dense_column[col.to(torch.int64)]
    # dense-column entries per row: a prefix sum read at the row bounds
    prefix = _ptr_from_counts(edge_dense_column)
    row_dense_degree = prefix[crow64[1:]] - prefix[crow64[:-1]]
    dense_row = row_dense_degree > threshold
    edge_dense_row = torch.repeat_interleave(dense_row, row_degree, output_size=nnz)
    cube_mask = edge_dense_column & edge_dense_row
    vector_mask = ~cube_mask
    cube_counts = torch.where(dense_row, row_dense_degree, torch.zeros_like(row_dense_degree))
    vector_counts = row_degree - cube_counts
    idt = crow.dtype
    cube = (_ptr_from_counts(cube_counts).to(idt), col[cube_mask].contiguous(), values[cube_mask].contiguous())
    vector = (_ptr_from_counts(vector_counts).to(idt), col[vector_mask].contiguous(),
              values[vector_mask].contiguous())
    metadata = {
        "threshold": threshold,
        "assume_symmetric": bool(assume_symmetric),
        "symmetry_shortcut_used": bool(assume_symmetric and rows == cols),
        "dense_rows": int(dense_row.sum()),
        "dense_columns": int(dense_column.sum()),
        "aic_nnz": int(cube_mask.sum()),
        "aiv_nnz": int(vector_mask.sum()),
    }
    return cube, vector, metadata


def naive_parts(crow, col, values, rows: int, fraction: float):
    """The first pivot nonzeros (nnz / 3 by default) to the window part
    (common.py:264-283)."""
    nnz = col.numel()
    pivot = nnz // 3 if math.isclose(fraction, 1.0 / 3.0) else int(nnz * fraction)
    pivot = max(0, min(nnz, pivot))
    cube = (crow.clamp_max(pivot).contiguous(), col[:pivot].contiguous(), values[:pivot].contiguous())
    vector = ((crow - pivot).clamp_min(0).contiguous(), col[pivot:].contiguous(), values[pivot:].contiguous())
    metadata = {"fraction": fraction, "pivot_nnz": pivot, "aic_nnz": pivot, "aiv_nnz": nnz - pivot}
    return cube, vector, metadata


def _empty_window(index_dtype, value_dtype, device):
    return {"crow_window_ptr": torch.zeros(1, dtype=index_dtype, device=device),
            "unique_col_ids": torch.empty(0, dtype=index_dtype, device=device),
            "value": torch.empty(0, dtype=value_dtype, device=device)}


def _pack_window(crow, col, values, cols: int, device):
    """Window layout of the window part, rows trimmed after the last
    nonempty one (common.py:241-249)."""
    if col.numel() == 0:
        return _empty_window(crow.dtype, values.dtype, device)
    counts = crow[1:] - crow[:-1]
    nonempty = torch.nonzero(counts > 0, as_tuple=False).flatten()
    if not nonempty.numel():
        return _empty_window(crow.dtype, values.dtype, device)
    packed_rows = int(nonempty[-1]) + 1
    trimmed = crow[:packed_rows + 1].contiguous()
    if int(trimmed[-1]) != col.numel():
        raise ValueError("cube CSR contains edges after its last nonempty row")
    return spmm_npu.csr_to_bcsr(trimmed, col.contiguous(), values.contiguous(), packed_rows, cols, WINDOW_SIZE)


def _combine(cube, vector, cols: int, device):
    packed = _pack_window(*cube, cols, device)
    vcrow, vcol, vval = vector
    return {
        "crow_window_ptr": packed["crow_window_ptr"].to(device).contiguous(),
        "unique_col_ids": packed["unique_col_ids"].to(device).contiguous(),
        "value": packed["value"].to(device).contiguous(),
        "vrow_window_ptr": vcrow.to(device).contiguous(),
        "vcol_indices": vcol.to(device).contiguous(),
        "vvalue": vval.to(device).contiguous(),
    }


def prepare_partition(method: str, rows: int, cols: int, crow: torch.Tensor, col: torch.Tensor,
                      values: torch.Tensor, block_ratio: float = DEFAULT_BLOCK_RATIO,
                      naive_fraction: float = DEFAULT_NAIVE_FRACTION, assume_symmetric: bool = False,
                      device=None) -> Tuple[Dict[str, torch.Tensor], dict]:
    """One Table 6 method -> (window/CSR mapping for spmm_ascend_cube,
    metadata), with the reference's argument checks (common.py:286-331).
    Inputs may live on the CPU or a GPU; the mapping lives on ``device``
    (default: the current CUDA device)."""
    if method not in METHODS:
        raise ValueError(f"unknown partition method: {method}")
    if block_ratio <= 0:
        raise ValueError("block_ratio must be positive")
    if not 0.0 <= naive_fraction <= 1.0:
        raise ValueError("naive_fraction must be in [0, 1]")
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    crow, col, values = crow.to(device), col.to(device), values.to(device)
    nnz = col.numel()
    if method == "ours":
        mapping = spmm_npu.preprocess(crow, col, values, rows, cols, WINDOW_SIZE)
        aiv = int(mapping["vcol_indices"].numel())
        metadata = {"aic_nnz": nnz - aiv, "aiv_nnz": aiv, "aic_blocks": int(mapping["unique_col_ids"].numel())}
    elif method == "block-split":
        mapping = spmm_npu.block_level_split(crow, col, values, rows, cols, block_ratio, WINDOW_SIZE)
        aiv = int(mapping["vcol_indices"].numel())
        metadata = {"ratio": block_ratio, "aic_nnz": nnz - aiv, "aiv_nnz": aiv,
                    "aic_blocks": int(mapping["unique_col_ids"].numel())}
    elif method == "neutronsparse":
        cube, vector, metadata = neutronsparse_parts(crow, col, values, rows, cols, assume_symmetric)
        mapping = _combine(cube, vector, cols, device)
    else:
        cube, vector, metadata = naive_parts(crow, col, values, rows, naive_fraction)
        mapping = _combine(cube, vector, cols, device)
    required = {"crow_window_ptr", "unique_col_ids", "value", "vrow_window_ptr", "vcol_indices", "vvalue"}
    missing = sorted(required.difference(mapping))
    if missing:
        raise ValueError(f"partition mapping is missing: {', '.join(missing)}")
    if metadata["aic_nnz"] + metadata["aiv_nnz"] != nnz:
        raise ValueError("partition does not preserve the original NNZ count")
    return mapping, {"method": method, "label": METHOD_LABELS[method], **metadata}


def build_mixed_invoker(mapping: Dict[str, torch.Tensor], dense: torch.Tensor):
    """Closure running spmm_ascend_cube on a mapping (common.py:334-347)."""
    dev = dense.device if dense.is_cuda else torch.device("cuda", torch.cuda.current_device())
    to_dev = lambda t, dt=None: t.to(device=dev, dtype=dt or t.dtype).contiguous()  # noqa: E731
    args = (
        to_dev(mapping["crow_window_ptr"], torch.int32), to_dev(mapping["unique_col_ids"], torch.int32),
        to_dev(mapping["value"]), to_dev(mapping["vrow_window_ptr"], torch.int32),
        to_dev(mapping["vcol_indices"], torch.int32), to_dev(mapping["vvalue"]), to_dev(dense),
        to_dev(make_start(mapping["crow_window_ptr"].cpu(), AIC_CORES)),
        to_dev(make_start(mapping["vrow_window_ptr"].cpu(), AIV_CORES)),
    )
    return lambda: spmm_npu.spmm_ascend_cube(*args)


def build_reference_invoker(crow, col, values, dense):
    """Closure running spmm_csr, the reference point of every method
    (common.py:350-364)."""
    dev = dense.device if dense.is_cuda else torch.device("cuda", torch.cuda.current_device())
    to_dev = lambda t, dt=None: t.to(device=dev, dtype=dt or t.dtype).contiguous()  # noqa: E731
    args = (to_dev(crow, torch.int32), to_dev(col, torch.int32), to_dev(values), to_dev(dense),
            to_dev(make_start(crow.cpu(), AIV_CORES)))
    return lambda: spmm_npu.spmm_csr(*args)


__all__ = [
    "AIC_CORES", "AIV_CORES", "WINDOW_SIZE", "METHODS", "METHOD_LABELS", "DEFAULT_BLOCK_RATIO",
    "DEFAULT_NAIVE_FRACTION", "load_payload", "save_payload", "convert_matrix", "discover_datasets",
    "stable_seed", "make_values", "make_dense", "make_start", "compute_neutronsparse_threshold",
    "neutronsparse_parts", "naive_parts", "prepare_partition", "build_mixed_invoker", "build_reference_invoker",
]
